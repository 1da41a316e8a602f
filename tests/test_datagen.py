"""The seeded generator is deterministic, shard-consistent, matches its NumPy
restatement and has the requested distributions."""
import numpy as np

from quasarml_b200 import datagen


def test_uniform_matches_numpy_restatement():
    for seed in (1, 2, 3, 12345):
        c = datagen.uniform(seed, (5000,), -1.0, 1.0)
        n = datagen.uniform_np(seed, 5000, -1.0, 1.0)
        assert np.array_equal(c, n)


def test_shards_reproduce_global_stream():
    full = datagen.normal(4, (4, 1000), 0.0, 1.0)
    for r in range(4):
        part = datagen.normal(4, (1000,), 0.0, 1.0, offset=r * 1000)
        assert np.array_equal(part, full[r])


def test_distributions():
    u = datagen.uniform(1, (1 << 20,), -1.0, 1.0)
    assert u.min() >= -1.0 and u.max() < 1.0
    assert abs(u.mean()) < 5e-3 and abs(u.var() - 1 / 3) < 5e-3
    g = datagen.normal(10, (1 << 20,), 0.5, 2.0)
    assert abs(g.mean() - 0.5) < 1e-2 and abs(g.std() - 2.0) < 1e-2
    d = datagen.uniform(3, (4096, 1), 0.5, 2.0)
    assert d.min() >= 0.5 and d.max() < 2.0


def test_iota():
    x = datagen.iota_i32((3, 8192))
    assert x[2, 5] == 2 * 8192 + 5
