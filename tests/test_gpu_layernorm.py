"""GPU layer norm (through the C ABI) against the oracle's binary64 result.

Tolerance (ref = the binary64 result rounded once to the output dtype):
|y - ref| <= bar * max(|ref|, 0.1), i.e. bar relative wherever |ref| >= 0.1
and an absolute floor of bar * 0.1 for outputs nearer zero (where a relative
bound would only measure the cancellation of (x - mean) * rstd * gamma
against beta); bar = 1e-5 for binary32 and 1e-3 for binary16."""
import numpy as np
import pytest

from helpers import d, dev, empty, host
from quasarml_b200 import abi, datagen

pytestmark = pytest.mark.gpu


def run(ctx, x, g, b, eps=1e-5):
    tx, tg, tb = dev(x), dev(g), dev(b)
    y = empty(x.shape, x.dtype)
    ctx.layer_norm(d(tx), d(tg), d(tb), eps, d(y))
    return host(y)


def assert_close(y, ref, tol):
    y64, r64 = y.astype(np.float64), ref.astype(np.float64)
    err = np.abs(y64 - r64)
    worst = np.max(err / (tol * np.maximum(np.abs(r64), 0.1)))
    big = np.abs(r64) >= 0.1
    rel = float(np.max(err[big] / np.abs(r64[big]))) if np.any(big) else 0.0
    print(f"max relative error where |y| >= 0.1: {rel:.3g}; worst {worst:.3g} x tolerance (bar {tol:g})")
    assert worst <= 1.0, f"error {worst:.3g} x tolerance"


@pytest.mark.parametrize("dtype", ["f32", "f16"])
def test_workload_16384x4096(ctx, orc, dtype):
    x = datagen.normal(datagen.SEEDS["ln_X"], (16384, 4096), 0.5, 2.0)
    g = datagen.normal(datagen.SEEDS["ln_gamma"], (4096,), 1.0, 0.1)
    b = datagen.normal(datagen.SEEDS["ln_beta"], (4096,), 0.0, 0.1)
    if dtype == "f16":
        x = x.astype(np.float16)
    y = run(ctx, x, g, b)
    ref = orc.layer_norm(x, g, b, 1e-5)
    assert_close(y, ref, 1e-5 if dtype == "f32" else 1e-3)


@pytest.mark.parametrize("shape", [(7, 96), (3, 5, 128), (64, 1024), (2, 8192), (9, 1000), (4, 33), (1, 16384),
                                   (5, 3)])
@pytest.mark.parametrize("dtype", [np.float32, np.float16])
def test_shapes(ctx, orc, shape, dtype):
    x = datagen.normal(31, shape, 0.5, 2.0).astype(dtype)
    g = datagen.normal(32, shape[-1:], 1.0, 0.1)
    b = datagen.normal(33, shape[-1:], 0.0, 0.1)
    y = run(ctx, x, g, b)
    ref = orc.layer_norm(x, g, b, 1e-5)
    assert_close(y, ref, 1e-5 if dtype == np.float32 else 1e-3)


def test_f16_gamma_beta(ctx, orc):
    x = datagen.normal(34, (16, 256), 0.5, 2.0).astype(np.float16)
    g = datagen.normal(35, (256,), 1.0, 0.1).astype(np.float16)
    b = datagen.normal(36, (256,), 0.0, 0.1).astype(np.float16)
    y = run(ctx, x, g, b)
    ref = orc.layer_norm(x, g.astype(np.float32), b.astype(np.float32), 1e-5)
    assert_close(y, ref, 1e-3)


def test_constant_rows_and_errors(ctx):
    x = np.full((4, 512), 3.0, np.float32)
    y = run(ctx, x, np.ones(512, np.float32), np.full(512, 0.25, np.float32))
    assert np.allclose(y, 0.25)
    with pytest.raises(abi.QsmlError):
        run(ctx, x, np.ones(511, np.float32), np.ones(511, np.float32))
