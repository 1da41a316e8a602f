"""Multi-rank host logic on CPU: two gloo ranks each reduce their shard of a
global X[2*8, 16, 32] (rows split along axis 0, the benchmark's layout and
seeded offsets) with the oracle, combine with quasarml_b200.sharding's plan
(all-reduce of axis-0 / full partials, mean rescaled), and must match the
oracle on the unsharded tensor: sums within 1e-5 * sum|x|, max/min exactly,
axis-1/2 slices exactly."""
import os
import socket
import sys

import numpy as np
import pytest
import torch.multiprocessing as mp

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
SHARD = (8, 16, 32)
WORLD = 2


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


def _rank(rank, port, q):
    sys.path.insert(0, ROOT)
    import torch
    import torch.distributed as dist
    from oracle import qsml_oracle as orc
    from quasarml_b200 import datagen, sharding

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=WORLD)
    try:
        n = int(np.prod(SHARD))
        x = datagen.normal(4, SHARD, 0.0, 1.0, offset=sharding.shard_offset(0, WORLD, rank, n))
        results = {}
        flat = {"sum": [], "mean": [], "max": [], "min": []}
        for axis in (None, 0, 1, 2):
            for op in (sharding.SUM, sharding.MEAN, sharding.MAX, sharding.MIN):
                o32 = orc.reduce(op, x, axis)[0].astype(np.float32).reshape(-1)
                t = torch.from_numpy(o32.copy())
                results[(axis, op)] = t
                if sharding.needs_exchange(axis):
                    flat[sharding.group(op)].append(t)
        # flat buffers per group, as the benchmark lays them out
        bufs, views = {}, []
        for grp, ts in flat.items():
            buf = torch.cat(ts)
            bufs[("f32", grp)] = buf
            off = 0
            for t in ts:
                results_key = next(k for k, v in results.items() if v is t)
                views.append((results_key, buf, off, t.numel()))
                off += t.numel()
        sharding.exchange(dist, bufs, WORLD)
        for (k, buf, off, cnt) in views:
            results[k] = buf[off:off + cnt].clone()
        # gather everything on rank 0 for the comparison
        out = {}
        for k, t in results.items():
            if sharding.needs_exchange(k[0]):
                out[k] = t.numpy()
            else:
                parts = [torch.zeros_like(t) for _ in range(WORLD)]
                dist.all_gather(parts, t)
                out[k] = torch.cat(parts).numpy()
        if rank == 0:
            q.put(out)
    finally:
        dist.destroy_process_group()


def test_two_rank_sharded_reductions_match_unsharded(orc):
    from quasarml_b200 import datagen, sharding
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_rank, args=(r, port, q)) for r in range(WORLD)]
    for p in procs:
        p.start()
    out = q.get(timeout=120)
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    glob = datagen.normal(4, (WORLD * SHARD[0],) + SHARD[1:], 0.0, 1.0)
    for (axis, op), got in out.items():
        o32, o64, ab = orc.reduce(op, glob, axis)
        want = o64.reshape(-1)
        if op in (sharding.MAX, sharding.MIN):
            assert np.array_equal(got, o32.reshape(-1)), (axis, op)
        else:
            scale = ab.reshape(-1)
            assert np.all(np.abs(got.astype(np.float64) - want) <= 1e-5 * scale + 1e-30), (axis, op)
