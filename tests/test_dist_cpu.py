"""Multi-rank host logic on CPU (gloo, two ranks).

Each rank reduces its row block of a global X[2*8, 16, 32] (the benchmark's
layout and seeded offsets) with the oracle and combines the results with
quasarml_b200.sharding.ExchangePlan, the plan bench.py drives through the
library: binary32 partials packed into one flat buffer per combine group,
sums added, max/min combined as order-preserving 32-bit keys (the mapping
qsml_allreduce_partials uses, restated here in NumPy), means finished from
the combined sum as sum * (1/n).  Rank 1's block holds a NaN and rank 0's a
column of -0 beside +0, so the combine must keep NaN propagation and -0 < +0.
The result must match the oracle on the unsharded tensor: max/min bit for
bit, sums within 1e-5 * sum|x|, axis-1/2 row blocks exactly.  Also checks the
row split of the library (qsml_shard_rows, host code) against its restatement.
"""
import os
import socket
import sys

import numpy as np
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


def shard_of(rank):
    from quasarml_b200 import datagen, sharding
    n = int(np.prod(SHARD))
    x = datagen.normal(4, SHARD, 0.0, 1.0, offset=sharding.shard_offset(0, WORLD, rank, n))
    if rank == 1:
        x[3, 5, 7] = np.nan
    else:
        x[:, 2, 9] = 0.0
        x[::2, 2, 9] = -0.0
    return x


def keys(v, is_max):
    """Order-preserving unsigned keys of binary32 values (NaN largest for
    max, smallest for min), as int64 for gloo."""
    u = np.ascontiguousarray(v, dtype=np.float32).view(np.uint32).astype(np.int64)
    k = np.where(u & 0x80000000, (~u) & 0xFFFFFFFF, u | 0x80000000)
    nan = (u & 0x7FFFFFFF) > 0x7F800000
    return np.where(nan, 0xFFFFFFFF if is_max else 0, k)


def values(k, is_max):
    nan = k == (0xFFFFFFFF if is_max else 0)
    u = np.where(k & 0x80000000, k & 0x7FFFFFFF, (~k) & 0xFFFFFFFF)
    u = np.where(nan, 0x7FFFFFFF, u)
    return u.astype(np.uint32).view(np.float32)


def _rank(rank, port, q):
    sys.path.insert(0, ROOT)
    import torch
    import torch.distributed as dist
    from oracle import qsml_oracle as orc
    from quasarml_b200 import sharding

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=WORLD)
    try:
        x = shard_of(rank)
        glob_rows = WORLD * SHARD[0]
        plan = sharding.ExchangePlan()
        calls = []
        local = {}
        for axis in (None, 0, 1, 2):
            for op in (sharding.SUM, sharding.MEAN, sharding.MAX, sharding.MIN):
                if sharding.needs_exchange(axis):
                    count = 1 if axis is None else int(np.prod(SHARD[1:]))
                    n = glob_rows * (int(np.prod(SHARD[1:])) if axis is None else 1)
                    calls.append(((axis, op), plan.add("X", op, axis, count, n)))
                else:
                    local[(axis, op)] = orc.reduce(op, x, axis)[0].astype(np.float32).reshape(-1)
        flat = {g: np.zeros(sz, np.float32) for g, sz in plan.sizes.items()}
        for key, axis, group, off, count in plan.partials:
            op = {"sum": sharding.SUM, "max": sharding.MAX, "min": sharding.MIN}[group]
            flat[group][off:off + count] = orc.reduce(op, x, axis)[0].astype(np.float32).reshape(-1)
        # the combine qsml_allreduce_partials performs
        t = torch.from_numpy(flat["sum"])
        dist.all_reduce(t, op=dist.ReduceOp.SUM)
        for g, is_max in (("max", True), ("min", False)):
            kt = torch.from_numpy(keys(flat[g], is_max))
            dist.all_reduce(kt, op=dist.ReduceOp.MAX if is_max else dist.ReduceOp.MIN)
            flat[g] = values(kt.numpy(), is_max)
        out = {}
        for (axis, op), i in calls:
            fop, group, off, count, n, idx = plan.finishes[i]
            assert idx == i and fop == op
            p = flat[group][off:off + count]
            # qsml_finish_partial: a mean is sum * (1.0f / (float)n)
            out[(axis, op)] = p * np.float32(1.0 / np.float32(n)) if op == sharding.MEAN else p.copy()
        for k, v in local.items():
            parts = [torch.zeros(v.size) for _ in range(WORLD)]
            dist.all_gather(parts, torch.from_numpy(v))
            out[k] = torch.cat(parts).numpy()
        if rank == 0:
            q.put(out)
    finally:
        dist.destroy_process_group()


def test_two_rank_sharded_reductions_match_unsharded(orc):
    from quasarml_b200 import sharding
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
    glob = np.concatenate([shard_of(r) for r in range(WORLD)])
    for (axis, op), got in out.items():
        o32, o64, ab = orc.reduce(op, glob, axis)
        if op in (sharding.MAX, sharding.MIN):
            want = o32.astype(np.float32).reshape(-1)
            gn, wn = np.isnan(got), np.isnan(want)
            assert np.array_equal(gn, wn), (axis, op)
            assert np.array_equal(got[~gn].view(np.uint32), want[~wn].view(np.uint32)), (axis, op)
        else:
            want, scale = o64.reshape(-1), ab.reshape(-1)
            gn, wn = np.isnan(got), np.isnan(want)
            assert np.array_equal(gn, wn), (axis, op)
            assert np.all(np.abs(got[~gn].astype(np.float64) - want[~wn]) <= 1e-5 * scale[~wn] + 1e-30), (axis, op)
    # the NaN reached the outputs that reduce over it, and -0 < +0 held
    assert np.isnan(out[(None, sharding.MAX)]).all()


def test_row_split_matches_the_library():
    from quasarml_b200 import abi, sharding
    for rows in (0, 1, 7, 64, 2729, 8192, 16387):
        for world in (1, 2, 3, 4, 8):
            covered = 0
            for r in range(world):
                b, c = abi.shard_rows(rows, world, r)
                assert (b, c) == sharding.shard_rows(rows, world, r)
                assert b == covered
                covered += c
            assert covered == rows
