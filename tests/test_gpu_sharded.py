"""Row-sharded reductions through the C ABI (qsml_reduce_sharded, which runs
qsml_reduce into binary32 partials, qsml_allreduce_partials and
qsml_finish_partial).

One GPU: a single-rank group.  The partial path is the same reduction kernel,
an exact key round trip for max/min and the same sum * (1/n) for mean, so
every result must be bit-identical to qsml_reduce's, binary16 outputs, NaN
and signed zeros included.

Two GPUs (one process each, NVLS off): rank 0 holds 5 rows and rank 1 holds 3
(or none) of a global X[8, 64, 48]; each rank's result must match the oracle
on the whole tensor: max/min bit for bit (a NaN in rank 1's rows must win, -0
must lose to +0 across ranks), sum/mean within 1e-5 * sum|x| (plus one
binary16 rounding for binary16 outputs), axis-1/2 results equal to the
rank's rows of the global result.
"""
import multiprocessing as mp
import os
import sys

import numpy as np
import pytest

from helpers import d, dev, empty, host
from quasarml_b200 import abi, datagen

pytestmark = pytest.mark.gpu
ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
OPS = (abi.RED_SUM, abi.RED_MEAN, abi.RED_MAX, abi.RED_MIN)


def n_gpus():
    import torch
    return torch.cuda.device_count()


def special_x(shape, seed):
    x = datagen.normal(seed, shape, 0.3, 1.5)
    x[..., 3, 7] = 0.0
    x[::2, 3, 7] = -0.0
    return x


@pytest.mark.parametrize("dtype", [np.float32, np.float16])
def test_single_rank_is_bit_identical_to_reduce(ctx, dtype):
    import torch
    g = abi.Group.init_rank(ctx, abi.group_unique_id(), 1, 0)
    try:
        x = special_x((37, 64, 48), 81).astype(dtype)
        x[11, 5, 9] = np.nan
        t = dev(x)
        for axis in (None, 0, 1, 2):
            code = abi.AXIS_ALL if axis is None else axis
            oshape = abi.reduced_shape(x.shape, axis, False)
            for op in OPS:
                want = empty(oshape, dtype)
                ctx.reduce(op, d(t), code, False, d(want))
                got = torch.full(oshape, 7.0, dtype=want.dtype, device="cuda")
                g.reduce_sharded(0, op, d(t), code, False, d(got), 0)
                a, b = host(got), host(want)
                assert np.array_equal(a.view(np.uint8), b.view(np.uint8)), (axis, op)
    finally:
        g.destroy()


def test_shard_rows_partition():
    assert abi.shard_rows(10, 3, 0) == (0, 4)
    assert abi.shard_rows(10, 3, 1) == (4, 3)
    assert abi.shard_rows(10, 3, 2) == (7, 3)
    with pytest.raises(abi.QsmlError):
        abi.shard_rows(10, 3, 3)


SPLITS = {"5+3": (5, 3), "8+0": (8, 0)}


def _rank_main(rank, uid, split, q):
    import torch
    sys.path.insert(0, ROOT)
    sys.path.insert(0, os.path.join(ROOT, "tests"))
    from quasarml_b200 import abi as a
    torch.cuda.set_device(rank)
    ctx = a.Context(rank, use_torch_stream=False)
    g = a.Group.init_rank(ctx, uid, 2, rank)
    try:
        rows = SPLITS[split]
        glob = special_x((8, 64, 48), 82)
        glob[6, 20, 30] = np.nan  # in rank 1's rows under "5+3"
        r0 = sum(rows[:rank])
        res = {}
        for dtype in (np.float32, np.float16):
            x = np.ascontiguousarray(glob[r0:r0 + rows[rank]].astype(dtype))
            t = torch.from_numpy(x).to(f"cuda:{rank}")
            for axis in (None, 0, 1, 2):
                code = a.AXIS_ALL if axis is None else axis
                oshape = a.reduced_shape(x.shape, axis, False)
                for op in (a.RED_SUM, a.RED_MEAN, a.RED_MAX, a.RED_MIN):
                    if rows[rank] == 0 and axis in (1, 2):
                        continue
                    out = torch.empty(oshape, dtype=t.dtype, device=f"cuda:{rank}")
                    torch.cuda.synchronize()
                    g.reduce_sharded(0, op, a.desc_of(t), code, False, a.desc_of(out), 8)
                    ctx.synchronize()
                    res[(np.dtype(dtype).name, axis, op)] = out.cpu().numpy()
        q.put((rank, res))
    except Exception as e:  # the parent reports it
        q.put((rank, repr(e)))
    finally:
        g.destroy()
        ctx.close()


@pytest.mark.skipif(n_gpus() < 2, reason="needs two GPUs")
@pytest.mark.parametrize("split", list(SPLITS))
def test_two_processes_match_the_whole_tensor(orc, split):
    uid = abi.group_unique_id()
    mpc = mp.get_context("spawn")
    q = mpc.Queue()
    env_old = os.environ.get("NCCL_NVLS_ENABLE")
    os.environ["NCCL_NVLS_ENABLE"] = "0"
    try:
        ps = [mpc.Process(target=_rank_main, args=(r, uid, split, q)) for r in range(2)]
        for p in ps:
            p.start()
        got = dict(q.get(timeout=240) for _ in range(2))
        for p in ps:
            p.join(timeout=120)
    finally:
        if env_old is None:
            os.environ.pop("NCCL_NVLS_ENABLE", None)
        else:
            os.environ["NCCL_NVLS_ENABLE"] = env_old
        for p in ps:
            if p.is_alive():
                p.kill()
    rows = SPLITS[split]
    glob = special_x((8, 64, 48), 82)
    glob[6, 20, 30] = np.nan
    for rank in (0, 1):
        assert isinstance(got[rank], dict), got[rank]
        r0 = sum(rows[:rank])
        for (dname, axis, op), out in got[rank].items():
            dtype = np.dtype(dname)
            gx = glob.astype(dtype)
            o32, o64, ab = orc.reduce(op, gx, axis)
            k = gx.size if axis is None else gx.shape[axis]  # elements reduced into each output
            if axis in (1, 2):
                o32, o64, ab = o32[r0:r0 + rows[rank]], o64[r0:r0 + rows[rank]], ab[r0:r0 + rows[rank]]
            out = out.reshape(o32.shape)
            if op in (abi.RED_MAX, abi.RED_MIN):
                want = o32.astype(dtype)
                assert np.array_equal(np.isnan(out), np.isnan(want)), (rank, dname, axis, op)
                ok = ~np.isnan(want)
                assert np.array_equal(out[ok].view(np.uint8), want[ok].view(np.uint8)), (rank, dname, axis, op)
            else:
                g64 = out.astype(np.float64)
                assert np.array_equal(np.isnan(g64), np.isnan(o64)), (rank, dname, axis, op)
                ok = ~np.isnan(o64)
                scale = ab if op == abi.RED_SUM else ab / k
                tol = 1e-5 * scale + 1e-30
                if dtype == np.float16:
                    tol = tol + np.abs(o64) * 2.0 ** -11
                assert np.all(np.abs(g64[ok] - o64[ok]) <= tol[ok]), (rank, dname, axis, op)
    # the NaN in rank 1's rows reached rank 0's full max
    assert np.isnan(got[0][("float32", None, abi.RED_MAX)]).all()
