"""Multi-GPU groups (qsml_group_* / qsml_allreduce, NCCL).

On one GPU: single-rank groups of both kinds (all-reduce is the identity,
MEAN included) and the failure path -- a rank that never joins makes
qsml_group_init_rank return QSML_E_TIMEOUT (run in a child process with a
short QSML_NCCL_TIMEOUT_MS and NVLS off; no GPU kernel is involved, the
missing rank only stalls the bootstrap).  With two GPUs: one process driving
both (start/end bracket) and two processes with one GPU each.
"""
import multiprocessing as mp
import os
import subprocess
import sys
import textwrap

import numpy as np
import pytest

from helpers import dev, host
from quasarml_b200 import abi

pytestmark = pytest.mark.gpu
ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def n_gpus():
    import torch
    return torch.cuda.device_count()


def test_single_rank_groups(ctx):
    x = np.arange(1, 1001, dtype=np.float32)
    for kind in ("all", "rank"):
        g = abi.Group.init_all([ctx]) if kind == "all" else abi.Group.init_rank(ctx, abi.group_unique_id(), 1, 0)
        try:
            assert g.size() == (1, 1)
            for op in (abi.RED_SUM, abi.RED_MEAN, abi.RED_MAX, abi.RED_MIN):
                t = dev(x)
                g.allreduce(0, t.data_ptr(), t.numel(), abi.F32, op)
                np.testing.assert_array_equal(host(t), x)
            with pytest.raises(abi.QsmlError) as e:
                t16 = dev(np.ones(8, np.int16))
                g.allreduce(0, t16.data_ptr(), 8, abi.I16, abi.RED_SUM)
            assert e.value.status == abi.E_DTYPE
        finally:
            g.destroy()


def test_missing_rank_times_out():
    code = textwrap.dedent("""
        import sys, time
        sys.path.insert(0, %r)
        from quasarml_b200 import abi
        ctx = abi.Context(0, use_torch_stream=False)
        uid = abi.group_unique_id()
        t0 = time.time()
        try:
            abi.Group.init_rank(ctx, uid, 2, 0)
            print("JOINED")
        except abi.QsmlError as e:
            print("STATUS", e.status, round(time.time() - t0, 1))
        ctx.close()
    """ % ROOT)
    env = dict(os.environ, QSML_NCCL_TIMEOUT_MS="3000", NCCL_NVLS_ENABLE="0")
    r = subprocess.run([sys.executable, "-c", code], env=env, capture_output=True, text=True, timeout=120)
    lines = [l for l in r.stdout.splitlines() if l.startswith(("STATUS", "JOINED"))]
    assert lines and lines[-1].split()[:2] == ["STATUS", str(abi.E_TIMEOUT)], (r.stdout, r.stderr[-2000:])
    assert float(lines[-1].split()[2]) < 60


@pytest.mark.skipif(n_gpus() < 2, reason="needs two GPUs")
def test_two_gpus_one_process():
    import torch
    ctxs = [abi.Context(i, use_torch_stream=False) for i in range(2)]
    g = abi.Group.init_all(ctxs)
    try:
        vals = [np.arange(4096, dtype=np.float32) * (i + 1) for i in range(2)]
        ts = [torch.from_numpy(v).to(f"cuda:{i}") for i, v in enumerate(vals)]
        torch.cuda.synchronize(0)
        torch.cuda.synchronize(1)
        for op, ref in ((abi.RED_SUM, vals[0] + vals[1]), (abi.RED_MAX, np.maximum(vals[0], vals[1]))):
            bufs = [t.clone() for t in ts]
            for i in range(2):
                torch.cuda.synchronize(i)
            abi.group_start()
            for i in range(2):
                g.allreduce(i, bufs[i].data_ptr(), bufs[i].numel(), abi.F32, op)
            abi.group_end()
            for i in range(2):
                ctxs[i].synchronize()
                np.testing.assert_array_equal(bufs[i].cpu().numpy(), ref)
    finally:
        g.destroy()
        for c in ctxs:
            c.close()


@pytest.mark.skipif(n_gpus() < 2, reason="needs two GPUs")
def test_partials_in_one_group_bracket():
    """The three partial combines of a sharded step (sum, max, min) issued
    inside one group bracket, as bench.py does: max/min keys are decoded
    after the bracket closes; results equal the binary32 sum and the IEEE
    754-2019 maximum/minimum (NaN wins as 0x7fffffff, -0 < +0)."""
    import torch
    ctxs = [abi.Context(i, use_torch_stream=False) for i in range(2)]
    g = abi.Group.init_all(ctxs)
    try:
        rng = np.random.default_rng(5)
        vals = [rng.normal(0, 1, 4099).astype(np.float32) for _ in range(2)]
        vals[0][:4] = [np.nan, -0.0, 0.0, 1.0]
        vals[1][:4] = [2.0, 0.0, -0.0, np.nan]
        bufs = {op: [torch.from_numpy(v.copy()).to(f"cuda:{i}") for i, v in enumerate(vals)]
                for op in (abi.RED_SUM, abi.RED_MAX, abi.RED_MIN)}
        for i in range(2):
            torch.cuda.synchronize(i)
        abi.group_start()
        try:
            for op, bs in bufs.items():
                for i in range(2):
                    g.allreduce_partials(i, op, bs[i].data_ptr(), bs[i].numel())
        finally:
            abi.group_end()
        for c in ctxs:
            c.synchronize()
        nan = np.array([0x7fffffff], np.uint32).view(np.float32)[0]
        want_max = np.maximum(vals[0], vals[1])
        want_min = np.minimum(vals[0], vals[1])
        for w in (want_max, want_min):
            w[np.isnan(w)] = nan
        want_max[1:3] = [0.0, 0.0]
        want_min[1:3] = [-0.0, -0.0]
        for i in range(2):
            np.testing.assert_array_equal(bufs[abi.RED_SUM][i].cpu().numpy(), vals[0] + vals[1])
            assert np.array_equal(bufs[abi.RED_MAX][i].cpu().numpy().view(np.uint32), want_max.view(np.uint32))
            assert np.array_equal(bufs[abi.RED_MIN][i].cpu().numpy().view(np.uint32), want_min.view(np.uint32))
    finally:
        g.destroy()
        for c in ctxs:
            c.close()


def _rank_main(rank, uid, q):
    import torch
    sys.path.insert(0, ROOT)
    from quasarml_b200 import abi as a
    torch.cuda.set_device(rank)
    ctx = a.Context(rank, use_torch_stream=False)
    g = a.Group.init_rank(ctx, uid, 2, rank)
    t = torch.full((1 << 20,), float(rank + 1), device=f"cuda:{rank}")
    torch.cuda.synchronize()
    g.allreduce(0, t.data_ptr(), t.numel(), a.F32, a.RED_MEAN)
    ctx.synchronize()
    q.put((rank, float(t[0].item()), float(t[-1].item())))
    g.destroy()
    ctx.close()


@pytest.mark.skipif(n_gpus() < 2, reason="needs two GPUs")
def test_two_processes():
    uid = abi.group_unique_id()
    mpc = mp.get_context("spawn")
    q = mpc.Queue()
    env_old = os.environ.get("NCCL_NVLS_ENABLE")
    os.environ["NCCL_NVLS_ENABLE"] = "0"
    try:
        ps = [mpc.Process(target=_rank_main, args=(r, uid, q)) for r in range(2)]
        for p in ps:
            p.start()
        for p in ps:
            p.join(timeout=180)
        res = sorted(q.get(timeout=10) for _ in range(2))
    finally:
        if env_old is None:
            os.environ.pop("NCCL_NVLS_ENABLE", None)
        else:
            os.environ["NCCL_NVLS_ENABLE"] = env_old
        for p in ps:
            if p.is_alive():
                p.kill()
    assert res == [(0, 1.5, 1.5), (1, 1.5, 1.5)]
