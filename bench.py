#!/usr/bin/env python
"""Benchmark of the QuasarML B200 backend (libqsml_cuda.so through its C ABI).

Headline workload (N=1 and every N): the reductions configuration --
sum/mean/max/min over axis 0, 1, 2 and all elements of X[64,512,1024] ~ N(0,1),
in fp32 and again with X in fp16 (fp32 accumulation).  One step processes a
batch of 8 distinct X per dtype (1.5 GB of input, so no input is L2-resident
when it is read again), i.e. 256 reduction calls.  Under torchrun each rank
holds its own [64,512,1024] shards of a [64N,512,1024] tensor (weak scaling);
axis-0 and full reductions combine their per-rank partials with NCCL
all-reduces (torch.distributed) that run while the axis-1/2 reductions, which
need no exchange, compute (two CUDA graphs per step, collectives between).

value     : algorithmic bytes (each input read once, each output written once)
            of all ranks / max-over-ranks device time, inputs resident in HBM.
e2e       : the same through the C ABI from pinned host buffers: every step
            copies X host->device and the results device->host inside the
            timed region.
roofline  : the dominant kernel family of the step, its algorithmic bytes per
            launch / its CUDA-event duration, against the measured HBM copy
            bandwidth (MEASURED_PEAKS.json).
cpu_baseline / --impl reference : the oracle's CPU restatement of the same
            reductions (OpenMP over all host cores) on a bounded sample.
other_workloads (N=1): the elementwise chain (op by op and fused), strided
            gathers, layer norm, softmax, argmax/argmin and matmul
            configurations, each timed the same way.
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import sys
import threading
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

import numpy as np  # noqa: E402

METRIC = "HBM GB/s (elementwise, reduce, gather) & matmul TFLOP/s vs roofline, 1–8 GPU"
FALLBACK_HBM_GBS = 6650.0
FALLBACK_BF16_TFLOPS = 1590.0


def peaks():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        j = json.load(open(p))
        return float(j["hbm_gbs"]), float(j["bf16_tflops"]), float(j.get("bf16_tflops_sustained", j["bf16_tflops"])), "measured"
    return FALLBACK_HBM_GBS, FALLBACK_BF16_TFLOPS, 1400.0, "fallback"


def ncu_traffic():
    """DRAM-traffic / algorithmic-bytes ratio of each kernel's committed ncu
    capture (profiles/ncu_traffic.txt: kernel, dram bytes, algorithmic bytes of
    the captured launch)."""
    p = os.path.join(ROOT, "profiles", "ncu_traffic.txt")
    out = {}
    if os.path.exists(p):
        for line in open(p):
            line = line.strip()
            if not line or line.startswith("#"):
                continue
            parts = line.split()
            if len(parts) >= 3:
                out[parts[0]] = float(parts[1]) / float(parts[2])
    return out


# ---------------------------------------------------------------------------
# Clock sampling (NVML, the data nvidia-smi's clocks line reports)
# ---------------------------------------------------------------------------
class ClockSampler:
    REASONS = {0x8: "hw_slowdown", 0x40: "hw_thermal_slowdown", 0x20: "sw_thermal_slowdown",
               0x4: "sw_power_cap", 0x80: "hw_power_brake_slowdown"}

    def __init__(self, index: int, period_s: float = 0.02):
        self.index, self.period = index, period_s
        self.samples, self.reasons, self.max_mhz = [], set(), None
        self._stop = threading.Event()
        self._t = None
        self.error = None

    def __enter__(self):
        try:
            import pynvml
            pynvml.nvmlInit()
            self.nv = pynvml
            self.h = pynvml.nvmlDeviceGetHandleByIndex(self.index)
            self.max_mhz = pynvml.nvmlDeviceGetMaxClockInfo(self.h, pynvml.NVML_CLOCK_SM)
            self._t = threading.Thread(target=self._run, daemon=True)
            self._t.start()
        except Exception as e:  # no NVML: report it, never fake numbers
            self.error = repr(e)
        return self

    def _run(self):
        nv = self.nv
        while not self._stop.is_set():
            try:
                self.samples.append(nv.nvmlDeviceGetClockInfo(self.h, nv.NVML_CLOCK_SM))
                r = nv.nvmlDeviceGetCurrentClocksEventReasons(self.h)
                for bit, name in self.REASONS.items():
                    if r & bit:
                        self.reasons.add(name)
            except Exception as e:
                self.error = repr(e)
                return
            time.sleep(self.period)

    def __exit__(self, *a):
        self._stop.set()
        if self._t:
            self._t.join()

    def summary(self):
        d = {"sm_mhz": statistics.median(self.samples) if self.samples else None,
             "sm_max_mhz": self.max_mhz, "reasons": sorted(self.reasons), "samples": len(self.samples),
             "source": "NVML (nvidia-smi clocks_event_reasons)"}
        if self.error:
            d["error"] = self.error
        return d


# ---------------------------------------------------------------------------
# Distributed plumbing
# ---------------------------------------------------------------------------
class Dist:
    def __init__(self):
        self.world = int(os.environ.get("WORLD_SIZE", "1"))
        self.rank = int(os.environ.get("RANK", "0"))
        self.local = int(os.environ.get("LOCAL_RANK", "0"))
        self.pg = None

    def init(self, backend="nccl"):
        if self.world > 1:
            import datetime
            import torch.distributed as dist
            os.environ.setdefault("MASTER_ADDR", "127.0.0.1")
            dist.init_process_group(backend, timeout=datetime.timedelta(seconds=120))
            self.pg = dist

    def barrier(self):
        if self.pg:
            import torch
            self.pg.barrier(device_ids=[torch.cuda.current_device()]) if self.pg.get_backend() == "nccl" else self.pg.barrier()

    def max(self, v: float) -> float:
        if not self.pg:
            return v
        import torch
        t = torch.tensor([v], dtype=torch.float64, device="cuda")
        self.pg.all_reduce(t, op=self.pg.ReduceOp.MAX)
        return float(t.item())

    def close(self):
        if self.pg:
            self.pg.destroy_process_group()


# ---------------------------------------------------------------------------
# Workloads
# ---------------------------------------------------------------------------
class Workload:
    """A step = compute() (the kernel calls, captured once in a CUDA graph)
    followed by exchange() (collectives between ranks, issued eagerly)."""
    calls = []

    def exchange(self):
        pass

    def step(self):
        self.compute()
        self.exchange()


def _t(x):
    import torch
    return torch.from_numpy(np.ascontiguousarray(x)).cuda()


class ReduceWorkload(Workload):
    """sum/mean/max/min over axis 0, 1, 2, all of X[64,512,1024], fp32 + fp16."""
    name = "reductions X[64,512,1024] fp32 and fp16: sum/mean/max/min over axis 0, 1, 2 and all"
    SHAPE = (64, 512, 1024)

    def __init__(self, ctx, dist: Dist, batch: int = 8):
        import torch
        from quasarml_b200 import abi, datagen, sharding
        self.ctx, self.dist, self.batch, self.abi = ctx, dist, batch, abi
        n = int(np.prod(self.SHAPE))
        self.x32, self.x16 = [], []
        host = np.empty(self.SHAPE, np.float32)
        for b in range(batch):
            datagen.normal(datagen.SEEDS["red_X"], self.SHAPE, 0.0, 1.0,
                           offset=sharding.shard_offset(b, dist.world, dist.rank, n), out=host)
            t = _t(host)
            self.x32.append(t)
            self.x16.append(t.half())
        torch.cuda.synchronize()
        self.ops = [abi.RED_SUM, abi.RED_MEAN, abi.RED_MAX, abi.RED_MIN]
        self.axes = [None, 0, 1, 2]
        # Output buffers: the exchanged ones (axis None / 0) live in one flat
        # buffer per (dtype, combine op) so each step all-reduces few buffers.
        self.calls = []       # (op, x, axis, out_tensor, family, bytes)
        self.flat = {}        # (dtype, 'sum'|'max'|'min') -> flat tensor
        self.bytes_per_step = 0
        for dt, xs in (("f32", self.x32), ("f16", self.x16)):
            tdt = torch.float32 if dt == "f32" else torch.float16
            es = 4 if dt == "f32" else 2
            sizes = {"sum": 0, "mean": 0, "max": 0, "min": 0}
            # batch entry innermost: consecutive calls read different X, and a
            # given X is read again only after the other seven (>= 448 MB), so
            # no call finds its input in L2
            plan = []
            for axis in self.axes:
                oshape = abi.reduced_shape(self.SHAPE, axis, False)
                on = int(np.prod(oshape))
                for op in self.ops:
                    grp = sharding.group(op)
                    exch = sharding.needs_exchange(axis)
                    for b in range(batch):
                        plan.append((b, axis, op, oshape, on, grp, exch))
                        if exch:
                            sizes[grp] += on
            for g, sz in sizes.items():
                self.flat[(dt, g)] = torch.empty(max(sz, 1), dtype=tdt, device="cuda")
            offs = {g: 0 for g in sizes}
            for (b, axis, op, oshape, on, grp, exch) in plan:
                if exch:
                    out = self.flat[(dt, grp)][offs[grp]:offs[grp] + on].view(oshape)
                    offs[grp] += on
                else:
                    out = torch.empty(oshape, dtype=tdt, device="cuda")
                fam = "k_reduce_seg" if axis is None else ("k_reduce_rows" if axis == 2 else "k_reduce_cols")
                nbytes = n * es + on * es
                self.calls.append((op, abi.desc_of(xs[b]), abi.AXIS_ALL if axis is None else axis,
                                   abi.desc_of(out), fam, nbytes, out))
                self.bytes_per_step += nbytes
        self.units_per_step = self.bytes_per_step
        self.unit = "GB/s"
        self.flat_desc = {k: abi.desc_of(v) for k, v in self.flat.items()}
        self.h2d_bytes = sum(x.numel() * 4 for x in self.x32) + sum(x.numel() * 2 for x in self.x16)
        self.d2h_bytes = sum(c[6].numel() * c[6].element_size() for c in self.calls)

    def compute(self, calls=None):
        ctx = self.ctx
        for (op, xd, axis, od, fam, nb, out) in (self.calls if calls is None else calls):
            ctx.reduce(op, xd, axis, False, od)

    def exchange(self):
        self.exchange_finish(self.exchange_start())

    # Overlapped step: the exchanged reductions (axis 0 and full) first, their
    # all-reduces started, the local ones (axes 1, 2) while NCCL runs, then
    # the wait and the mean rescale.
    @property
    def calls_x(self):
        return [c for c in self.calls if c[2] in (0, self.abi.AXIS_ALL)]

    @property
    def calls_l(self):
        return [c for c in self.calls if c[2] not in (0, self.abi.AXIS_ALL)]

    def exchange_start(self):
        if not self.dist.pg:
            return []
        from quasarml_b200 import sharding
        return sharding.exchange_start(self.dist.pg, self.flat)

    def exchange_finish(self, works):
        if not self.dist.pg:
            return
        from quasarml_b200 import sharding
        abi, ctx = self.abi, self.ctx
        sharding.exchange_finish(works, self.flat, self.dist.world,
                                 scale_fn=lambda key, f: ctx.binary_scalar(abi.OP_MUL, self.flat_desc[key], f,
                                                                            self.flat_desc[key]))

    def step(self):
        if not self.dist.pg:
            self.compute()
            return
        self.compute(self.calls_x)
        works = self.exchange_start()
        self.compute(self.calls_l)
        self.exchange_finish(works)

    # End-to-end: host -> device copies of X, the reductions, results back.
    # The uploads run on a second library context (its own stream, a copy
    # engine) one batch entry at a time; the reductions of entry b start as
    # soon as its X has landed (an event per entry), so compute overlaps the
    # PCIe transfers of the entries after it.
    def e2e_setup(self):
        import torch
        from quasarml_b200 import abi
        self.h32 = [x.cpu().pin_memory() for x in self.x32]
        self.h16 = [x.cpu().pin_memory() for x in self.x16]
        self.hout = [c[6].cpu().pin_memory() for c in self.calls]
        self.copy_stream = torch.cuda.Stream()
        self.copy_ctx = abi.Context(torch.cuda.current_device())
        self.copy_ctx.set_stream(self.copy_stream.cuda_stream)
        self.back_stream = torch.cuda.Stream()
        self.back_ctx = abi.Context(torch.cuda.current_device())
        self.back_ctx.set_stream(self.back_stream.cuda_stream)
        self.landed = [torch.cuda.Event() for _ in range(self.batch)]
        self.reduced = [torch.cuda.Event() for _ in range(self.batch)]
        self.calls_by_entry = [[i for i, c in enumerate(self.calls) if self._entry(c) == b] for b in range(self.batch)]

    def _entry(self, call):
        ptr = call[1].data
        for b in range(self.batch):
            if ptr in (self.x32[b].data_ptr(), self.x16[b].data_ptr()):
                return b
        raise ValueError("call input is not one of the batch entries")

    def e2e_step(self):
        import torch
        cur = torch.cuda.current_stream()
        self.copy_stream.wait_stream(cur)  # the previous step has read X
        for b in range(self.batch):
            self.copy_ctx.h2d(self.x32[b].data_ptr(), self.h32[b].data_ptr(), self.h32[b].numel() * 4)
            self.copy_ctx.h2d(self.x16[b].data_ptr(), self.h16[b].data_ptr(), self.h16[b].numel() * 2)
            self.landed[b].record(self.copy_stream)
        # Results travel back on a third stream as each entry finishes (the
        # other PCIe direction), except the exchanged ones at N > 1, which are
        # read after the all-reduces.
        exchanged = set()
        if self.dist.pg:
            exchanged = {i for i, c in enumerate(self.calls) if c[2] in (0, self.abi.AXIS_ALL)}
        for b in range(self.batch):
            cur.wait_event(self.landed[b])
            self.compute([self.calls[i] for i in self.calls_by_entry[b]])
            self.reduced[b].record(cur)
            self.back_stream.wait_event(self.reduced[b])
            for i in self.calls_by_entry[b]:
                if i not in exchanged:
                    out = self.calls[i][6]
                    self.back_ctx.d2h(self.hout[i].data_ptr(), out.data_ptr(), out.numel() * out.element_size(),
                                      sync=False)
        if self.dist.pg:
            self.exchange_finish(self.exchange_start())
            for i in sorted(exchanged):
                out = self.calls[i][6]
                self.ctx.d2h(self.hout[i].data_ptr(), out.data_ptr(), out.numel() * out.element_size(), sync=False)
        cur.wait_stream(self.back_stream)


class ChainWorkload(Workload):
    """relu(pow((A+B)*B - A, 2) / D), A[4096,4096], B[1,4096], D[4096,1]."""
    name = "elementwise chain relu(pow((A+B)*B - A, 2.0) / D), A[4096,4096], B[1,4096], D[4096,1] fp32"

    def __init__(self, ctx, dist: Dist, batch: int = 4):
        import torch
        from quasarml_b200 import abi, datagen
        self.ctx, self.abi = ctx, abi
        N = 4096 * 4096
        self.sets = []
        for b in range(batch):
            A = _t(datagen.uniform(datagen.SEEDS["ew_A"], (4096, 4096), -1, 1, offset=(b * dist.world + dist.rank) * N))
            B = _t(datagen.uniform(datagen.SEEDS["ew_B"], (1, 4096), -1, 1))
            D = _t(datagen.uniform(datagen.SEEDS["ew_D"], (4096, 1), 0.5, 2, offset=(b * dist.world + dist.rank) * 4096))
            ts = [torch.empty((4096, 4096), device="cuda") for _ in range(6)]
            self.sets.append((A, B, D, ts))
        d = abi.desc_of
        self.calls = []
        for A, B, D, t in self.sets:
            self.calls += [("bin", abi.OP_ADD, d(A), d(B), d(t[0]), 134234112),
                           ("bin", abi.OP_MUL, d(t[0]), d(B), d(t[1]), 134234112),
                           ("bin", abi.OP_SUB, d(t[1]), d(A), d(t[2]), 201326592),
                           ("scal", abi.OP_POW, d(t[2]), 2.0, d(t[3]), 134217728),
                           ("bin", abi.OP_DIV, d(t[3]), d(D), d(t[4]), 134234112),
                           ("un", abi.UN_RELU, d(t[4]), None, d(t[5]), 134217728)]
        self.units_per_step = sum(c[5] for c in self.calls)
        self.unit = "GB/s"

    def compute(self, calls=None):
        ctx = self.ctx
        for kind, op, a, b, out, _ in (self.calls if calls is None else calls):
            if kind == "bin":
                ctx.binary(op, a, b, out)
            elif kind == "scal":
                ctx.binary_scalar(op, a, b, out)
            else:
                ctx.unary(op, a, out)


class FusedChainWorkload(Workload):
    """The same chain as ChainWorkload in one qsml_elementwise_fused call per
    set; algorithmic bytes = read A, B, D once + write the result."""
    name = ("elementwise chain relu(pow((A+B)*B - A, 2.0) / D) fused into one kernel, A[4096,4096], B[1,4096], "
            "D[4096,1] fp32")

    def __init__(self, ctx, dist: Dist, batch: int = 4):
        import torch
        from quasarml_b200 import abi, datagen
        self.ctx = ctx
        N = 4096 * 4096
        e = abi.Expr()
        a, b, dd = e.input(0), e.input(1), e.input(2)
        t = e.binary(abi.OP_SUB, e.binary(abi.OP_MUL, e.binary(abi.OP_ADD, a, b), b), a)
        e.unary(abi.UN_RELU, e.binary(abi.OP_DIV, e.binary(abi.OP_POW, t, e.const(2.0)), dd))
        self.nodes = (abi.FuseNode * len(e.nodes))(*[abi.FuseNode(*n) for n in e.nodes])
        self.keep, self.calls = [], []
        d = abi.desc_of
        for bi in range(batch):
            off = (bi * dist.world + dist.rank)
            A = _t(datagen.uniform(datagen.SEEDS["ew_A"], (4096, 4096), -1, 1, offset=off * N))
            B = _t(datagen.uniform(datagen.SEEDS["ew_B"], (1, 4096), -1, 1))
            D = _t(datagen.uniform(datagen.SEEDS["ew_D"], (4096, 1), 0.5, 2, offset=off * 4096))
            out = torch.empty((4096, 4096), device="cuda")
            self.keep += [A, B, D, out]
            self.calls.append(([d(A), d(B), d(D)], d(out), 2 * N * 4 + 2 * 4096 * 4))
        self.units_per_step = sum(c[2] for c in self.calls)
        self.unit = "GB/s"

    def compute(self, calls=None):
        for ins, out, _ in (self.calls if calls is None else calls):
            self.ctx.elementwise_fused(self.nodes, ins, out)


class GatherWorkload(Workload):
    name = "strided gather X[5::3, 1::2] and X.T[::4, :] of X[8192,8192] int32 and fp32"

    def __init__(self, ctx, dist: Dist):
        import torch
        from quasarml_b200 import abi, datagen
        self.ctx = ctx
        Xi = _t(datagen.iota_i32((8192, 8192)))
        Xf = _t(datagen.uniform(datagen.SEEDS["gather_f32"], (8192, 8192), -1, 1))
        self.keep = [Xi, Xf]
        self.calls = []
        for X, code in ((Xi, abi.I32), (Xf, abi.F32)):
            o1 = torch.empty((2729, 4096), dtype=X.dtype, device="cuda")
            o2 = torch.empty((2048, 8192), dtype=X.dtype, device="cuda")
            self.keep += [o1, o2]
            v1 = abi.make_desc(X.data_ptr() + (5 * 8192 + 1) * 4, code, (2729, 4096), (3 * 8192, 2))
            v2 = abi.make_desc(X.data_ptr(), code, (2048, 8192), (4, 8192))
            self.calls += [(v1, abi.desc_of(o1), 134135808), (v2, abi.desc_of(o2), 335544320)]
        self.units_per_step = sum(c[2] for c in self.calls)
        self.unit = "GB/s"

    def compute(self, calls=None):
        for v, o, _ in (self.calls if calls is None else calls):
            self.ctx.gather(v, o)


class ArgReduceWorkload(Workload):
    name = "argmax/argmin X[64,512,1024] fp32 and fp16 over axis 0, 1, 2 and all, I32 indices (4 distinct X per dtype)"
    SHAPE = (64, 512, 1024)

    def __init__(self, ctx, dist: Dist, batch: int = 4):
        import torch
        from quasarml_b200 import abi, datagen
        self.ctx = ctx
        n = int(np.prod(self.SHAPE))
        # `batch` distinct X per dtype, batch entry innermost in the call order:
        # no call finds its input in L2
        self.keep = []
        xs32, xs16 = [], []
        for b in range(batch):
            X = _t(datagen.normal(datagen.SEEDS["red_X"], self.SHAPE, 0.0, 1.0, offset=(b * dist.world + dist.rank) * n))
            xs32.append(X)
            xs16.append(X.half())
        self.keep += xs32 + xs16
        self.calls = []
        for xs, es in ((xs32, 4), (xs16, 2)):
            for axis in (None, 0, 1, 2):
                oshape = abi.reduced_shape(self.SHAPE, axis, False)
                for op in (abi.ARG_MAX, abi.ARG_MIN):
                    for x in xs:
                        out = torch.empty(oshape, dtype=torch.int32, device="cuda")
                        self.keep.append(out)
                        self.calls.append((op, abi.desc_of(x), abi.AXIS_ALL if axis is None else axis,
                                           abi.desc_of(out), n * es + out.numel() * 4))
        self.units_per_step = sum(c[4] for c in self.calls)
        self.unit = "GB/s"

    def compute(self, calls=None):
        for op, x, axis, o, _ in (self.calls if calls is None else calls):
            self.ctx.arg_reduce(op, x, axis, False, o)


class LayerNormWorkload(Workload):
    name = "layer norm X[16384,4096] fp32 and fp16, gamma/beta fp32, eps 1e-5"

    def __init__(self, ctx, dist: Dist):
        import torch
        from quasarml_b200 import abi, datagen
        self.ctx = ctx
        n = 16384 * 4096
        X = _t(datagen.normal(datagen.SEEDS["ln_X"], (16384, 4096), 0.5, 2.0, offset=dist.rank * n))
        g = _t(datagen.normal(datagen.SEEDS["ln_gamma"], (4096,), 1.0, 0.1))
        b = _t(datagen.normal(datagen.SEEDS["ln_beta"], (4096,), 0.0, 0.1))
        Xh = X.half()
        Y, Yh = torch.empty_like(X), torch.empty_like(Xh)
        self.keep = [X, g, b, Xh, Y, Yh]
        d = abi.desc_of
        self.calls = [(d(X), d(g), d(b), d(Y), 536903680), (d(Xh), d(g), d(b), d(Yh), 268468224)]
        self.units_per_step = sum(c[4] for c in self.calls)
        self.unit = "GB/s"

    def compute(self, calls=None):
        for x, g, b, y, _ in (self.calls if calls is None else calls):
            self.ctx.layer_norm(x, g, b, 1e-5, y)


class SoftmaxWorkload(Workload):
    name = "softmax over the last axis of X[16384,4096] fp32 and fp16"

    def __init__(self, ctx, dist: Dist):
        import torch
        from quasarml_b200 import abi, datagen
        self.ctx = ctx
        n = 16384 * 4096
        X = _t(datagen.normal(datagen.SEEDS["ln_X"], (16384, 4096), 0.5, 2.0, offset=dist.rank * n))
        Xh = X.half()
        Y, Yh = torch.empty_like(X), torch.empty_like(Xh)
        self.keep = [X, Xh, Y, Yh]
        d = abi.desc_of
        self.calls = [(d(X), d(Y), 2 * n * 4), (d(Xh), d(Yh), 2 * n * 2)]
        self.units_per_step = sum(c[2] for c in self.calls)
        self.unit = "GB/s"

    def compute(self, calls=None):
        for x, y, _ in (self.calls if calls is None else calls):
            self.ctx.softmax(x, -1, y)


class MatmulWorkload(Workload):
    def __init__(self, ctx, dist: Dist, dtype: str, batched: bool, fp32_precision: str = "3xtf32"):
        import torch
        from quasarml_b200 import abi, datagen
        self.ctx, self.abi = ctx, abi
        if batched:
            s = 1.0 / np.sqrt(1024.0)
            A = _t(datagen.uniform(datagen.SEEDS["mm_Ab"], (32, 2048, 1024), -s, s))
            B = _t(datagen.uniform(datagen.SEEDS["mm_Bb"], (32, 1024, 2048), -s, s))
            C = torch.empty((32, 2048, 2048), device="cuda")
            self.flops = 2.0 * 32 * 2048 * 2048 * 1024
            self.name = f"batched matmul [32,2048,1024]x[32,1024,2048] {dtype}"
        else:
            s = 1.0 / np.sqrt(8192.0)
            A = _t(datagen.uniform(datagen.SEEDS["mm_A"], (8192, 8192), -s, s))
            B = _t(datagen.uniform(datagen.SEEDS["mm_B"], (8192, 8192), -s, s))
            C = torch.empty((8192, 8192), device="cuda")
            self.flops = 2.0 * 8192 ** 3
            self.name = f"matmul 8192x8192x8192 {dtype}"
        if dtype == "f16":
            A, B = A.half(), B.half()
            self.prec = abi.MM_FP16_F32ACC
        else:
            self.prec = abi.MM_FP32_3XTF32 if fp32_precision == "3xtf32" else abi.MM_FP32_FFMA
            self.name += f" ({fp32_precision})"
        self.keep = [A, B, C]
        self.a, self.b, self.c = abi.desc_of(A), abi.desc_of(B), abi.desc_of(C)
        self.units_per_step = self.flops
        self.unit = "TFLOP/s"

    def compute(self, calls=None):
        self.ctx.matmul(self.a, self.b, self.c, self.prec)


# ---------------------------------------------------------------------------
# Timing
# ---------------------------------------------------------------------------
def capture(fn, stream):
    """Captures fn() (which enqueues on `stream`) into a CUDA graph."""
    import torch
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g, stream=stream):
        fn()
    return g


def time_steps(wl, dist: Dist, stream, steps: int, warmup: int, sampler=None, use_graph=True):
    """Times `steps` steps on `stream` with CUDA events; returns the max over
    ranks (ms), the kernel launches counted by the library and the graph."""
    import torch
    with torch.cuda.stream(stream):
        for _ in range(warmup):
            wl.step()
        torch.cuda.synchronize()
        # Workloads with an exchange and a split step (ReduceWorkload) replay
        # two graphs with the collectives started between them.
        split = use_graph and dist.pg is not None and hasattr(wl, "exchange_start")
        g = None
        if split:
            gx = capture(lambda: wl.compute(wl.calls_x), stream)
            gl = capture(lambda: wl.compute(wl.calls_l), stream)
            g = (gx, gl)
        elif use_graph:
            g = capture(wl.compute, stream)
        torch.cuda.synchronize()
        dist.barrier()
        torch.cuda.synchronize()
        start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        per_step = None
        if g is not None:
            # launches per step: the library counts each launch it enqueues
            l0 = wl.ctx.launch_count()
            wl.compute()
            per_step = wl.ctx.launch_count() - l0
            torch.cuda.synchronize()
        launches0 = wl.ctx.launch_count()
        if sampler:
            sampler.__enter__()
        start.record(stream)
        for _ in range(steps):
            if split:
                g[0].replay()
                works = wl.exchange_start()
                g[1].replay()
                wl.exchange_finish(works)
            elif g is not None:
                g.replay()
                wl.exchange()
            else:
                wl.step()
        end.record(stream)
        torch.cuda.synchronize()
        if sampler:
            sampler.__exit__()
    launches = wl.ctx.launch_count() - launches0
    if g is not None:
        launches += per_step * steps
    ms = start.elapsed_time(end)
    dist.barrier()
    return dist.max(ms), launches, g


def family_times(wl, stream, reps: int = 5):
    """Average device duration of one launch of each kernel family: the
    family's calls of one step captured alone in a CUDA graph and replayed."""
    import torch
    # each call's family is the kernel the library chose for it
    fams = {}
    with torch.cuda.stream(stream):
        for c in wl.calls:
            wl.compute([c])
            fams.setdefault(wl.ctx.last_kernel(), []).append(c)
    torch.cuda.synchronize()
    out = {}
    with torch.cuda.stream(stream):
        for fam, calls in fams.items():
            g = capture(lambda: wl.compute(calls), stream)
            g.replay()
            torch.cuda.synchronize()
            a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            a.record(stream)
            for _ in range(reps):
                g.replay()
            b.record(stream)
            torch.cuda.synchronize()
            ms = a.elapsed_time(b) / reps
            out[fam] = {"launches": len(calls), "ms": ms, "bytes": sum(c[5] for c in calls)}
            del g
    return out


def time_e2e(wl, dist: Dist, stream, steps: int, warmup: int):
    import torch
    with torch.cuda.stream(stream):
        wl.e2e_setup()
        for _ in range(warmup):
            wl.e2e_step()
        torch.cuda.synchronize()
        dist.barrier()
        torch.cuda.synchronize()
        start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        start.record(stream)
        for _ in range(steps):
            wl.e2e_step()
        end.record(stream)
        torch.cuda.synchronize()
    return dist.max(start.elapsed_time(end))


def roofline_from_families(fam, hbm_peak, peak_kind):
    total = sum(f["ms"] for f in fam.values())
    dom = max(fam, key=lambda k: fam[k]["ms"])
    f = fam[dom]
    per_launch_ms = f["ms"] / f["launches"]
    achieved = f["bytes"] / (f["ms"] / 1e3) / 1e9
    ratio = ncu_traffic().get(dom)
    # DRAM bytes per launch: the captured launch's traffic/algorithmic ratio
    # (profiles/) applied to this family's average algorithmic bytes per launch.
    traffic = round(ratio * f["bytes"] / f["launches"]) if ratio else None
    return {"kernel": dom, "bound": "hbm", "achieved": round(achieved, 1), "peak": hbm_peak, "unit": "GB/s",
            "frac": round(achieved / hbm_peak, 4), "peak_source": peak_kind,
            "traffic": traffic, "traffic_source": "ncu capture in profiles/, scaled by bytes processed"
            if ratio else None,
            "algorithmic_bytes_per_launch": round(f["bytes"] / f["launches"]),
            "avg_launch_us": round(per_launch_ms * 1e3, 2),
            "share_of_step": round(f["ms"] / total, 3),
            "timing": "CUDA events around replays of a graph holding one step's launches of this kernel",
            "families": {k: {"share": round(v["ms"] / total, 3),
                             "gbs": round(v["bytes"] / (v["ms"] / 1e3) / 1e9, 1),
                             "frac": round(v["bytes"] / (v["ms"] / 1e3) / 1e9 / hbm_peak, 4),
                             "avg_launch_us": round(v["ms"] / v["launches"] * 1e3, 2),
                             "launches": v["launches"]} for k, v in fam.items()}}


# ---------------------------------------------------------------------------
# CPU side (oracle): baseline and the reference arm
# ---------------------------------------------------------------------------
class CpuReduceSample:
    """The headline reductions on X[8,512,1024] (1/8 of one X), fp32 and fp16,
    through the oracle's OpenMP restatement."""
    SHAPE = (8, 512, 1024)

    def __init__(self):
        from oracle import qsml_oracle as orc
        from quasarml_b200 import datagen
        self.orc = orc
        self.L = orc.lib()
        self.x32 = datagen.normal(datagen.SEEDS["red_X"], self.SHAPE, 0.0, 1.0)
        self.x16 = self.x32.astype(np.float16)
        self.out = np.empty(int(np.prod(self.SHAPE)), np.float32)
        self.bytes = 0
        self.plan = []
        for x, es, fn in ((self.x32, 4, self.L.orc_reduce_f32_par), (self.x16, 2, self.L.orc_reduce_f16_par)):
            for axis in (None, 0, 1, 2):
                if axis is None:
                    o, k, i = 1, x.size, 1
                else:
                    o = int(np.prod(x.shape[:axis]))
                    k = x.shape[axis]
                    i = int(np.prod(x.shape[axis + 1:]))
                for op in range(4):
                    self.plan.append((fn, op, x, o, k, i))
                    self.bytes += x.size * es + o * i * es

    def run(self):
        for fn, op, x, o, k, i in self.plan:
            fn(op, x.ctypes.data, o, k, i, self.out.ctypes.data)

    def cores(self):
        return self.orc.lib().orc_num_threads()


def cpu_baseline(min_seconds=10.0, max_seconds=30.0):
    s = CpuReduceSample()
    s.orc.lib().orc_set_num_threads(host_threads())
    s.run()
    t0 = time.perf_counter()
    n = 0
    while True:
        s.run()
        n += 1
        el = time.perf_counter() - t0
        if el >= min_seconds or el >= max_seconds:
            break
    gbs = s.bytes * n / el / 1e9
    return {"value": round(gbs, 2), "unit": "GB/s", "cores": s.cores(), "kind": "port",
            "sample": f"the same 32 reductions on X[8,512,1024] (1/8 of one X) fp32+fp16, {n} passes in {el:.1f} s"}


def host_threads() -> int:
    try:
        return len(os.sched_getaffinity(0))
    except (AttributeError, OSError):
        return os.cpu_count() or 1


def run_reference(args, dist: Dist):
    if dist.rank != 0:
        return
    s = CpuReduceSample()
    # rank 0 alone runs: every host thread, whatever OMP_NUM_THREADS the
    # launcher set for its ranks
    s.orc.lib().orc_set_num_threads(host_threads())
    for _ in range(max(args.warmup, 0)):
        s.run()
    t0 = time.perf_counter()
    for _ in range(args.steps):
        s.run()
    el = time.perf_counter() - t0
    gbs = s.bytes * args.steps / el / 1e9
    line = {"impl": "reference", "metric": METRIC, "value": round(gbs, 3), "unit": "GB/s", "n_gpus": args.gpus,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(el / args.steps * 1e3, 3),
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32+f16 (fp32 accumulate)",
            "data": "synthetic (seeded normal)",
            "config": {"workload": ReduceWorkload.name, "sample": "X[8,512,1024] per step (1/8 of one X)",
                       "parallelism": "host cores (OpenMP)"},
            "cpu_baseline": {"value": round(gbs, 3), "unit": "GB/s", "cores": s.cores(), "kind": "port",
                             "sample": "X[8,512,1024] fp32+fp16, 32 reductions per step"},
            "e2e": {"value": round(gbs, 3), "unit": "GB/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
            "note": "the reference's only compute path is Vulkan (no graphics stack on this box); its arithmetic is "
                    "restated by oracle/qsml_oracle.c and timed on the host cores"}
    print(json.dumps(line), flush=True)


def run_single(which: str, reps: int = 3):
    """One kernel of the workloads, `reps` launches on full-size inputs (for
    ncu: the launch to capture is then the 2nd or 3rd)."""
    import torch
    from quasarml_b200 import abi, datagen
    torch.cuda.set_device(0)
    ctx = abi.Context(0)
    d = abi.desc_of
    if which.startswith("reduce"):
        x = _t(datagen.normal(datagen.SEEDS["red_X"], (64, 512, 1024), 0.0, 1.0))
        if which.endswith("f16"):
            x = x.half()
        axis = {"reduce_all": None, "reduce_all_f16": None, "reduce_axis0": 0, "reduce_axis1": 1,
                "reduce_axis2": 2}[which]
        out = torch.empty(abi.reduced_shape(tuple(x.shape), axis, False), dtype=x.dtype, device="cuda")
        for _ in range(reps):
            ctx.reduce(abi.RED_SUM, d(x), abi.AXIS_ALL if axis is None else axis, False, d(out))
    elif which == "chain_add":
        A = _t(datagen.uniform(1, (4096, 4096), -1, 1))
        B = _t(datagen.uniform(2, (1, 4096), -1, 1))
        out = torch.empty_like(A)
        for _ in range(reps):
            ctx.binary(abi.OP_ADD, d(A), d(B), d(out))
    elif which == "chain_fused":
        wl = FusedChainWorkload(ctx, Dist(), batch=1)
        for _ in range(reps):
            wl.compute()
    elif which.startswith("argmax"):
        x = _t(datagen.normal(datagen.SEEDS["red_X"], (64, 512, 1024), 0.0, 1.0))
        if which.endswith("_f16"):
            x = x.half()
        axis = None if which == "argmax_all" else 1
        out = torch.empty(abi.reduced_shape(tuple(x.shape), axis, False), dtype=torch.int32, device="cuda")
        for _ in range(reps):
            ctx.arg_reduce(abi.ARG_MAX, d(x), abi.AXIS_ALL if axis is None else axis, False, d(out))
    elif which.startswith("gather"):
        X = _t(datagen.iota_i32((8192, 8192)))
        if which == "gather_t":
            v, out = abi.make_desc(X.data_ptr(), abi.I32, (2048, 8192), (4, 8192)), torch.empty((2048, 8192), dtype=torch.int32, device="cuda")
        else:
            v = abi.make_desc(X.data_ptr() + (5 * 8192 + 1) * 4, abi.I32, (2729, 4096), (3 * 8192, 2))
            out = torch.empty((2729, 4096), dtype=torch.int32, device="cuda")
        for _ in range(reps):
            ctx.gather(v, d(out))
    elif which in ("layernorm", "layernorm_f16", "layernorm_f16_8192"):
        R, C = (8192, 8192) if which == "layernorm_f16_8192" else (16384, 4096)
        X = _t(datagen.normal(10, (R, C), 0.5, 2.0))
        if which != "layernorm":
            X = X.half()
        g = _t(datagen.normal(11, (C,), 1.0, 0.1))
        b = _t(datagen.normal(12, (C,), 0.0, 0.1))
        Y = torch.empty_like(X)
        for _ in range(reps):
            ctx.layer_norm(d(X), d(g), d(b), 1e-5, d(Y))
    elif which == "matmul_f16":
        s = 1.0 / np.sqrt(8192.0)
        A = _t(datagen.uniform(6, (8192, 8192), -s, s)).half()
        B = _t(datagen.uniform(7, (8192, 8192), -s, s)).half()
        C = torch.empty((8192, 8192), device="cuda")
        for _ in range(reps):
            ctx.matmul(d(A), d(B), d(C), abi.MM_FP16_F32ACC)
    elif which in ("softmax", "softmax_f16"):
        X = _t(datagen.normal(10, (16384, 4096), 0.5, 2.0))
        if which == "softmax_f16":
            X = X.half()
        Y = torch.empty_like(X)
        for _ in range(reps):
            ctx.softmax(d(X), -1, d(Y))
    elif which == "bmm_f16":
        s = 1.0 / np.sqrt(1024.0)
        A = _t(datagen.uniform(9, (32, 2048, 1024), -s, s)).half()
        B = _t(datagen.uniform(8, (32, 1024, 2048), -s, s)).half()
        C = torch.empty((32, 2048, 2048), device="cuda")
        for _ in range(reps):
            ctx.matmul(d(A), d(B), d(C), abi.MM_FP16_F32ACC)
    elif which == "matmul_3xtf32":
        s = 1.0 / np.sqrt(8192.0)
        A = _t(datagen.uniform(6, (8192, 8192), -s, s))
        B = _t(datagen.uniform(7, (8192, 8192), -s, s))
        C = torch.empty((8192, 8192), device="cuda")
        for _ in range(reps):
            ctx.matmul(d(A), d(B), d(C), abi.MM_FP32_3XTF32)
    torch.cuda.synchronize()
    ctx.close()


# ---------------------------------------------------------------------------
# Main
# ---------------------------------------------------------------------------
def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--no-extras", action="store_true", help="skip the other workloads at N=1")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--workload", default="reduce",
                    choices=["reduce", "chain", "gather", "layernorm", "matmul_f16", "matmul_f32"])
    ap.add_argument("--single", default=None,
                    choices=["reduce_all", "reduce_axis0", "reduce_axis1", "reduce_axis2", "reduce_all_f16",
                             "chain_add", "chain_fused", "gather_t", "gather_s", "layernorm", "matmul_f16",
                             "matmul_3xtf32", "bmm_f16", "argmax_all", "argmax_axis1", "argmax_axis1_f16", "softmax",
                             "softmax_f16",
                             "layernorm_f16", "layernorm_f16_8192"],
                    help="run one kernel of the workloads a few times and exit (profiling aid, prints nothing)")
    args = ap.parse_args()
    args.warmup = max(args.warmup, 3)

    if args.single:
        run_single(args.single)
        return

    # Ranks share the host: split its cores between the input generators.
    if int(os.environ.get("WORLD_SIZE", "1")) > 1 and "OMP_NUM_THREADS" not in os.environ:
        local = int(os.environ.get("LOCAL_WORLD_SIZE", os.environ.get("WORLD_SIZE", "1")))
        os.environ["OMP_NUM_THREADS"] = str(max(1, (os.cpu_count() or 1) // local))

    dist = Dist()
    if args.impl == "reference":
        run_reference(args, dist)
        return

    import torch
    from quasarml_b200 import abi
    torch.cuda.set_device(dist.local)
    dist.init("nccl")
    # All library work goes to one non-default stream so it can be captured.
    stream = torch.cuda.Stream()
    ctx = abi.Context(dist.local, use_torch_stream=False)
    ctx.set_stream(stream.cuda_stream)
    hbm, tf_burst, tf_sus, peak_kind = peaks()

    wl = {"reduce": lambda: ReduceWorkload(ctx, dist), "chain": lambda: ChainWorkload(ctx, dist),
          "gather": lambda: GatherWorkload(ctx, dist), "layernorm": lambda: LayerNormWorkload(ctx, dist),
          "matmul_f16": lambda: MatmulWorkload(ctx, dist, "f16", False),
          "matmul_f32": lambda: MatmulWorkload(ctx, dist, "f32", False)}[args.workload]()

    sampler = ClockSampler(dist.local)
    ms, launches, graph = time_steps(wl, dist, stream, args.steps, args.warmup, sampler=sampler)
    del graph
    units = wl.units_per_step * args.steps * dist.world
    value = units / (ms / 1e3) / (1e9 if wl.unit == "GB/s" else 1e12)

    line = {"metric": METRIC, "value": round(value, 2), "unit": wl.unit, "n_gpus": dist.world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(ms / args.steps, 4),
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
            "dtype": "f32+f16 (fp32 accumulate)" if args.workload == "reduce" else "f32",
            "data": "synthetic (seeded, counter-based generator)",
            "config": {"workload": wl.name, "parallelism": f"dp{dist.world}",
                       "l2": "inputs larger than L2: 8 distinct X per dtype per step (1.5 GB), batch entry innermost in the call order so no call finds its input in L2"
                       if args.workload == "reduce" else "inputs larger than L2",
                       "calls_per_step": len(getattr(wl, "calls", [])) or 1,
                       "launch": "each step's kernel calls replayed from one CUDA graph (N=1); for N>1 two "
                                 "graphs, the exchanged reductions then the local ones, with the NCCL "
                                 "all-reduces started between them and waited for after"},
            "gpu_launches": launches, "clocks": sampler.summary()}
    if args.workload == "reduce":
        line["roofline"] = roofline_from_families(family_times(wl, stream), hbm, peak_kind)
    if hasattr(wl, "e2e_step"):
        e_steps = max(2, min(args.steps, 5))
        ems = time_e2e(wl, dist, stream, e_steps, 1)
        ev = wl.units_per_step * e_steps * dist.world / (ems / 1e3) / 1e9
        line["e2e"] = {"value": round(ev, 2), "unit": wl.unit, "h2d_bytes_per_step": wl.h2d_bytes,
                       "d2h_bytes_per_step": wl.d2h_bytes, "ms_per_step": round(ems / e_steps, 3),
                       "path": "pinned host -> qsml_h2d per batch entry on a second context's stream -> "
                               "qsml_reduce x256, each entry's 32 as soon as its X has landed -> "
                               "qsml_d2h_async of each entry's results on a third stream, per step"}

    if dist.world == 1 and not args.no_extras and args.workload == "reduce":
        extras = {}
        del wl
        torch.cuda.empty_cache()
        for key, mk, st in (("elementwise_chain", lambda: ChainWorkload(ctx, dist), 10),
                            ("elementwise_chain_fused", lambda: FusedChainWorkload(ctx, dist), 20),
                            ("gather", lambda: GatherWorkload(ctx, dist), 20),
                            ("layernorm", lambda: LayerNormWorkload(ctx, dist), 20),
                            ("argmax_argmin", lambda: ArgReduceWorkload(ctx, dist), 20),
                            ("softmax", lambda: SoftmaxWorkload(ctx, dist), 20),
                            ("matmul_f16_8192", lambda: MatmulWorkload(ctx, dist, "f16", False), 5),
                            ("matmul_f32_8192_3xtf32", lambda: MatmulWorkload(ctx, dist, "f32", False), 5),
                            ("matmul_f32_8192_ffma", lambda: MatmulWorkload(ctx, dist, "f32", False, "ffma"), 3),
                            ("batched_matmul_f16", lambda: MatmulWorkload(ctx, dist, "f16", True), 5),
                            ("batched_matmul_f32_3xtf32", lambda: MatmulWorkload(ctx, dist, "f32", True), 5)):
            try:
                w = mk()
                ms_x, l_x, g = time_steps(w, dist, stream, st, 3)
                del g
                v = w.units_per_step * st / (ms_x / 1e3) / (1e9 if w.unit == "GB/s" else 1e12)
                peak = hbm if w.unit == "GB/s" else tf_burst
                extras[key] = {"workload": w.name, "value": round(v, 2), "unit": w.unit,
                               "frac_of_peak": round(v / peak, 4), "peak": peak,
                               "ms_per_step": round(ms_x / st, 3), "launches_per_step": l_x // st}
                del w
                torch.cuda.synchronize()
                torch.cuda.empty_cache()
            except Exception as e:  # report, do not hide
                extras[key] = {"error": repr(e)[:300]}
        line["other_workloads"] = extras

    if dist.world == 1 and dist.rank == 0 and not args.no_cpu_baseline and args.workload == "reduce":
        line["cpu_baseline"] = cpu_baseline()

    torch.cuda.synchronize()
    ctx.close()
    if dist.rank == 0:
        print(json.dumps(line), flush=True)
    dist.close()


if __name__ == "__main__":
    main()
