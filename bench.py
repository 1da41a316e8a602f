#!/usr/bin/env python
"""Benchmark of the QuasarML B200 backend (libqsml_cuda.so through its C ABI).

Headline workload (every N): the reductions configuration -- sum/mean/max/min
over axis 0, 1, 2 and all elements of X[64,512,1024] ~ N(0,1), in fp32 and
again with X in fp16 (fp32 accumulation).  One step processes a batch of 8
distinct X per dtype (1.5 GB of input, so no input is L2-resident when it is
read again), i.e. 256 reduction calls at N=1.  Under torchrun X is
row-sharded: each rank holds its own [64,512,1024] block of a
[64N,512,1024] tensor (weak scaling).  The axis-1/2 reductions need no
exchange; the axis-0 and full reductions write binary32 partials that the
library combines across ranks (qsml_allreduce_partials, NCCL over NVLink, on
a second stream while the axis-1/2 reductions run) and qsml_finish_partial
turns into the outputs (means from the combined sums, sum * 1/n).

value     : algorithmic bytes (each input read once, each output written once)
            of all ranks / max-over-ranks device time, inputs resident in HBM.
e2e       : the same through the C ABI from pinned host buffers: every step
            copies X host->device and the results device->host inside the
            timed region.
roofline  : the dominant kernel family of the step (per input dtype), its
            algorithmic bytes per launch / its CUDA-event duration, against
            the measured HBM copy bandwidth (MEASURED_PEAKS.json).
exchange  : (N>1) the combine timed alone on its stream.
cpu_baseline / --impl reference : the oracle's CPU restatement of the same
            reductions (OpenMP over all host cores), one X[64,512,1024] per
            dtype per step.
other_workloads: the elementwise chain (op by op and fused), strided
            gathers, layer norm, softmax, argmax/argmin and matmul
            configurations, each row-sharded over the ranks and timed the
            same way: weak scaling at every N (each rank the configuration's
            size) and, at N>1, strong scaling too (the configuration's tensor
            split N ways, "<name>_strong").
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

    @classmethod
    def single(cls) -> "Dist":
        """One rank without collectives (a rank timing work alone)."""
        d = cls.__new__(cls)
        d.world, d.rank, d.local, d.pg = 1, 0, 0, None
        return d

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

    def sum(self, v: float) -> float:
        if not self.pg:
            return v
        import torch
        t = torch.tensor([v], dtype=torch.float64, device="cuda")
        self.pg.all_reduce(t, op=self.pg.ReduceOp.SUM)
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


class RCall:
    """One library call of the reductions step: kind "reduce" (qsml_reduce of
    x over axis into out) or "finish" (qsml_finish_partial of partial x into
    out, n elements per output); nbytes its algorithmic bytes; out_t the
    output tensor; entry the batch entry it reads (None for a finish); dt
    "f32" or "f16", the input dtype (for the per-dtype roofline families)."""
    __slots__ = ("kind", "op", "x", "axis", "out", "n", "nbytes", "out_t", "entry", "dt")

    def __init__(self, kind, op, x, axis, out, nbytes, out_t, entry, dt, n=0):
        self.kind, self.op, self.x, self.axis, self.out = kind, op, x, axis, out
        self.nbytes, self.out_t, self.entry, self.dt, self.n = nbytes, out_t, entry, dt, n


class ReduceWorkload(Workload):
    """sum/mean/max/min over axis 0, 1, 2, all of X[64,512,1024], fp32 + fp16.

    N=1: 256 qsml_reduce calls per step.  N>1 (X row-sharded, rank r holding
    rows [64r, 64r+64) of X[64N,512,1024]): the axis-1/2 reductions are local
    (qsml_reduce, no exchange); for axis 0 and all elements each rank writes
    binary32 partials (SUM, MAX, MIN) into three flat buffers, the library
    combines each buffer across ranks (qsml_allreduce_partials on a second
    context's stream, NCCL over NVLink, while the axis-1/2 reductions run) and
    qsml_finish_partial writes the outputs: sums and max/min as combined, means
    as the combined sum * (1/n) with n counted over all ranks."""
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
        self.sharded = dist.world > 1
        # calls_l: reductions needing no exchange (all of them at N=1);
        # calls_x: the local partials of the exchanged ones; finishes: after
        # the exchange.  Batch entry innermost everywhere: consecutive calls
        # read different X, and a given X is read again only after the other
        # seven (>= 448 MB), so no call finds its input in L2.
        self.calls_l, self.calls_x, self.finishes = [], [], []
        self.keep = []
        for dt, xs in (("f32", self.x32), ("f16", self.x16)):
            tdt = torch.float32 if dt == "f32" else torch.float16
            es = 4 if dt == "f32" else 2
            for axis in self.axes:
                code = abi.AXIS_ALL if axis is None else axis
                oshape = abi.reduced_shape(self.SHAPE, axis, False)
                on = int(np.prod(oshape))
                if self.sharded and sharding.needs_exchange(axis):
                    continue
                for op in self.ops:
                    for b in range(batch):
                        out = torch.empty(oshape, dtype=tdt, device="cuda")
                        self.calls_l.append(RCall("reduce", op, abi.desc_of(xs[b]), code, abi.desc_of(out),
                                                  n * es + on * es, out, b, dt))
        if self.sharded:
            self._plan_exchange(batch, n)
        self.calls = self.calls_x + self.calls_l + self.finishes
        self.bytes_per_step = sum(c.nbytes for c in self.calls)
        self.units_per_step = self.bytes_per_step
        self.unit = "GB/s"
        self.h2d_bytes = sum(x.numel() * 4 for x in self.x32)  # X only: its fp16 copy is cast on the device
        self.d2h_bytes = sum(o.numel() * o.element_size() for o in self.outputs())

    def _plan_exchange(self, batch, n):
        import torch
        from quasarml_b200 import sharding
        abi = self.abi
        plan = sharding.ExchangePlan()
        G = self.dist.world * self.SHAPE[0]  # rows of the global X
        runs = []  # (dt, axis, op, per-entry count, finish index)
        for dt in ("f32", "f16"):
            for axis in (None, 0):
                on = int(np.prod(abi.reduced_shape(self.SHAPE, axis, False)))
                # elements reduced into each output over all ranks
                nglob = G * (n // self.SHAPE[0]) if axis is None else G
                for op in self.ops:
                    runs.append((dt, axis, op, on, plan.add((dt, axis), op, axis, batch * on, nglob)))
        self.flat = {g: torch.empty(max(sz, 1), dtype=torch.float32, device="cuda") for g, sz in plan.sizes.items()}
        group_op = {"sum": abi.RED_SUM, "max": abi.RED_MAX, "min": abi.RED_MIN}
        for (dt, axis), ax, group, off, count in plan.partials:
            xs, es = (self.x32, 4) if dt == "f32" else (self.x16, 2)
            oshape = abi.reduced_shape(self.SHAPE, axis, False)
            on = count // batch
            for b in range(batch):
                part = self.flat[group][off + b * on: off + (b + 1) * on].view(oshape)
                self.calls_x.append(RCall("reduce", group_op[group], abi.desc_of(xs[b]),
                                          abi.AXIS_ALL if axis is None else axis, abi.desc_of(part),
                                          n * es + on * 4, part, b, dt))
        self.exchanged_out = []
        for (dt, axis, op, on, fi) in runs:
            fop, group, off, count, nglob, _ = plan.finishes[fi]
            part = self.flat[group][off:off + count]
            if dt == "f32" and op != abi.RED_MEAN:
                out = part  # the combined partial is the result
            else:
                out = torch.empty(count, dtype=torch.float32 if dt == "f32" else torch.float16, device="cuda")
                es = 4 if dt == "f32" else 2
                self.finishes.append(RCall("finish", op, abi.desc_of(part), None, abi.desc_of(out),
                                           count * 4 + count * es, out, None, dt, n=nglob))
            self.exchanged_out.append(out)
        self.group = None

    def outputs(self):
        outs = [c.out_t for c in self.calls_l]
        if self.sharded:
            outs += self.exchanged_out
        return outs

    def compute(self, calls=None):
        ctx = self.ctx
        for c in (self.calls_l if calls is None else calls):
            if c.kind == "reduce":
                ctx.reduce(c.op, c.x, c.axis, False, c.out)
            else:
                ctx.finish_partial(c.op, c.x, c.n, c.out)

    # The library's own collective: a group over a second context whose stream
    # runs the combines while the main stream runs the local reductions.
    def init_exchange(self):
        if not self.sharded or self.group is not None:
            return
        import torch
        abi = self.abi
        self.xstream = torch.cuda.Stream(priority=-1)  # NCCL CTAs ahead of the local reductions
        self.xctx = abi.Context(torch.cuda.current_device(), use_torch_stream=False)
        self.xctx.set_stream(self.xstream.cuda_stream)
        uid = [abi.group_unique_id() if self.dist.rank == 0 else None]
        self.dist.pg.broadcast_object_list(uid, src=0)
        self.group = abi.Group.init_rank(self.xctx, uid[0], self.dist.world, self.dist.rank)
        self.ev_ready, self.ev_done = torch.cuda.Event(), torch.cuda.Event()

    def close_exchange(self):
        if getattr(self, "group", None) is not None:
            import torch
            torch.cuda.synchronize()
            self.group.destroy()
            self.group = None
            self.xctx.close()

    def exchange_start(self):
        if not self.sharded:
            return None
        import torch
        abi = self.abi
        self.init_exchange()
        self.ev_ready.record(torch.cuda.current_stream())
        self.xstream.wait_event(self.ev_ready)
        # one NCCL group for the three combines (launched together)
        abi.group_start()
        try:
            for g, op in (("sum", abi.RED_SUM), ("max", abi.RED_MAX), ("min", abi.RED_MIN)):
                self.group.allreduce_partials(0, op, self.flat[g].data_ptr(), self.flat[g].numel())
        finally:
            abi.group_end()
        self.ev_done.record(self.xstream)
        return self.ev_done

    def exchange_finish(self, done):
        if not self.sharded:
            return
        import torch
        torch.cuda.current_stream().wait_event(done)
        self.compute(self.finishes)

    def exchange(self):
        self.exchange_finish(self.exchange_start())

    def step(self):
        if not self.sharded:
            self.compute()
            return
        self.compute(self.calls_x)
        done = self.exchange_start()
        self.compute(self.calls_l)
        self.exchange_finish(done)

    # End-to-end: host -> device copies of X, the reductions, results back.
    # The uploads run on a second library context (its own stream, a copy
    # engine) one batch entry at a time; the reductions of entry b start as
    # soon as its X has landed (an event per entry), so compute overlaps the
    # PCIe transfers of the entries after it.
    def e2e_setup(self):
        import torch
        from quasarml_b200 import abi
        self.init_exchange()
        self.h32 = [x.cpu().pin_memory() for x in self.x32]
        self.local_out = [c.out_t for c in self.calls_l]
        self.hout = [o.cpu().pin_memory() for o in self.local_out]
        self.hxout = [o.cpu().pin_memory() for o in self.exchanged_out] if self.sharded else []
        self.copy_stream = torch.cuda.Stream()
        self.copy_ctx = abi.Context(torch.cuda.current_device())
        self.copy_ctx.set_stream(self.copy_stream.cuda_stream)
        self.back_stream = torch.cuda.Stream()
        self.back_ctx = abi.Context(torch.cuda.current_device())
        self.back_ctx.set_stream(self.back_stream.cuda_stream)
        self.d32 = [abi.desc_of(x) for x in self.x32]
        self.d16 = [abi.desc_of(x) for x in self.x16]
        self.landed = [torch.cuda.Event() for _ in range(self.batch)]
        self.reduced = [torch.cuda.Event() for _ in range(self.batch)]
        self.l_by_entry = [[i for i, c in enumerate(self.calls_l) if c.entry == b] for b in range(self.batch)]
        self.x_by_entry = [[c for c in self.calls_x if c.entry == b] for b in range(self.batch)]

    def e2e_step(self):
        import torch
        cur = torch.cuda.current_stream()
        self.copy_stream.wait_stream(cur)  # the previous step has read X
        for b in range(self.batch):
            # X crosses PCIe once; its binary16 copy is made on the device
            self.copy_ctx.h2d(self.x32[b].data_ptr(), self.h32[b].data_ptr(), self.h32[b].numel() * 4)
            self.copy_ctx.cast(self.d32[b], self.d16[b])
            self.landed[b].record(self.copy_stream)
        # Local results travel back on a third stream as each entry finishes
        # (the other PCIe direction); exchanged ones after the combine.
        for b in range(self.batch):
            cur.wait_event(self.landed[b])
            self.compute(self.x_by_entry[b])
            self.compute([self.calls_l[i] for i in self.l_by_entry[b]])
            self.reduced[b].record(cur)
            self.back_stream.wait_event(self.reduced[b])
            for i in self.l_by_entry[b]:
                out = self.local_out[i]
                self.back_ctx.d2h(self.hout[i].data_ptr(), out.data_ptr(), out.numel() * out.element_size(),
                                  sync=False)
        if self.sharded:
            self.exchange_finish(self.exchange_start())
            for h, out in zip(self.hxout, self.exchanged_out):
                self.ctx.d2h(h.data_ptr(), out.data_ptr(), out.numel() * out.element_size(), sync=False)
        cur.wait_stream(self.back_stream)


def row_block(total_rows: int, dist: Dist, scale: str):
    """(first global row, rows, global rows) of this rank's block of a
    tensor whose configuration has `total_rows` rows.  weak: every rank holds
    `total_rows` rows of an N-times-taller tensor; strong: the configuration's
    own tensor is split over the ranks (qsml_shard_rows' balanced split)."""
    if scale == "weak" or dist.world == 1:
        return dist.rank * total_rows, total_rows, total_rows * dist.world
    from quasarml_b200 import abi
    b, c = abi.shard_rows(total_rows, dist.world, dist.rank)
    return b, c, total_rows


class ChainWorkload(Workload):
    """relu(pow((A+B)*B - A, 2) / D), A[4096,4096], B[1,4096], D[4096,1]:
    A and D row-sharded, B replicated."""
    name = "elementwise chain relu(pow((A+B)*B - A, 2.0) / D), A[4096,4096], B[1,4096], D[4096,1] fp32"

    def __init__(self, ctx, dist: Dist, batch: int = 4, scale: str = "weak"):
        import torch
        from quasarml_b200 import abi, datagen
        self.ctx, self.abi = ctx, abi
        r0, R, G = row_block(4096, dist, scale)
        self.sets = []
        for b in range(batch):
            off = b * G + r0  # batch entry b is its own [G, 4096] tensor
            A = _t(datagen.uniform(datagen.SEEDS["ew_A"], (R, 4096), -1, 1, offset=off * 4096))
            B = _t(datagen.uniform(datagen.SEEDS["ew_B"], (1, 4096), -1, 1))
            D = _t(datagen.uniform(datagen.SEEDS["ew_D"], (R, 1), 0.5, 2, offset=off))
            ts = [torch.empty((R, 4096), device="cuda") for _ in range(6)]
            self.sets.append((A, B, D, ts))
        d = abi.desc_of
        n4 = R * 4096 * 4
        self.calls = []
        for A, B, D, t in self.sets:
            self.calls += [("bin", abi.OP_ADD, d(A), d(B), d(t[0]), 2 * n4 + 16384),
                           ("bin", abi.OP_MUL, d(t[0]), d(B), d(t[1]), 2 * n4 + 16384),
                           ("bin", abi.OP_SUB, d(t[1]), d(A), d(t[2]), 3 * n4),
                           ("scal", abi.OP_POW, d(t[2]), 2.0, d(t[3]), 2 * n4),
                           ("bin", abi.OP_DIV, d(t[3]), d(D), d(t[4]), 2 * n4 + R * 4),
                           ("un", abi.UN_RELU, d(t[4]), None, d(t[5]), 2 * n4)]
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

    def __init__(self, ctx, dist: Dist, batch: int = 4, scale: str = "weak"):
        import torch
        from quasarml_b200 import abi, datagen
        self.ctx = ctx
        r0, R, G = row_block(4096, dist, scale)
        e = abi.Expr()
        a, b, dd = e.input(0), e.input(1), e.input(2)
        t = e.binary(abi.OP_SUB, e.binary(abi.OP_MUL, e.binary(abi.OP_ADD, a, b), b), a)
        e.unary(abi.UN_RELU, e.binary(abi.OP_DIV, e.binary(abi.OP_POW, t, e.const(2.0)), dd))
        self.nodes = (abi.FuseNode * len(e.nodes))(*[abi.FuseNode(*n) for n in e.nodes])
        self.keep, self.calls = [], []
        d = abi.desc_of
        for bi in range(batch):
            off = bi * G + r0
            A = _t(datagen.uniform(datagen.SEEDS["ew_A"], (R, 4096), -1, 1, offset=off * 4096))
            B = _t(datagen.uniform(datagen.SEEDS["ew_B"], (1, 4096), -1, 1))
            D = _t(datagen.uniform(datagen.SEEDS["ew_D"], (R, 1), 0.5, 2, offset=off))
            out = torch.empty((R, 4096), device="cuda")
            self.keep += [A, B, D, out]
            self.calls.append(([d(A), d(B), d(D)], d(out), 2 * R * 4096 * 4 + 4096 * 4 + R * 4))
        self.units_per_step = sum(c[2] for c in self.calls)
        self.unit = "GB/s"

    def compute(self, calls=None):
        for ins, out, _ in (self.calls if calls is None else calls):
            self.ctx.elementwise_fused(self.nodes, ins, out)


class GatherWorkload(Workload):
    """X[5::3, 1::2] and X.T[::4, :] of X[8192,8192], X row-sharded: each rank
    materialises the output rows whose source rows it holds (X[5::3, 1::2])
    and the output columns of its rows (X.T[::4, :], out[i, j] = X[j, 4i]),
    each as a contiguous block."""
    name = "strided gather X[5::3, 1::2] and X.T[::4, :] of X[8192,8192] int32 and fp32"

    def __init__(self, ctx, dist: Dist, scale: str = "weak"):
        import torch
        from quasarml_b200 import abi, datagen
        self.ctx = ctx
        r0, R, G = row_block(8192, dist, scale)
        rows = (np.arange(R, dtype=np.int64) + r0)[:, None] * 8192 + np.arange(8192, dtype=np.int64)[None, :]
        Xi = _t(rows.astype(np.int32))  # X[i, j] = i*8192 + j over the global rows
        Xf = _t(datagen.uniform(datagen.SEEDS["gather_f32"], (R, 8192), -1, 1, offset=r0 * 8192))
        self.keep = [Xi, Xf]
        # X[5::3, 1::2]: global source rows 5 + 3i inside this block
        s0 = max(5, r0 + ((5 - r0) % 3))
        n1 = len(range(s0, r0 + R, 3))
        self.first_out_row = (s0 - 5) // 3
        self.calls = []
        for X, code in ((Xi, abi.I32), (Xf, abi.F32)):
            o1 = torch.empty((n1, 4096), dtype=X.dtype, device="cuda")
            o2 = torch.empty((2048, R), dtype=X.dtype, device="cuda")
            self.keep += [o1, o2]
            v1 = abi.make_desc(X.data_ptr() + ((s0 - r0) * 8192 + 1) * 4, code, (n1, 4096), (3 * 8192, 2))
            v2 = abi.make_desc(X.data_ptr(), code, (2048, R), (4, 8192))
            # bytes: writes + the read footprint in 32-byte sectors
            self.calls += [(v1, abi.desc_of(o1), n1 * (4096 * 4 + 8192 * 4)),
                           (v2, abi.desc_of(o2), 2048 * R * 4 + R * 8192 * 4)]
        self.units_per_step = sum(c[2] for c in self.calls)
        self.unit = "GB/s"

    def compute(self, calls=None):
        for v, o, _ in (self.calls if calls is None else calls):
            self.ctx.gather(v, o)


class ReduceViewWorkload(Workload):
    """Reductions of non-contiguous views of X[8192,8192] fp32, read in place:
    X[5::3, 1::2] ([2729,4096], element strides (24576, 2)) and X.T
    ([8192,8192], strides (1, 8192)), sum over each axis and max over the
    last.  Bytes: the views' 32-byte-sector read footprint (stride-2 columns
    touch every sector of their rows) plus the output."""
    name = "reductions of strided views X[5::3, 1::2] and X.T of X[8192,8192] fp32: sum over each axis, max over the last"

    def __init__(self, ctx, dist: Dist, scale: str = "weak"):
        import torch
        from quasarml_b200 import abi, datagen
        self.ctx = ctx
        r0, R, G = row_block(8192, dist, scale)
        # one X per view (the views of X[8192N,8192], 2 x 256 MiB), calls
        # alternating between them: no call finds its input in L2
        Xa = _t(datagen.uniform(datagen.SEEDS["gather_f32"], (R, 8192), -1, 1, offset=r0 * 8192))
        Xb = _t(datagen.uniform(datagen.SEEDS["gather_f32"], (R, 8192), -1, 1, offset=(G + r0) * 8192))
        self.keep = [Xa, Xb]
        s0 = max(5, r0 + ((5 - r0) % 3))
        n1 = len(range(s0, r0 + R, 3))
        v1 = abi.make_desc(Xa.data_ptr() + ((s0 - r0) * 8192 + 1) * 4, abi.F32, (n1, 4096), (3 * 8192, 2))
        v2 = abi.make_desc(Xb.data_ptr(), abi.F32, (8192, R), (1, 8192))
        foot1, foot2 = n1 * 8192 * 4, R * 8192 * 4
        self.calls = []
        for op, axis in ((abi.RED_SUM, 0), (abi.RED_SUM, 1), (abi.RED_MAX, 1)):
            for view, shape, foot in ((v1, (n1, 4096), foot1), (v2, (8192, R), foot2)):
                oshape = abi.reduced_shape(shape, axis, False)
                out = torch.empty(oshape, device="cuda")
                self.keep.append(out)
                self.calls.append((op, view, axis, abi.desc_of(out), foot + out.numel() * 4))
        self.units_per_step = sum(c[4] for c in self.calls)
        self.unit = "GB/s"

    def compute(self, calls=None):
        for op, x, axis, o, _ in (self.calls if calls is None else calls):
            self.ctx.reduce(op, x, axis, False, o)


class ArgReduceWorkload(Workload):
    """argmax/argmin of X[64,512,1024], fp32 and fp16.  Under sharding only the
    axes whose result needs no exchange (1 and 2) run."""
    name = "argmax/argmin X[64,512,1024] fp32 and fp16 over axis 0, 1, 2 and all, I32 indices (4 distinct X per dtype)"
    SHAPE = (64, 512, 1024)

    def __init__(self, ctx, dist: Dist, batch: int = 4, scale: str = "weak"):
        import torch
        from quasarml_b200 import abi, datagen
        self.ctx = ctx
        r0, R, G = row_block(self.SHAPE[0], dist, scale)
        shape = (R,) + self.SHAPE[1:]
        n = int(np.prod(shape))
        per_row = int(np.prod(self.SHAPE[1:]))
        axes = (None, 0, 1, 2) if dist.world == 1 else (1, 2)
        if dist.world > 1:
            self.name = ("argmax/argmin X[64,512,1024] fp32 and fp16 over axis 1 and 2 (row-local under sharding), "
                         "I32 indices (4 distinct X per dtype)")
        # `batch` distinct X per dtype, batch entry innermost in the call order:
        # no call finds its input in L2
        self.keep = []
        xs32, xs16 = [], []
        for b in range(batch):
            X = _t(datagen.normal(datagen.SEEDS["red_X"], shape, 0.0, 1.0, offset=(b * G + r0) * per_row))
            xs32.append(X)
            xs16.append(X.half())
        self.keep += xs32 + xs16
        self.calls = []
        for xs, es in ((xs32, 4), (xs16, 2)):
            for axis in axes:
                oshape = abi.reduced_shape(shape, axis, False)
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

    def __init__(self, ctx, dist: Dist, scale: str = "weak"):
        import torch
        from quasarml_b200 import abi, datagen
        self.ctx = ctx
        r0, R, G = row_block(16384, dist, scale)
        X = _t(datagen.normal(datagen.SEEDS["ln_X"], (R, 4096), 0.5, 2.0, offset=r0 * 4096))
        g = _t(datagen.normal(datagen.SEEDS["ln_gamma"], (4096,), 1.0, 0.1))
        b = _t(datagen.normal(datagen.SEEDS["ln_beta"], (4096,), 0.0, 0.1))
        Xh = X.half()
        Y, Yh = torch.empty_like(X), torch.empty_like(Xh)
        self.keep = [X, g, b, Xh, Y, Yh]
        d = abi.desc_of
        n = R * 4096
        self.calls = [(d(X), d(g), d(b), d(Y), 2 * n * 4 + 32768), (d(Xh), d(g), d(b), d(Yh), 2 * n * 2 + 32768)]
        self.units_per_step = sum(c[4] for c in self.calls)
        self.unit = "GB/s"

    def compute(self, calls=None):
        for x, g, b, y, _ in (self.calls if calls is None else calls):
            self.ctx.layer_norm(x, g, b, 1e-5, y)


class SoftmaxWorkload(Workload):
    name = "softmax over the last axis of X[16384,4096] fp32 and fp16"

    def __init__(self, ctx, dist: Dist, scale: str = "weak"):
        import torch
        from quasarml_b200 import abi, datagen
        self.ctx = ctx
        r0, R, G = row_block(16384, dist, scale)
        X = _t(datagen.normal(datagen.SEEDS["ln_X"], (R, 4096), 0.5, 2.0, offset=r0 * 4096))
        Xh = X.half()
        Y, Yh = torch.empty_like(X), torch.empty_like(Xh)
        self.keep = [X, Xh, Y, Yh]
        d = abi.desc_of
        n = R * 4096
        self.calls = [(d(X), d(Y), 2 * n * 4), (d(Xh), d(Yh), 2 * n * 2)]
        self.units_per_step = sum(c[2] for c in self.calls)
        self.unit = "GB/s"

    def compute(self, calls=None):
        for x, y, _ in (self.calls if calls is None else calls):
            self.ctx.softmax(x, -1, y)


class MatmulWorkload(Workload):
    """C = A.B with A's rows sharded and B replicated (batched: the batch dim
    sharded)."""

    def __init__(self, ctx, dist: Dist, dtype: str, batched: bool, fp32_precision: str = "3xtf32",
                 scale: str = "weak", out16: bool = False):
        import torch
        from quasarml_b200 import abi, datagen
        self.ctx, self.abi = ctx, abi
        if batched:
            s = 1.0 / np.sqrt(1024.0)
            e0, E, _ = row_block(32, dist, scale)
            A = _t(datagen.uniform(datagen.SEEDS["mm_Ab"], (E, 2048, 1024), -s, s, offset=e0 * 2048 * 1024))
            B = _t(datagen.uniform(datagen.SEEDS["mm_Bb"], (E, 1024, 2048), -s, s, offset=e0 * 1024 * 2048))
            C = torch.empty((E, 2048, 2048), device="cuda", dtype=torch.float16 if out16 else torch.float32)
            self.flops = 2.0 * E * 2048 * 2048 * 1024
            self.name = f"batched matmul [32,2048,1024]x[32,1024,2048] {dtype}"
        else:
            s = 1.0 / np.sqrt(8192.0)
            r0, R, _ = row_block(8192, dist, scale)
            A = _t(datagen.uniform(datagen.SEEDS["mm_A"], (R, 8192), -s, s, offset=r0 * 8192))
            B = _t(datagen.uniform(datagen.SEEDS["mm_B"], (8192, 8192), -s, s))
            C = torch.empty((R, 8192), device="cuda", dtype=torch.float16 if out16 else torch.float32)
            self.flops = 2.0 * R * 8192 * 8192
            self.name = f"matmul 8192x8192x8192 {dtype}"
        if dtype == "f16":
            A, B = A.half(), B.half()
            self.prec = abi.MM_FP16_F32ACC
            self.name += (" (fp32 accumulate, fp16 out: the input dtype, as the drop-in batch_matmul returns)"
                          if out16 else " (fp32 accumulate, fp32 out)")
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


def _launches(wl) -> int:
    """Kernels launched so far by the workload's library contexts."""
    n = wl.ctx.launch_count()
    if getattr(wl, "group", None) is not None:
        n += wl.xctx.launch_count()
    return n


def time_steps(wl, dist: Dist, stream, steps: int, warmup: int, sampler=None, use_graph=True, timeline=None):
    """Times `steps` steps on `stream` with CUDA events; returns the max over
    ranks (ms), the kernel launches in the timed steps and the graph(s).

    A step's local kernel calls are replayed from CUDA graphs; a workload
    with an exchange (ReduceWorkload under sharding) replays two graphs --
    the partials of the exchanged reductions, then the local reductions --
    with the combine started between them on its own stream and the
    finishing calls issued after it.  With a `timeline` dict (sharded
    workloads), it also receives rank 0's median per-step times (ms from the
    step's start) at which the partials, the combines, the local reductions
    and the finishing calls ended (CUDA events; the events themselves sit
    between the graphs and do not change the work)."""
    import torch
    with torch.cuda.stream(stream):
        for _ in range(warmup):
            wl.step()
        torch.cuda.synchronize()
        # launches per step, counted by the library on one eager step
        l0 = _launches(wl)
        wl.step()
        torch.cuda.synchronize()
        per_step = _launches(wl) - l0
        split = use_graph and getattr(wl, "sharded", False)
        g = None
        if split:
            g = (capture(lambda: wl.compute(wl.calls_x), stream), capture(lambda: wl.compute(wl.calls_l), stream))
        elif use_graph:
            g = capture(wl.compute, stream)
        torch.cuda.synchronize()
        dist.barrier()
        torch.cuda.synchronize()
        start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        if sampler:
            sampler.__enter__()
        start.record(stream)
        marks = []
        for _ in range(steps):
            if split:
                ev = [torch.cuda.Event(enable_timing=True) for _ in range(5)] if timeline is not None else None
                if ev:
                    ev[0].record(stream)
                g[0].replay()
                if ev:
                    ev[1].record(stream)
                done = wl.exchange_start()
                if ev:
                    ev[2].record(wl.xstream)
                g[1].replay()
                if ev:
                    ev[3].record(stream)
                wl.exchange_finish(done)
                if ev:
                    ev[4].record(stream)
                    marks.append(ev)
            elif g is not None:
                g.replay()
                wl.exchange()
            else:
                wl.step()
        end.record(stream)
        torch.cuda.synchronize()
        if sampler:
            sampler.__exit__()
    ms = start.elapsed_time(end)
    if marks and timeline is not None:
        rows = [[e[0].elapsed_time(x) for x in e[1:]] for e in marks]
        med = [sorted(r[i] for r in rows)[len(rows) // 2] for i in range(4)]
        timeline.update({k: round(v, 3) for k, v in zip(
            ("partials_end_ms", "combines_end_ms", "local_end_ms", "finish_end_ms"), med)})
    dist.barrier()
    return dist.max(ms), per_step * steps, g


def family_times(wl, stream, reps: int = 5):
    """Average device duration of one launch of each kernel family, per input
    dtype: the family's calls of one step captured alone in a CUDA graph and
    replayed."""
    import torch
    # each call's family is the kernel the library chose for it
    fams = {}
    with torch.cuda.stream(stream):
        for c in wl.calls:
            wl.compute([c])
            fams.setdefault(f"{wl.ctx.last_kernel()}[{c.dt}]", []).append(c)
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
            out[fam] = {"launches": len(calls), "ms": ms, "bytes": sum(c.nbytes for c in calls)}
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


def read_only_reference(stream, reps: int = 10) -> dict:
    """A read-only HBM stream for comparison with the copy peak: torch's sum
    over 2 GiB of binary32 (a library kernel, not this project's), CUDA
    events around `reps` launches after warm-up."""
    import torch
    x = torch.ones(1 << 29, device="cuda")
    with torch.cuda.stream(stream):
        for _ in range(3):
            x.sum()
        torch.cuda.synchronize()
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record(stream)
        for _ in range(reps):
            x.sum()
        b.record(stream)
        torch.cuda.synchronize()
    gbs = x.numel() * 4 * reps / (a.elapsed_time(b) / 1e3) / 1e9
    del x
    torch.cuda.empty_cache()
    return {"gbs": round(gbs, 1), "how": "torch.sum over 2 GiB fp32 (reads only), CUDA events, 10 launches"}


def roofline_from_families(fam, hbm_peak, peak_kind, read_ref=None):
    total = sum(f["ms"] for f in fam.values())
    dom = max(fam, key=lambda k: fam[k]["ms"])
    f = fam[dom]
    per_launch_ms = f["ms"] / f["launches"]
    achieved = f["bytes"] / (f["ms"] / 1e3) / 1e9
    traffic_ratios = ncu_traffic()
    ratio = traffic_ratios.get(dom, traffic_ratios.get(dom.split("[")[0]))
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
            "read_only_reference": read_ref,
            "frac_of_read_only": round(achieved / read_ref["gbs"], 4) if read_ref else None,
            "families": {k: {"share": round(v["ms"] / total, 3),
                             "gbs": round(v["bytes"] / (v["ms"] / 1e3) / 1e9, 1),
                             "frac": round(v["bytes"] / (v["ms"] / 1e3) / 1e9 / hbm_peak, 4),
                             "avg_launch_us": round(v["ms"] / v["launches"] * 1e3, 2),
                             "launches": v["launches"]} for k, v in fam.items()}}


# ---------------------------------------------------------------------------
# CPU side (oracle): baseline and the reference arm
# ---------------------------------------------------------------------------
class CpuReduceSample:
    """The headline reductions on one X[64,512,1024] per dtype (fp32 and
    fp16: the configuration's tensor, not a sample of it), through the
    oracle's OpenMP restatement; a step is these 32 reductions."""
    SHAPE = (64, 512, 1024)

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
            "sample": f"the 32 reductions of one X[64,512,1024] fp32 and one fp16 (the configuration's tensor), "
                      f"{n} passes in {el:.1f} s"}


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
            "config": {"workload": ReduceWorkload.name, "per_step": "one X[64,512,1024] per dtype (32 reductions)",
                       "parallelism": "host cores (OpenMP)"},
            "cpu_baseline": {"value": round(gbs, 3), "unit": "GB/s", "cores": s.cores(), "kind": "port",
                             "sample": "one X[64,512,1024] fp32 and one fp16 per step, 32 reductions"},
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
                "reduce_axis2": 2, "reduce_axis0_f16": 0, "reduce_axis1_f16": 1, "reduce_axis2_f16": 2}[which]
        out = torch.empty(abi.reduced_shape(tuple(x.shape), axis, False), dtype=x.dtype, device="cuda")
        for _ in range(reps):
            ctx.reduce(abi.RED_SUM, d(x), abi.AXIS_ALL if axis is None else axis, False, d(out))
    elif which == "chain_add":
        A = _t(datagen.uniform(1, (4096, 4096), -1, 1))
        B = _t(datagen.uniform(2, (1, 4096), -1, 1))
        out = torch.empty_like(A)
        for _ in range(reps):
            ctx.binary(abi.OP_ADD, d(A), d(B), d(out))
    elif which in ("view_rows", "view_cols", "cast_f16"):
        X = _t(datagen.uniform(5, (8192, 8192), -1, 1))
        if which == "cast_f16":
            Y = torch.empty((8192, 8192), dtype=torch.float16, device="cuda")
            for _ in range(reps):
                ctx.cast(d(X), d(Y))
        else:
            # X[5::3, 1::2]: rows read along k (view_rows, axis 1) or a thread per column (view_cols, axis 0)
            v = abi.make_desc(X.data_ptr() + (5 * 8192 + 1) * 4, abi.F32, (2729, 4096), (3 * 8192, 2))
            axis = 1 if which == "view_rows" else 0
            out = torch.empty(abi.reduced_shape((2729, 4096), axis, False), device="cuda")
            for _ in range(reps):
                ctx.reduce(abi.RED_SUM, v, axis, False, d(out))
    elif which in ("chain_pow", "chain_relu"):
        A = _t(datagen.uniform(1, (4096, 4096), -1, 1))
        out = torch.empty_like(A)
        for _ in range(reps):
            if which == "chain_pow":
                ctx.binary_scalar(abi.OP_POW, d(A), 2.0, d(out))
            else:
                ctx.unary(abi.UN_RELU, d(A), d(out))
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
    elif which == "matmul_ffma":
        s = 1.0 / np.sqrt(8192.0)
        A = _t(datagen.uniform(6, (8192, 8192), -s, s))
        B = _t(datagen.uniform(7, (8192, 8192), -s, s))
        C = torch.empty((8192, 8192), device="cuda")
        for _ in range(reps):
            ctx.matmul(d(A), d(B), d(C), abi.MM_FP32_FFMA)
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
    ap.add_argument("--no-extras", action="store_true", help="skip the other workloads")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--workload", default="reduce",
                    choices=["reduce", "chain", "gather", "layernorm", "matmul_f16", "matmul_f32"])
    ap.add_argument("--timeline", action="store_true",
                    help="sharded runs: add rank 0's median per-step timeline (partials, combines, local, finish)")
    ap.add_argument("--no-overlap", action="store_true",
                    help="reductions wait for the previous kernel at their start (qsml_set_overlap off)")
    ap.add_argument("--single", default=None,
                    choices=["reduce_all", "reduce_axis0", "reduce_axis1", "reduce_axis2", "reduce_all_f16",
                             "reduce_axis0_f16", "reduce_axis1_f16", "reduce_axis2_f16", "chain_pow", "chain_relu",
                             "matmul_ffma", "view_rows", "view_cols", "cast_f16",
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
    # independent reductions on the stream overlap (only library kernels and
    # copies run on it)
    ctx.set_overlap(not args.no_overlap)
    hbm, tf_burst, tf_sus, peak_kind = peaks()

    wl = {"reduce": lambda: ReduceWorkload(ctx, dist), "chain": lambda: ChainWorkload(ctx, dist),
          "gather": lambda: GatherWorkload(ctx, dist), "layernorm": lambda: LayerNormWorkload(ctx, dist),
          "matmul_f16": lambda: MatmulWorkload(ctx, dist, "f16", False),
          "matmul_f32": lambda: MatmulWorkload(ctx, dist, "f32", False)}[args.workload]()

    sampler = ClockSampler(dist.local)
    timeline = {} if args.timeline else None
    ms, launches, graph = time_steps(wl, dist, stream, args.steps, args.warmup, sampler=sampler, timeline=timeline)
    del graph
    units = wl.units_per_step * args.steps * dist.world
    value = units / (ms / 1e3) / (1e9 if wl.unit == "GB/s" else 1e12)

    sharded = getattr(wl, "sharded", False)
    line = {"metric": METRIC, "value": round(value, 2), "unit": wl.unit, "n_gpus": dist.world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(ms / args.steps, 4),
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
            "dtype": "f32+f16 (fp32 accumulate)" if args.workload == "reduce" else "f32",
            "data": "synthetic (seeded, counter-based generator)",
            "config": {"workload": wl.name, "parallelism": f"dp{dist.world}",
                       "l2": "inputs larger than L2: 8 distinct X per dtype per step (1.5 GB), batch entry innermost in the call order so no call finds its input in L2"
                       if args.workload == "reduce" else "inputs larger than L2",
                       "calls_per_step": len(getattr(wl, "calls", [])) or 1,
                       "launch": "each step's kernel calls replayed from one CUDA graph"
                       if not sharded else
                       "X row-sharded (each rank X[64,512,1024] of X[64N,512,1024]); per step: graph 1 = the "
                       "binary32 partials of the axis-0 and full reductions (sum, max, min; means are finished "
                       "from the combined sums), then qsml_allreduce_partials of the three partial buffers on a "
                       "second context's stream (NCCL over NVLink) while graph 2 = the axis-1/2 reductions runs, "
                       "then qsml_finish_partial of the outputs"},
            "gpu_launches": launches, "clocks": sampler.summary()}
    line["config"]["overlap"] = ("off" if args.no_overlap else
                                 "qsml_set_overlap(ctx, 1): a reduction sharing no buffer with the library kernels "
                                 "still running on the stream starts at once and waits for them at its end")
    if args.workload == "reduce":
        line["roofline"] = roofline_from_families(family_times(wl, stream), hbm, peak_kind,
                                                  read_only_reference(stream))
        if sharded:
            line["exchange"] = exchange_alone(wl, dist, stream)
            if timeline:
                line["exchange"]["timeline_rank0"] = timeline
    if hasattr(wl, "e2e_step"):
        e_steps = max(2, min(args.steps, 5))
        ems = time_e2e(wl, dist, stream, e_steps, 1)
        ev = wl.units_per_step * e_steps * dist.world / (ems / 1e3) / 1e9
        line["e2e"] = {"value": round(ev, 2), "unit": wl.unit, "h2d_bytes_per_step": wl.h2d_bytes,
                       "d2h_bytes_per_step": wl.d2h_bytes, "ms_per_step": round(ems / e_steps, 3),
                       "path": "pinned host -> qsml_h2d of each batch entry's X (fp32) on a second context's "
                               "stream, qsml_cast to its fp16 copy there -> the step's qsml_reduce calls of each "
                               "entry as soon as both have landed -> "
                               "qsml_d2h_async of each entry's results on a third stream"
                               + ("; the exchanged outputs after qsml_allreduce_partials / "
                                  "qsml_finish_partial" if sharded else "") + ", per step"}
    if hasattr(wl, "close_exchange"):
        wl.close_exchange()

    if not args.no_extras and args.workload == "reduce":
        del wl
        torch.cuda.empty_cache()
        line["other_workloads"] = run_extras(ctx, dist, stream, hbm, tf_burst)

    if dist.world == 1 and not args.no_extras and args.workload == "reduce":
        torch.cuda.synchronize()
        torch.cuda.empty_cache()
        line["cpp_api"] = run_cpp_api()

    if dist.world == 1 and dist.rank == 0 and not args.no_cpu_baseline and args.workload == "reduce":
        line["cpu_baseline"] = cpu_baseline()

    torch.cuda.synchronize()
    ctx.close()
    if dist.rank == 0:
        print(json.dumps(line), flush=True)
    dist.close()


CPP_API_PROGRAM = os.path.join(ROOT, "quasarml_b200", "cpp", "_build", "bench_configs")


def run_cpp_api(timeout_s: int = 600) -> dict:
    """The configurations through the unchanged C++ qsml:: API (a separate
    process: quasarml_b200/cpp/examples/bench_configs.cpp, every op allocating
    its result as a reference user's code does), wall clock around many steps
    with qsml::synchronize() on both sides."""
    import subprocess
    if not os.path.exists(CPP_API_PROGRAM):
        return {"error": f"{CPP_API_PROGRAM} not built"}
    try:
        r = subprocess.run([CPP_API_PROGRAM], capture_output=True, text=True, timeout=timeout_s)
    except subprocess.TimeoutExpired:
        return {"error": "timed out"}
    out = {}
    for ln in r.stdout.splitlines():
        if ln.startswith("{"):
            j = json.loads(ln)
            out[j.pop("key")] = j
    if r.returncode != 0:
        out["error"] = f"rc={r.returncode}: {r.stderr[-300:]}"
    out["path"] = "C++ qsml:: API (QuasarML.h), results allocated per op from the caching allocator"
    return out


def exchange_alone(wl, dist: Dist, stream, reps: int = 5) -> dict:
    """The step's combine alone: the three qsml_allreduce_partials (with their
    key passes) timed on their stream, max over ranks."""
    import torch
    wl.init_exchange()
    with torch.cuda.stream(stream):
        for _ in range(2):
            wl.exchange()
        torch.cuda.synchronize()
        dist.barrier()
        torch.cuda.synchronize()
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record(wl.xstream)
        for _ in range(reps):
            wl.exchange_start()
        b.record(wl.xstream)
        torch.cuda.synchronize()
    ms = dist.max(a.elapsed_time(b) / reps)
    nbytes = sum(f.numel() * 4 for f in wl.flat.values())
    return {"ms": round(ms, 4), "bytes_per_rank": nbytes, "collectives": len(wl.flat),
            "what": "qsml_allreduce_partials of the sum / max / min partial buffers (binary32 sums, "
                    "order-preserving 32-bit max/min keys), timed alone on its stream"}


EXTRAS = (("elementwise_chain", lambda c, d, s: ChainWorkload(c, d, scale=s), 10),
          ("elementwise_chain_fused", lambda c, d, s: FusedChainWorkload(c, d, scale=s), 20),
          ("gather", lambda c, d, s: GatherWorkload(c, d, scale=s), 20),
          ("layernorm", lambda c, d, s: LayerNormWorkload(c, d, scale=s), 20),
          ("argmax_argmin", lambda c, d, s: ArgReduceWorkload(c, d, scale=s), 20),
          ("reduce_views", lambda c, d, s: ReduceViewWorkload(c, d, scale=s), 20),
          ("softmax", lambda c, d, s: SoftmaxWorkload(c, d, scale=s), 20),
          ("matmul_f16_8192", lambda c, d, s: MatmulWorkload(c, d, "f16", False, scale=s), 5),
          ("matmul_f32_8192_3xtf32", lambda c, d, s: MatmulWorkload(c, d, "f32", False, scale=s), 5),
          ("matmul_f32_8192_ffma", lambda c, d, s: MatmulWorkload(c, d, "f32", False, "ffma", scale=s), 3),
          ("batched_matmul_f16", lambda c, d, s: MatmulWorkload(c, d, "f16", True, scale=s), 5),
          ("batched_matmul_f16_out16", lambda c, d, s: MatmulWorkload(c, d, "f16", True, scale=s, out16=True), 5),
          ("batched_matmul_f32_3xtf32", lambda c, d, s: MatmulWorkload(c, d, "f32", True, scale=s), 5))


def fp32_ceiling(w, tf_burst: float):
    """(TFLOP/s, what) for the binary32 matmul paths, whose ceiling is not the
    fp16 tensor rate: the FFMA pipe (SMs x 128 lanes x 2 flops x the maximum
    SM clock) for the CUDA-core kernel, one sixth of the fp16 rate for 3xTF32
    (tf32 runs at half the fp16 rate and each product is three MMAs)."""
    import torch
    from quasarml_b200 import abi
    prec = getattr(w, "prec", None)
    if prec == abi.MM_FP32_FFMA:
        mhz = 1965.0
        p = os.path.join(ROOT, "MEASURED_PEAKS.json")
        if os.path.exists(p):
            mhz = float(json.load(open(p)).get("sm_max_mhz", mhz))
        sms = torch.cuda.get_device_properties(torch.cuda.current_device()).multi_processor_count
        return (round(sms * 128 * 2 * mhz * 1e6 / 1e12, 1), f"FFMA pipe: {sms} SMs x 128 x 2 x {mhz:.0f} MHz")
    if prec == abi.MM_FP32_3XTF32:
        return (round(tf_burst / 6.0, 1), "3xTF32: measured fp16 tensor rate / 2 (tf32) / 3 (products)")
    return None


def run_extras(ctx, dist: Dist, stream, hbm: float, tf_burst: float) -> dict:
    """The other configurations, each row-sharded over the ranks: weak
    scaling at every N (each rank the configuration's size), and at N>1 also
    strong scaling (the configuration's tensor split N ways).  Every rank
    builds the workload, all agree it was built, then all time it.  At N>1
    rank 0 first times each weak-scaling workload alone (the same per-rank
    work on one GPU, in this run), which gives efficiency_vs_one_gpu =
    per-GPU value at N / that one-GPU value."""
    import torch
    extras = {}
    scales = ("weak",) if dist.world == 1 else ("weak", "strong")
    for scale in scales:
        for key, mk, st in EXTRAS:
            name = key if scale == "weak" else key + "_strong"
            w, err = None, None
            try:
                w = mk(ctx, dist, scale)
            except Exception as e:  # reported, never hidden
                err = repr(e)[:300]
            if dist.max(1.0 if err else 0.0) > 0:
                extras[name] = {"error": err or "failed on another rank"}
                w = None
                torch.cuda.synchronize()
                torch.cuda.empty_cache()
                continue
            scale_unit = 1e9 if w.unit == "GB/s" else 1e12
            alone = None
            err = None
            if scale == "weak" and dist.world > 1:
                # the same per-rank work on one GPU in this run: rank 0 alone
                # while the other ranks wait at the barrier
                if dist.rank == 0:
                    try:
                        ms_a, _, g = time_steps(w, Dist.single(), stream, st, 3)
                        del g
                        alone = w.units_per_step * st / (ms_a / 1e3) / scale_unit
                    except Exception as e:
                        err = repr(e)[:300]
                dist.barrier()
                if dist.max(1.0 if err else 0.0) > 0:
                    err = err or "failed on rank 0"
            if err is None:
                try:
                    ms_x, l_x, g = time_steps(w, dist, stream, st, 3)
                    del g
                except Exception as e:  # a library error of this workload: the same on every rank
                    err = repr(e)[:300]
            if err is not None:
                extras[name] = {"error": err}
                del w
                torch.cuda.synchronize()
                torch.cuda.empty_cache()
                continue
            units = w.units_per_step * dist.world if scale == "weak" else dist.sum(w.units_per_step)
            v = units * st / (ms_x / 1e3) / scale_unit
            peak = hbm if w.unit == "GB/s" else tf_burst
            extras[name] = {"workload": w.name, "scaling": scale, "value": round(v, 2),
                            "per_gpu": round(v / dist.world, 2), "unit": w.unit,
                            "frac_of_peak": round(v / dist.world / peak, 4), "peak": peak,
                            "ms_per_step": round(ms_x / st, 3), "launches_per_step": l_x // st}
            ceiling = fp32_ceiling(w, tf_burst)
            if ceiling:
                extras[name]["ceiling"] = ceiling
                extras[name]["frac_of_ceiling"] = round(v / dist.world / ceiling[0], 4)
            if alone:
                extras[name]["one_gpu_same_run"] = round(alone, 2)
                extras[name]["efficiency_vs_one_gpu"] = round(v / dist.world / alone, 4)
            del w
            torch.cuda.synchronize()
            torch.cuda.empty_cache()
    return extras


if __name__ == "__main__":
    main()
