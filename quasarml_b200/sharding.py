"""Data-parallel sharding of the reductions across ranks (one process per GPU).

A global tensor X[N*64, 512, 1024] is split along axis 0; rank r holds rows
[64r, 64r+64) (for batch entry b, elements start at flat offset
(b*world + r) * shard_numel of the seeded stream).  Per-rank results combine:

* axis 1 / axis 2: each rank's output is its own slice of the global output,
  no exchange;
* axis 0 / all elements: partial outputs are all-reduced -- sum and max/min
  with the matching reduction; mean as the all-reduced sum of per-rank means
  times 1/world (every shard has the same size).

The same plan drives bench.py (NCCL over NVLink) and the CPU test with gloo.
"""
from __future__ import annotations

SUM, MEAN, MAX, MIN = range(4)  # qsml_reduce codes


def shard_offset(batch_index: int, world: int, rank: int, shard_numel: int) -> int:
    """Flat offset in the seeded stream of rank `rank`'s shard of entry `batch_index`."""
    return (batch_index * world + rank) * shard_numel


def needs_exchange(axis) -> bool:
    """Axis-0 and full reductions combine partials across ranks."""
    return axis is None or axis == 0 or axis == -1000


def collective(op: int) -> str:
    """The all-reduce that combines per-rank partials of reduction `op`."""
    return {SUM: "sum", MEAN: "sum", MAX: "max", MIN: "min"}[op]


def post_scale(op: int, world: int) -> float:
    """Factor applied after the all-reduce (mean of equal-size shards)."""
    return 1.0 / world if op == MEAN else 1.0


def exchange(dist, buffers_by_collective: dict, scale_views=(), world: int = 1, scale_fn=None) -> None:
    """All-reduces each flat buffer with its collective, then rescales the
    mean views.  `dist` is torch.distributed; `scale_fn(view, factor)` scales
    in place (the GPU path passes a qsml_binary_scalar call)."""
    ops = {"sum": dist.ReduceOp.SUM, "max": dist.ReduceOp.MAX, "min": dist.ReduceOp.MIN}
    for key, buf in buffers_by_collective.items():
        grp = key[-1] if isinstance(key, tuple) else key
        dist.all_reduce(buf, op=ops[grp])
    if world > 1:
        for v in scale_views:
            if scale_fn is None:
                v.mul_(1.0 / world)
            else:
                scale_fn(v, 1.0 / world)
