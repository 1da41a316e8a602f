"""Data-parallel sharding of the reductions across ranks (one process per GPU).

A global tensor X[N*64, 512, 1024] is split along axis 0; rank r holds rows
[64r, 64r+64) (for batch entry b, elements start at flat offset
(b*world + r) * shard_numel of the seeded stream).  Per-rank results combine:

* axis 1 / axis 2: each rank's output is its own slice of the global output,
  no exchange;
* axis 0 / all elements: partial outputs are all-reduced -- sums and max/min
  with the matching reduction; means as the all-reduced sum of per-rank means
  times 1/world (every shard has the same size).

Exchanged outputs live in one flat buffer per (dtype, group), group one of
"sum", "mean", "max", "min", so a step issues one all-reduce per buffer and
one rescale per mean buffer.  The same plan drives bench.py (NCCL over
NVLink) and the CPU test with gloo.
"""
from __future__ import annotations

SUM, MEAN, MAX, MIN = range(4)  # qsml_reduce codes


def shard_offset(batch_index: int, world: int, rank: int, shard_numel: int) -> int:
    """Flat offset in the seeded stream of rank `rank`'s shard of entry `batch_index`."""
    return (batch_index * world + rank) * shard_numel


def needs_exchange(axis) -> bool:
    """Axis-0 and full reductions combine partials across ranks."""
    return axis is None or axis == 0 or axis == -1000


def group(op: int) -> str:
    """Flat-buffer group of reduction `op`'s exchanged outputs."""
    return {SUM: "sum", MEAN: "mean", MAX: "max", MIN: "min"}[op]


def _group_of(key) -> str:
    return key[-1] if isinstance(key, tuple) else key


def exchange_start(dist, buffers: dict) -> list:
    """Starts the all-reduce of every flat buffer (keys end in the group name)
    and returns the work handles.  With NCCL the collectives run on NCCL's
    stream after the work already enqueued on the current stream, so kernels
    enqueued next overlap them."""
    ops = {"sum": dist.ReduceOp.SUM, "mean": dist.ReduceOp.SUM, "max": dist.ReduceOp.MAX,
           "min": dist.ReduceOp.MIN}
    return [dist.all_reduce(buf, op=ops[_group_of(key)], async_op=True) for key, buf in buffers.items()]


def exchange_finish(works: list, buffers: dict, world: int, scale_fn=None) -> None:
    """Waits for the all-reduces (the current stream waits; the host does not
    block with NCCL), then scales the mean buffers by 1/world.  `scale_fn(key,
    factor)` rescales a buffer in place (the GPU path issues one
    qsml_binary_scalar per buffer); without it the tensor's mul_ is used."""
    for w in works:
        w.wait()
    if world > 1:
        for key, buf in buffers.items():
            if _group_of(key) == "mean":
                if scale_fn is None:
                    buf.mul_(1.0 / world)
                else:
                    scale_fn(key, 1.0 / world)


def exchange(dist, buffers: dict, world: int, scale_fn=None) -> None:
    """exchange_start + exchange_finish."""
    exchange_finish(exchange_start(dist, buffers), buffers, world, scale_fn)
