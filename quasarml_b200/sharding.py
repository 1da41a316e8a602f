"""Row sharding of the workloads across ranks (one process per GPU).

Every workload splits its global tensor along axis 0 and gives each rank a
contiguous block of rows (qsml_shard_rows; in the benchmark every rank holds
the configuration's full size, so the global tensor has N times its rows --
weak scaling).  For batch entry b, rank r's block starts at flat offset
(b*world + r) * shard_numel of the seeded stream, so the global tensor is the
same whatever N.

Reductions (the only workload with an exchange):

* axis 1 / axis 2: each rank's output is its own row block of the global
  output, no exchange;
* axis 0 / all elements: each rank computes a binary32 partial with
  qsml_reduce (SUM for sum and mean, MAX / MIN for max / min; binary16 inputs
  give binary32 partials too, so sums are never combined in binary16), the
  partials are packed into one flat buffer per combine group ("sum", "max",
  "min": one qsml_allreduce_partials each, whatever the dtypes) and combined
  across ranks, and qsml_finish_partial writes each output in its dtype.  A
  mean is finished from the combined sum of the same input and axis as
  sum * (1.0f / (float)n), n the elements reduced over all ranks -- the
  reference's definition of mean (Ops/Reduction.cpp:347-356) -- so it needs
  no partial of its own.

ExchangePlan lays this out; bench.py drives it with the library (NCCL over
NVLink) and tests/test_dist_cpu.py drives the same plan with gloo on CPU.
"""
from __future__ import annotations

SUM, MEAN, MAX, MIN = range(4)  # qsml_reduce codes
AXIS_ALL = -1000

GROUP_OF = {SUM: "sum", MEAN: "sum", MAX: "max", MIN: "min"}


def shard_offset(batch_index: int, world: int, rank: int, shard_numel: int) -> int:
    """Flat offset in the seeded stream of rank `rank`'s shard of entry `batch_index`."""
    return (batch_index * world + rank) * shard_numel


def shard_rows(rows: int, world: int, rank: int) -> tuple:
    """(begin, count): the balanced contiguous split of qsml_shard_rows (the
    first rows % world ranks hold one row more)."""
    base, extra = divmod(rows, world)
    return rank * base + min(rank, extra), base + (1 if rank < extra else 0)


def needs_exchange(axis) -> bool:
    """Axis-0 and full reductions combine partials across ranks."""
    return axis is None or axis == 0 or axis == AXIS_ALL


class ExchangePlan:
    """Partials and finishing of the exchanged reductions of one step.

    add(key, op, axis, count, n) registers the output of reduction `op` over
    `axis` of input `key` (any hashable naming the input), `count` elements,
    n elements reduced into each over all ranks.  Afterwards:

    * partials: (key, axis, group, offset, count) -- one local qsml_reduce
      into the flat buffer of `group` at `offset` per entry; a mean shares the
      sum's entry (its sum is added for it if the step has none);
    * finishes: (op, group, offset, count, n, out_index) -- one
      qsml_finish_partial per registered output, in registration order;
    * sizes[group]: elements of each flat buffer.
    """

    def __init__(self):
        self.sizes = {"sum": 0, "max": 0, "min": 0}
        self.partials = []
        self.finishes = []
        self._slot = {}

    def _partial(self, key, axis, group, count):
        k = (key, axis, group)
        if k not in self._slot:
            off = self.sizes[group]
            self.sizes[group] += count
            self._slot[k] = off
            self.partials.append((key, axis, group, off, count))
        return self._slot[k]

    def add(self, key, op: int, axis, count: int, n: int) -> int:
        group = GROUP_OF[op]
        off = self._partial(key, axis, group, count)
        self.finishes.append((op, group, off, count, n, len(self.finishes)))
        return len(self.finishes) - 1
