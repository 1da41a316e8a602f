// Multi-GPU helpers of this backend (the reference is single-GPU): combine
// per-device partial results of sharded work.
#pragma once

#include <memory>
#include <vector>

#include "../Common/Types.h"

namespace QuasarML {

class Tensor;

enum class ReduceOp : u32 { Sum = 0, Mean = 1, Max = 2, Min = 3, Prod = 4 };

namespace Ops {

// In-place all-reduce across devices: tensors[i] lives on its own device (one
// process driving them all), every tensor has the same shape and dtype and is
// contiguous; afterwards each holds the combination of all of them.  The NCCL
// group for a set of devices is created on first use and kept until
// DeviceManager::shutdown.  Mean divides the sum by tensors.size().
QS_API void all_reduce(const std::vector<std::shared_ptr<Tensor>>& tensors, ReduceOp op = ReduceOp::Sum);

// Sum / mean / max / min of a tensor split by rows over devices: blocks[i]
// lives on its own device (one process driving them all) and holds a block of
// the global tensor's rows (the other dims agree; blocks may differ in rows,
// or be empty).  Over axis 0, or over all elements (the overload without an
// axis), every device receives the whole result; over any other axis, each
// device receives its rows of the result.  Partials combine in binary32
// (binary16 inputs included) and max/min as exact order-preserving keys, so
// the result equals the single-device reduction of the whole tensor up to the
// summation order; a mean divides by the global count (sum * (1/n)).
QS_API std::vector<std::shared_ptr<Tensor>> sharded_reduce(const std::vector<std::shared_ptr<Tensor>>& blocks,
                                                           ReduceOp op, i32 axis, bool keepdims = false);
QS_API std::vector<std::shared_ptr<Tensor>> sharded_reduce(const std::vector<std::shared_ptr<Tensor>>& blocks,
                                                           ReduceOp op);

// Splits host data of `shape` by rows over `devices` (the balanced split of
// qsml_shard_rows) and uploads each block to its device.
QS_API std::vector<std::shared_ptr<Tensor>> scatter_rows(const void* host, const std::vector<u32>& shape,
                                                         DataType dtype, const std::vector<Device*>& devices);

// Releases the cached device groups (DeviceManager::shutdown calls it).
QS_API void release_device_groups();

}  // namespace Ops
}  // namespace QuasarML
