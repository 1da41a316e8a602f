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

// Releases the cached device groups (DeviceManager::shutdown calls it).
QS_API void release_device_groups();

}  // namespace Ops
}  // namespace QuasarML
