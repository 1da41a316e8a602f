// Shape manipulation (QuasarML/src/Ops/Manipulation.h).  reshape/flatten/
// squeeze/unsqueeze and slice are views; concat/stack/broadcast_to/copy and
// contiguous are device copies (the reference round-trips through the host).
#pragma once

#include <memory>
#include <vector>

#include "../Core/Device.h"
#include "../Core/Tensor.h"

namespace QuasarML {
namespace Ops {

QS_API std::shared_ptr<Tensor> reshape(Device& device, std::shared_ptr<Tensor> a, const std::vector<u32>& new_shape);
QS_API std::shared_ptr<Tensor> flatten(Device& device, std::shared_ptr<Tensor> a);
QS_API std::shared_ptr<Tensor> squeeze(Device& device, std::shared_ptr<Tensor> a);
QS_API std::shared_ptr<Tensor> squeeze(Device& device, std::shared_ptr<Tensor> a, i32 dim);
QS_API std::shared_ptr<Tensor> unsqueeze(Device& device, std::shared_ptr<Tensor> a, i32 dim);
QS_API std::shared_ptr<Tensor> concat(Device& device, const std::vector<std::shared_ptr<Tensor>>& tensors,
                                      i32 axis = 0);
QS_API std::shared_ptr<Tensor> stack(Device& device, const std::vector<std::shared_ptr<Tensor>>& tensors,
                                     i32 axis = 0);
QS_API std::shared_ptr<Tensor> slice(Device& device, std::shared_ptr<Tensor> a, i32 axis, u64 start, u64 end);
QS_API std::shared_ptr<Tensor> slice(Device& device, std::shared_ptr<Tensor> a, i32 axis, u64 start, u64 end,
                                     u64 step);
QS_API std::shared_ptr<Tensor> broadcast_to(Device& device, std::shared_ptr<Tensor> a, const std::vector<u32>& shape);
QS_API std::shared_ptr<Tensor> copy(Device& device, std::shared_ptr<Tensor> a);
QS_API std::shared_ptr<Tensor> contiguous(Device& device, std::shared_ptr<Tensor> a);
// A new tensor holding `a` converted to `dtype` (F32 <-> F16; same dtype copies).
QS_API std::shared_ptr<Tensor> cast(Device& device, std::shared_ptr<Tensor> a, DataType dtype);

}  // namespace Ops
}  // namespace QuasarML
