// Reductions (QuasarML/src/Ops/Reduction.h).  Axis max/min are real here
// (stubs in the reference); accumulation is fp32, results keep the input
// dtype and are run-to-run deterministic.
#pragma once

#include <memory>

#include "../Core/Device.h"
#include "../Core/Tensor.h"

namespace QuasarML {
namespace Ops {

QS_API std::shared_ptr<Tensor> sum(Device& device, std::shared_ptr<Tensor> a);
QS_API std::shared_ptr<Tensor> sum(Device& device, std::shared_ptr<Tensor> a, i32 axis, bool keepdims = false);
QS_API std::shared_ptr<Tensor> mean(Device& device, std::shared_ptr<Tensor> a);
QS_API std::shared_ptr<Tensor> mean(Device& device, std::shared_ptr<Tensor> a, i32 axis, bool keepdims = false);
QS_API std::shared_ptr<Tensor> max(Device& device, std::shared_ptr<Tensor> a);
QS_API std::shared_ptr<Tensor> max(Device& device, std::shared_ptr<Tensor> a, i32 axis, bool keepdims = false);
QS_API std::shared_ptr<Tensor> min(Device& device, std::shared_ptr<Tensor> a);
QS_API std::shared_ptr<Tensor> min(Device& device, std::shared_ptr<Tensor> a, i32 axis, bool keepdims = false);
QS_API std::shared_ptr<Tensor> prod(Device& device, std::shared_ptr<Tensor> a);
QS_API std::shared_ptr<Tensor> argmax(Device& device, std::shared_ptr<Tensor> a, i32 axis = -1);
QS_API std::shared_ptr<Tensor> argmin(Device& device, std::shared_ptr<Tensor> a, i32 axis = -1);

}  // namespace Ops
}  // namespace QuasarML
