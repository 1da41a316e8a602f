// Linear algebra (QuasarML/src/Ops/LinAlg.h).  matmul of F16 inputs runs on
// the tcgen05 tensor cores with fp32 accumulation; transpose is a view.
#pragma once

#include <memory>

#include "../Core/Device.h"
#include "../Core/Tensor.h"

namespace QuasarML {
namespace Ops {

QS_API std::shared_ptr<Tensor> matmul(Device& device, std::shared_ptr<Tensor> a, std::shared_ptr<Tensor> b);
// Same, with the result's dtype chosen (F32 keeps the fp32 accumulator of F16 inputs).
QS_API std::shared_ptr<Tensor> matmul(Device& device, std::shared_ptr<Tensor> a, std::shared_ptr<Tensor> b,
                                      DataType out_dtype);
QS_API std::shared_ptr<Tensor> batch_matmul(Device& device, std::shared_ptr<Tensor> a, std::shared_ptr<Tensor> b);
QS_API std::shared_ptr<Tensor> dot(Device& device, std::shared_ptr<Tensor> a, std::shared_ptr<Tensor> b);
QS_API std::shared_ptr<Tensor> transpose(Device& device, std::shared_ptr<Tensor> a);
QS_API std::shared_ptr<Tensor> transpose(Device& device, std::shared_ptr<Tensor> a, i32 dim0, i32 dim1);
QS_API std::shared_ptr<Tensor> outer(Device& device, std::shared_ptr<Tensor> a, std::shared_ptr<Tensor> b);
QS_API std::shared_ptr<Tensor> layer_norm(Device& device, std::shared_ptr<Tensor> x, std::shared_ptr<Tensor> gamma,
                                          std::shared_ptr<Tensor> beta, f32 eps = 1e-5f);

}  // namespace Ops
}  // namespace QuasarML
