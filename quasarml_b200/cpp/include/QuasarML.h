// qsml:: facade of QuasarML (QuasarML/include/QuasarML.h), unchanged in
// names and signatures, over the B200 backend.  Additions: pow, axis-aware
// slice with a step, transpose(x, d0, d1) as a view, contiguous, cast,
// layer_norm, batch_matmul, matmul with an output dtype, cpu_fallback_count,
// row-sharded reductions over several devices.
// The Vulkan-only Kernel type (GLSL pipelines) has no counterpart.
#pragma once

#include <cstdint>
#include <memory>
#include <string>
#include <vector>

#include "Common/Assert.h"
#include "Common/Logger.h"
#include "Common/Types.h"
#include "Core/Device.h"
#include "Core/DeviceManager.h"
#include "Core/Tensor.h"
#include "Ops/Distributed.h"
#include "Ops/Elementwise.h"
#include "Ops/LinAlg.h"
#include "Ops/Manipulation.h"
#include "Ops/Reduction.h"

namespace qsml {

using QuasarML::DataType;
using QuasarML::Device;
using QuasarML::DeviceManager;
using QuasarML::Tensor;
using QuasarML::f32;
using QuasarML::f64;
using QuasarML::i16;
using QuasarML::i32;
using QuasarML::i64;
using QuasarML::i8;
using QuasarML::u16;
using QuasarML::u32;
using QuasarML::u64;
using QuasarML::u8;

using TensorPtr = std::shared_ptr<Tensor>;

namespace detail {
inline Device*& current_device_ptr() {
    static Device* dev = nullptr;
    return dev;
}
}  // namespace detail

inline void init() { QuasarML::Logger::init(); }

inline void shutdown() {
    detail::current_device_ptr() = nullptr;
    DeviceManager::instance().shutdown();
    QuasarML::Logger::shutdown();
}

inline u32 device_count() { return DeviceManager::instance().device_count(); }
inline std::vector<std::string> device_names() { return DeviceManager::instance().device_names(); }

inline void set_device(u32 device_id) {
    DeviceManager::instance().set_default(device_id);
    detail::current_device_ptr() = DeviceManager::instance().get(device_id);
}

inline u32 current_device_id() { return DeviceManager::instance().get_default(); }

inline Device& device() {
    if (!detail::current_device_ptr()) detail::current_device_ptr() = DeviceManager::instance().get(0);
    QS_ASSERT(detail::current_device_ptr(), "No GPU device available");
    return *detail::current_device_ptr();
}

inline Device& device(u32 device_id) {
    Device* dev = DeviceManager::instance().get(device_id);
    QS_ASSERT(dev, "Failed to get device");
    return *dev;
}

inline bool is_valid() { return detail::current_device_ptr() && detail::current_device_ptr()->is_valid(); }
inline void synchronize() { device().synchronize(); }
inline void flush_pending() { device().flush_pending(); }

inline TensorPtr zeros(const std::vector<u32>& shape, DataType dtype = DataType::F32) {
    auto t = device().create_tensor(shape, dtype);
    t->zero();
    return t;
}

inline TensorPtr ones(const std::vector<u32>& shape, DataType dtype = DataType::F32) {
    auto t = device().create_tensor(shape, dtype);
    switch (dtype) {
        case DataType::F32: { f32 v = 1.0f; t->fill(&v); break; }
        case DataType::F16: { u16 v = 0x3C00; t->fill(&v); break; }
        case DataType::I32: case DataType::U32: { i32 v = 1; t->fill(&v); break; }
        case DataType::I16: case DataType::U16: { i16 v = 1; t->fill(&v); break; }
        case DataType::I8: case DataType::U8: { i8 v = 1; t->fill(&v); break; }
    }
    return t;
}

inline TensorPtr empty(const std::vector<u32>& shape, DataType dtype = DataType::F32) {
    return device().create_tensor(shape, dtype);
}

inline TensorPtr tensor(const std::vector<f32>& data, const std::vector<u32>& shape, DataType dtype = DataType::F32) {
    auto t = device().create_tensor(shape, dtype);
    t->upload(data.data(), data.size() * sizeof(f32));
    return t;
}

inline TensorPtr from_data(const void* data, const std::vector<u32>& shape, DataType dtype = DataType::F32) {
    auto t = device().create_tensor(shape, dtype);
    t->upload(data, t->numel() * QuasarML::dtype_size(dtype));
    return t;
}

inline TensorPtr add(TensorPtr a, TensorPtr b) { return QuasarML::Ops::add(device(), a, b); }
inline TensorPtr sub(TensorPtr a, TensorPtr b) { return QuasarML::Ops::subtract(device(), a, b); }
inline TensorPtr mul(TensorPtr a, TensorPtr b) { return QuasarML::Ops::multiply(device(), a, b); }
inline TensorPtr div(TensorPtr a, TensorPtr b) { return QuasarML::Ops::divide(device(), a, b); }
inline TensorPtr pow(TensorPtr a, TensorPtr exponent) { return QuasarML::Ops::pow(device(), a, exponent); }
inline TensorPtr pow(TensorPtr a, f32 exponent) { return QuasarML::Ops::pow(device(), a, exponent); }
inline TensorPtr neg(TensorPtr x) { return QuasarML::Ops::neg(device(), x); }
inline TensorPtr abs(TensorPtr x) { return QuasarML::Ops::abs(device(), x); }
inline TensorPtr add_scalar(TensorPtr x, f32 scalar) { return QuasarML::Ops::add_scalar(device(), x, scalar); }
inline TensorPtr mul_scalar(TensorPtr x, f32 scalar) { return QuasarML::Ops::multiply_scalar(device(), x, scalar); }
inline TensorPtr sqrt(TensorPtr x) { return QuasarML::Ops::sqrt(device(), x); }
inline TensorPtr exp(TensorPtr x) { return QuasarML::Ops::exp(device(), x); }
inline TensorPtr log(TensorPtr x) { return QuasarML::Ops::log(device(), x); }
inline TensorPtr sin(TensorPtr x) { return QuasarML::Ops::sin(device(), x); }
inline TensorPtr cos(TensorPtr x) { return QuasarML::Ops::cos(device(), x); }
inline TensorPtr tanh(TensorPtr x) { return QuasarML::Ops::tanh(device(), x); }
inline TensorPtr relu(TensorPtr x) { return QuasarML::Ops::relu(device(), x); }
inline TensorPtr sigmoid(TensorPtr x) { return QuasarML::Ops::sigmoid(device(), x); }
inline TensorPtr gelu(TensorPtr x) { return QuasarML::Ops::gelu(device(), x); }
inline TensorPtr softmax(TensorPtr x, i32 axis = -1) { return QuasarML::Ops::softmax(device(), x, axis); }

inline TensorPtr sum(TensorPtr x) { return QuasarML::Ops::sum(device(), x); }
inline TensorPtr sum(TensorPtr x, i32 axis, bool keepdims = false) { return QuasarML::Ops::sum(device(), x, axis, keepdims); }
inline TensorPtr mean(TensorPtr x) { return QuasarML::Ops::mean(device(), x); }
inline TensorPtr mean(TensorPtr x, i32 axis, bool keepdims = false) { return QuasarML::Ops::mean(device(), x, axis, keepdims); }
inline TensorPtr max(TensorPtr x) { return QuasarML::Ops::max(device(), x); }
inline TensorPtr max(TensorPtr x, i32 axis, bool keepdims = false) { return QuasarML::Ops::max(device(), x, axis, keepdims); }
inline TensorPtr min(TensorPtr x) { return QuasarML::Ops::min(device(), x); }
inline TensorPtr min(TensorPtr x, i32 axis, bool keepdims = false) { return QuasarML::Ops::min(device(), x, axis, keepdims); }
inline TensorPtr prod(TensorPtr x) { return QuasarML::Ops::prod(device(), x); }
inline TensorPtr argmax(TensorPtr x, i32 axis = -1) { return QuasarML::Ops::argmax(device(), x, axis); }
inline TensorPtr argmin(TensorPtr x, i32 axis = -1) { return QuasarML::Ops::argmin(device(), x, axis); }

inline TensorPtr matmul(TensorPtr a, TensorPtr b) { return QuasarML::Ops::matmul(device(), a, b); }
inline TensorPtr matmul(TensorPtr a, TensorPtr b, DataType out_dtype) { return QuasarML::Ops::matmul(device(), a, b, out_dtype); }
inline TensorPtr batch_matmul(TensorPtr a, TensorPtr b) { return QuasarML::Ops::batch_matmul(device(), a, b); }
inline TensorPtr dot(TensorPtr a, TensorPtr b) { return QuasarML::Ops::dot(device(), a, b); }
inline TensorPtr outer(TensorPtr a, TensorPtr b) { return QuasarML::Ops::outer(device(), a, b); }
inline TensorPtr transpose(TensorPtr x) { return QuasarML::Ops::transpose(device(), x); }
inline TensorPtr transpose(TensorPtr x, i32 d0, i32 d1) { return QuasarML::Ops::transpose(device(), x, d0, d1); }
inline TensorPtr layer_norm(TensorPtr x, TensorPtr gamma, TensorPtr beta, f32 eps = 1e-5f) {
    return QuasarML::Ops::layer_norm(device(), x, gamma, beta, eps);
}

inline TensorPtr reshape(TensorPtr x, const std::vector<u32>& new_shape) { return QuasarML::Ops::reshape(device(), x, new_shape); }
inline TensorPtr flatten(TensorPtr x) { return QuasarML::Ops::flatten(device(), x); }
inline TensorPtr squeeze(TensorPtr x) { return QuasarML::Ops::squeeze(device(), x); }
inline TensorPtr squeeze(TensorPtr x, i32 dim) { return QuasarML::Ops::squeeze(device(), x, dim); }
inline TensorPtr unsqueeze(TensorPtr x, i32 dim) { return QuasarML::Ops::unsqueeze(device(), x, dim); }
inline TensorPtr concat(const std::vector<TensorPtr>& ts, i32 axis = 0) { return QuasarML::Ops::concat(device(), ts, axis); }
inline TensorPtr stack(const std::vector<TensorPtr>& ts, i32 axis = 0) { return QuasarML::Ops::stack(device(), ts, axis); }
inline TensorPtr slice(TensorPtr x, i32 axis, u64 start, u64 end) { return QuasarML::Ops::slice(device(), x, axis, start, end); }
inline TensorPtr slice(TensorPtr x, i32 axis, u64 start, u64 end, u64 step) {
    return QuasarML::Ops::slice(device(), x, axis, start, end, step);
}
inline TensorPtr broadcast_to(TensorPtr x, const std::vector<u32>& shape) { return QuasarML::Ops::broadcast_to(device(), x, shape); }
inline TensorPtr copy(TensorPtr x) { return QuasarML::Ops::copy(device(), x); }
inline TensorPtr contiguous(TensorPtr x) { return QuasarML::Ops::contiguous(device(), x); }
inline TensorPtr cast(TensorPtr x, DataType dtype) { return QuasarML::Ops::cast(device(), x, dtype); }

// Ops that ran on the host instead of the GPU: always 0 in this backend.
// Multi-GPU: in-place all-reduce of one tensor per device (this process
// drives all of them).
using QuasarML::ReduceOp;
inline void all_reduce(const std::vector<TensorPtr>& per_device, ReduceOp op = ReduceOp::Sum) {
    QuasarML::Ops::all_reduce(per_device, op);
}
// Row-sharded tensors: one block of rows per device (scatter_rows splits host
// data over devices 0..n-1), reduced across all of them by sharded_reduce.
inline std::vector<TensorPtr> scatter_rows(const void* host, const std::vector<u32>& shape, u32 num_devices,
                                           DataType dtype = DataType::F32) {
    std::vector<Device*> devs;
    for (u32 i = 0; i < num_devices; ++i) devs.push_back(&device(i));
    return QuasarML::Ops::scatter_rows(host, shape, dtype, devs);
}
inline std::vector<TensorPtr> sharded_reduce(const std::vector<TensorPtr>& blocks, ReduceOp op, i32 axis,
                                             bool keepdims = false) {
    return QuasarML::Ops::sharded_reduce(blocks, op, axis, keepdims);
}
inline std::vector<TensorPtr> sharded_reduce(const std::vector<TensorPtr>& blocks, ReduceOp op) {
    return QuasarML::Ops::sharded_reduce(blocks, op);
}

// Elementwise fusion (deferred results evaluated as one kernel on access).
inline void set_fusion(bool on) { device().set_fusion(on); }
inline bool fusion_enabled() { return device().fusion(); }

// Overlap of independent calls on the device's stream (on by default).
inline void set_overlap(bool on) { device().set_overlap(on); }

inline u64 cpu_fallback_count() {
    uint64_t n = 0;
    device().check(qsml_cpu_fallback_count(device().ctx(), &n));
    return n;
}

}  // namespace qsml
