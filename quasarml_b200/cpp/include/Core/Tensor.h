// QuasarML's Tensor (QuasarML/src/Core/Tensor.h) on CUDA device memory.
//
// Same interface as the reference, with two changes the hot path needs:
//  * real strides: views (transpose, slice with a step, unsqueeze of a view)
//    are zero-copy and strides() reports them; is_contiguous() tells them
//    apart and contiguous() materialises one with a device gather;
//  * refcounted storage: a view keeps its parent's buffer alive (the
//    reference's views hold a raw handle with owns_buffer = false,
//    Core/Tensor.cpp:128-136, and dangle when the parent dies);
//  * deferred elementwise results: with fusion on (Device::set_fusion, or
//    inside begin_batch / end_batch) an elementwise op returns a tensor that
//    holds the expression over its materialised inputs instead of memory.
//    The first access to its data evaluates the whole expression in one
//    fused kernel (qsml_elementwise_fused); writes into a buffer first
//    evaluate the deferred tensors that read it, so results equal eager
//    execution.
#pragma once

#include <functional>
#include <memory>
#include <mutex>
#include <numeric>
#include <string>
#include <vector>

#include "../Common/Types.h"
#include "qsml_cuda.h"

namespace QuasarML {

class Device;
class Tensor;

// A device allocation from the context's caching allocator.
struct QS_API Storage {
    Storage(Device* device, u64 bytes);
    ~Storage();
    Storage(const Storage&) = delete;
    Storage& operator=(const Storage&) = delete;
    Device* device;
    void* ptr = nullptr;
    u64 bytes = 0;
    std::weak_ptr<int> alive;  // expires when the device (and its allocator) is gone
    // Deferred tensors whose expression reads this buffer; evaluated before
    // the buffer is written.
    std::mutex readers_mu;
    std::vector<std::weak_ptr<Tensor>> readers;
};

// A deferred elementwise expression: qsml_elementwise_fused's node list over
// materialised input tensors (the last node is the value).
struct LazyExpr {
    std::vector<qsml_fuse_node> nodes;
    std::vector<std::shared_ptr<Tensor>> inputs;
};

class QS_API Tensor : public std::enable_shared_from_this<Tensor> {
public:
    Tensor(Device* device, const std::vector<u32>& shape, DataType dtype = DataType::F32, bool host_visible = false);
    // View over existing storage (element strides and element offset).
    Tensor(std::shared_ptr<Storage> storage, const std::vector<u32>& shape, const std::vector<u64>& strides,
           u64 element_offset, DataType dtype);
    // Deferred result of an elementwise expression (see the file comment);
    // register_reads() must follow once the tensor is owned by a shared_ptr.
    Tensor(Device* device, const std::vector<u32>& shape, DataType dtype, std::shared_ptr<LazyExpr> expr);
    ~Tensor() = default;
    Tensor(const Tensor&) = delete;
    Tensor& operator=(const Tensor&) = delete;

    // Host transfers; offsets and sizes in bytes of the tensor's element
    // order (a non-contiguous tensor is gathered first on download).
    void upload(const void* data);
    void upload(const void* data, u64 size, u64 offset = 0);
    void download(void* data) const;
    void download(void* data, u64 size, u64 offset = 0) const;
    void fill(const void* value);
    void zero();
    void copy_from(const Tensor& src);

    const std::vector<u32>& shape() const { return _shape; }
    u32 rank() const { return static_cast<u32>(_shape.size()); }
    u32 dim(u32 i) const;
    u64 numel() const { return _numel; }
    DataType dtype() const { return _dtype; }
    u32 element_size() const { return dtype_size(_dtype); }
    u64 size_bytes() const { return _numel * element_size(); }
    bool is_host_visible() const { return false; }

    Tensor& reshape(const std::vector<u32>& new_shape);  // in place; contiguous tensors only
    std::shared_ptr<Tensor> view(const std::vector<u32>& new_shape) const;
    std::shared_ptr<Tensor> flatten() const;

    bool is_valid() const { return _storage != nullptr || _lazy != nullptr; }
    bool is_shape_compatible(const Tensor& other) const { return _shape == other._shape; }
    bool is_broadcastable(const std::vector<u32>& target) const;

    std::string shape_str() const;
    std::string info() const;
    std::vector<u64> strides() const { return _strides; }
    u64 element_offset() const { return _offset; }
    Device* device() const;

    // Additions of this backend.
    bool is_contiguous() const;
    std::shared_ptr<Tensor> contiguous() const;  // *this if contiguous, else a gathered copy
    std::shared_ptr<Tensor> strided_view(const std::vector<u32>& shape, const std::vector<u64>& strides,
                                         u64 element_offset) const;
    const std::shared_ptr<Storage>& storage() const;
    void* data() const;            // device address of element [0, ..., 0]
    qsml_tdesc desc() const;       // descriptor for the C ABI

    // Deferred results.
    bool is_lazy() const { return _lazy != nullptr; }
    const std::shared_ptr<LazyExpr>& lazy_expr() const { return _lazy; }
    void materialize() const;      // evaluates a deferred result (no-op otherwise)
    void register_reads();         // records this deferred tensor on its inputs' buffers

private:
    mutable std::shared_ptr<Storage> _storage;
    mutable std::shared_ptr<LazyExpr> _lazy;
    Device* _device = nullptr;
    std::vector<u32> _shape;
    std::vector<u64> _strides;
    u64 _offset = 0;
    DataType _dtype = DataType::F32;
    u64 _numel = 0;
    void compute_numel();
    // Evaluates deferred tensors that read this tensor's buffer (and this
    // tensor itself if deferred) before it is written.
    void prepare_write();
};

inline u64 compute_numel(const std::vector<u32>& shape) {
    return std::accumulate(shape.begin(), shape.end(), u64(1), std::multiplies<u64>());
}
inline bool shapes_equal(const std::vector<u32>& a, const std::vector<u32>& b) { return a == b; }
QS_API std::string shape_to_string(const std::vector<u32>& shape);
QS_API std::vector<u64> contiguous_strides(const std::vector<u32>& shape);

}  // namespace QuasarML
