// Core of the C++ QuasarML layer: Tensor, Device, DeviceManager, Logger.
// Device memory, transfers and copies go through libqsml_cuda.so's C ABI.
#include <cstdarg>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <sstream>

#include "Common/Assert.h"
#include "Common/Logger.h"
#include "Core/Device.h"
#include "Core/DeviceManager.h"
#include "Core/Tensor.h"
#include "Ops/Distributed.h"

namespace QuasarML {

// ---------------------------------------------------------------------------
// Types / Logger
// ---------------------------------------------------------------------------
const char* dtype_to_string(DataType dtype) {
    switch (dtype) {
        case DataType::F32: return "F32";
        case DataType::F16: return "F16";
        case DataType::I32: return "I32";
        case DataType::I16: return "I16";
        case DataType::I8: return "I8";
        case DataType::U32: return "U32";
        case DataType::U16: return "U16";
        case DataType::U8: return "U8";
    }
    return "Unknown";
}

static Logger::Level g_level = Logger::Warn;

void Logger::init() {
    const char* s = std::getenv("QSML_LOG");
    if (!s) return;
    std::string v(s);
    if (v == "trace") g_level = Trace;
    else if (v == "debug") g_level = Debug;
    else if (v == "info") g_level = Info;
    else if (v == "warn") g_level = Warn;
    else if (v == "error") g_level = Error;
    else if (v == "off") g_level = Off;
}

void Logger::shutdown() {}

Logger::Level Logger::level() { return g_level; }

void Logger::log(Level level, const char* fmt, ...) {
    if (level < g_level) return;
    static const char* names[] = {"trace", "debug", "info", "warn", "error", "off"};
    std::fprintf(stderr, "[qsml %s] ", names[level]);
    va_list ap;
    va_start(ap, fmt);
    std::vfprintf(stderr, fmt, ap);
    va_end(ap);
    std::fputc('\n', stderr);
}

// ---------------------------------------------------------------------------
// Storage / Tensor
// ---------------------------------------------------------------------------
Storage::Storage(Device* d, u64 n) : device(d), bytes(n) {
    QS_ASSERT(d && d->is_valid(), "Tensor needs a valid device");
    d->check(qsml_alloc(d->ctx(), n ? n : 1, &ptr));
    alive = d->alive_token();
}

Storage::~Storage() {
    // The device's context frees every block when it is destroyed; only
    // return the block while the device still lives.
    if (ptr && !alive.expired()) qsml_free(device->ctx(), ptr);
}

std::vector<u64> contiguous_strides(const std::vector<u32>& shape) {
    std::vector<u64> s(shape.size());
    u64 st = 1;
    for (int i = static_cast<int>(shape.size()) - 1; i >= 0; --i) {
        s[i] = st;
        st *= shape[i];
    }
    return s;
}

Tensor::Tensor(Device* device, const std::vector<u32>& shape, DataType dtype, bool)
    : _device(device), _shape(shape), _dtype(dtype) {
    // Core/Tensor.cpp:70-73 of the reference: a shape is non-empty with positive dims.
    QS_ASSERT(!shape.empty(), "Shape cannot be empty");
    for (u32 d : shape) QS_ASSERT(d > 0, "Dimension must be positive");
    compute_numel();
    _strides = contiguous_strides(shape);
    _storage = std::make_shared<Storage>(device, _numel * dtype_size(dtype));
}

Tensor::Tensor(std::shared_ptr<Storage> storage, const std::vector<u32>& shape, const std::vector<u64>& strides,
               u64 element_offset, DataType dtype)
    : _storage(std::move(storage)), _shape(shape), _strides(strides), _offset(element_offset), _dtype(dtype) {
    QS_ASSERT(_shape.size() == _strides.size(), "shape and strides differ in rank");
    _device = _storage ? _storage->device : nullptr;
    compute_numel();
}

Tensor::Tensor(Device* device, const std::vector<u32>& shape, DataType dtype, std::shared_ptr<LazyExpr> expr)
    : _lazy(std::move(expr)), _device(device), _shape(shape), _dtype(dtype) {
    QS_ASSERT(device && device->is_valid(), "Tensor needs a valid device");
    QS_ASSERT(!shape.empty(), "Shape cannot be empty");
    compute_numel();
    _strides = contiguous_strides(shape);
}

void Tensor::register_reads() {
    if (!_lazy) return;
    std::weak_ptr<Tensor> self = weak_from_this();
    for (const auto& in : _lazy->inputs) {
        const auto& st = in->storage();
        std::lock_guard<std::mutex> lk(st->readers_mu);
        if (st->readers.size() >= 64) {  // drop readers that are gone
            std::vector<std::weak_ptr<Tensor>> live;
            for (auto& w : st->readers)
                if (!w.expired()) live.push_back(w);
            st->readers.swap(live);
        }
        st->readers.push_back(self);
    }
}

void Tensor::materialize() const {
    if (!_lazy) return;
    std::shared_ptr<LazyExpr> e = _lazy;
    auto st = std::make_shared<Storage>(_device, _numel * element_size());
    std::vector<qsml_tdesc> ins(e->inputs.size());
    for (size_t j = 0; j < ins.size(); ++j) ins[j] = e->inputs[j]->desc();
    qsml_tdesc out;
    std::memset(&out, 0, sizeof(out));
    out.data = st->ptr;
    out.dtype = static_cast<int32_t>(_dtype);
    out.ndim = static_cast<int32_t>(_shape.size());
    for (size_t i = 0; i < _shape.size(); ++i) {
        out.shape[i] = _shape[i];
        out.stride[i] = static_cast<int64_t>(_strides[i]);
    }
    _device->check(qsml_elementwise_fused(_device->ctx(), e->nodes.data(), static_cast<int32_t>(e->nodes.size()),
                                          ins.data(), static_cast<int32_t>(ins.size()), &out));
    _storage = st;
    _lazy.reset();
}

void Tensor::prepare_write() {
    materialize();
    std::vector<std::shared_ptr<Tensor>> pending;
    {
        std::lock_guard<std::mutex> lk(_storage->readers_mu);
        for (auto& w : _storage->readers)
            if (auto t = w.lock()) pending.push_back(t);
        _storage->readers.clear();
    }
    for (auto& t : pending) t->materialize();
}

const std::shared_ptr<Storage>& Tensor::storage() const {
    materialize();
    return _storage;
}

void Tensor::compute_numel() {
    _numel = 1;
    for (u32 d : _shape) _numel *= d;
}

u32 Tensor::dim(u32 i) const {
    QS_ASSERT(i < _shape.size(), "Dimension index out of range");
    return _shape[i];
}

Device* Tensor::device() const { return _device; }

void* Tensor::data() const {
    materialize();
    return static_cast<char*>(_storage->ptr) + _offset * element_size();
}

qsml_tdesc Tensor::desc() const {
    qsml_tdesc d;
    std::memset(&d, 0, sizeof(d));
    QS_ASSERT(_shape.size() <= QSML_MAX_DIMS, "Tensor rank above 8 is not supported");
    d.data = data();
    d.dtype = static_cast<int32_t>(_dtype);
    d.ndim = static_cast<int32_t>(_shape.size());
    for (size_t i = 0; i < _shape.size(); ++i) {
        d.shape[i] = _shape[i];
        d.stride[i] = static_cast<int64_t>(_strides[i]);
    }
    return d;
}

bool Tensor::is_contiguous() const {
    if (_lazy) return true;  // evaluates into a contiguous buffer
    u64 s = 1;
    for (int i = static_cast<int>(_shape.size()) - 1; i >= 0; --i) {
        if (_shape[i] != 1 && _strides[i] != s) return false;
        s *= _shape[i];
    }
    return true;
}

std::shared_ptr<Tensor> Tensor::contiguous() const {
    materialize();
    if (is_contiguous()) return std::const_pointer_cast<Tensor>(shared_from_this());
    auto out = device()->create_tensor(_shape, _dtype);
    qsml_tdesc s = desc(), o = out->desc();
    device()->check(qsml_gather(device()->ctx(), &s, &o));
    return out;
}

std::shared_ptr<Tensor> Tensor::strided_view(const std::vector<u32>& shape, const std::vector<u64>& strides,
                                             u64 element_offset) const {
    materialize();
    return std::make_shared<Tensor>(_storage, shape, strides, element_offset, _dtype);
}

void Tensor::upload(const void* data) { upload(data, size_bytes(), 0); }

void Tensor::upload(const void* src, u64 size, u64 offset) {
    QS_ASSERT(is_valid(), "Tensor not valid");
    prepare_write();
    QS_ASSERT(is_contiguous(), "upload into a non-contiguous view");
    QS_ASSERT(offset + size <= size_bytes(), "upload beyond the tensor");
    device()->check(qsml_h2d(device()->ctx(), static_cast<char*>(this->data()) + offset, src, size));
}

void Tensor::download(void* dst) const { download(dst, size_bytes(), 0); }

void Tensor::download(void* dst, u64 size, u64 offset) const {
    QS_ASSERT(is_valid(), "Tensor not valid");
    QS_ASSERT(offset + size <= size_bytes(), "download beyond the tensor");
    auto c = contiguous();
    device()->check(qsml_d2h(device()->ctx(), dst, static_cast<const char*>(c->data()) + offset, size));
}

void Tensor::fill(const void* value) {
    QS_ASSERT(is_valid(), "Tensor not valid");
    prepare_write();
    if (is_contiguous()) {
        device()->check(qsml_fill(device()->ctx(), data(), value, static_cast<int32_t>(element_size()),
                                  static_cast<int64_t>(_numel)));
        return;
    }
    auto tmp = device()->create_tensor(_shape, _dtype);
    tmp->fill(value);
    copy_from(*tmp);
}

void Tensor::zero() {
    std::vector<unsigned char> z(element_size(), 0);
    fill(z.data());
}

void Tensor::copy_from(const Tensor& src) {
    QS_ASSERT(size_bytes() == src.size_bytes(), "Size mismatch");
    src.materialize();
    prepare_write();
    QS_ASSERT(src.dtype() == _dtype || (is_contiguous() && src.is_contiguous()), "Type mismatch");
    if (src.shape() == _shape) {
        qsml_tdesc s = src.desc(), o = desc();
        device()->check(qsml_gather(device()->ctx(), &s, &o));
        return;
    }
    // Different shapes, same byte count: a raw copy (Core/Tensor.cpp:114-119).
    auto c = src.contiguous();
    QS_ASSERT(is_contiguous(), "copy_from into a non-contiguous view with another shape");
    device()->check(qsml_d2d(device()->ctx(), data(), c->data(), size_bytes()));
}

Tensor& Tensor::reshape(const std::vector<u32>& new_shape) {
    QS_ASSERT(QuasarML::compute_numel(new_shape) == _numel, "Element count mismatch in reshape");
    prepare_write();  // deferred readers of this tensor see its old shape
    QS_ASSERT(is_contiguous(), "reshape of a non-contiguous view (use contiguous() first)");
    _shape = new_shape;
    _strides = contiguous_strides(new_shape);
    return *this;
}

std::shared_ptr<Tensor> Tensor::view(const std::vector<u32>& new_shape) const {
    QS_ASSERT(QuasarML::compute_numel(new_shape) == _numel, "Element count mismatch in view");
    materialize();
    QS_ASSERT(is_contiguous(), "view of a non-contiguous tensor (use contiguous() first)");
    return strided_view(new_shape, contiguous_strides(new_shape), _offset);
}

std::shared_ptr<Tensor> Tensor::flatten() const { return view({static_cast<u32>(_numel)}); }

// Core/Tensor.cpp:142-151: right-aligned, each pair equal or one of them 1.
bool Tensor::is_broadcastable(const std::vector<u32>& target) const {
    if (target.size() < _shape.size()) return false;
    size_t diff = target.size() - _shape.size();
    for (size_t i = 0; i < _shape.size(); ++i) {
        u32 a = _shape[i], b = target[diff + i];
        if (a != b && a != 1 && b != 1) return false;
    }
    return true;
}

std::string Tensor::shape_str() const { return shape_to_string(_shape); }

std::string Tensor::info() const {
    std::ostringstream ss;
    ss << "Tensor(" << shape_str() << ", " << dtype_to_string(_dtype) << ")";
    return ss.str();
}

std::string shape_to_string(const std::vector<u32>& shape) {
    std::ostringstream ss;
    ss << "[";
    for (size_t i = 0; i < shape.size(); ++i) {
        if (i > 0) ss << ", ";
        ss << shape[i];
    }
    ss << "]";
    return ss.str();
}

// ---------------------------------------------------------------------------
// Device
// ---------------------------------------------------------------------------
Device::Device(const std::string& name, u32 device_index)
    : _alive(std::make_shared<int>(0)), _name(name), _device_index(device_index) {
    qsml_ctx* c = nullptr;
    if (qsml_init(static_cast<int32_t>(device_index), &c) == QSML_OK) {
        _ctx = c;
        // The device's stream is the library's own (qsml_init creates it) and
        // carries only library work, so independent calls may overlap on it;
        // QSML_OVERLAP=0 turns that off.
        const char* env = std::getenv("QSML_OVERLAP");
        qsml_set_overlap(_ctx, env && env[0] == '0' ? 0 : 1);
    } else {
        LOG_WARN("device %u unavailable: %s", device_index, qsml_last_error(nullptr));
    }
}

Device::~Device() {
    _alive.reset();
    if (_ctx) qsml_destroy(_ctx);
}

void Device::check(int st) const {
    if (st != QSML_OK)
        throw std::runtime_error(std::string("QuasarML (status ") + std::to_string(st) + "): " +
                                 qsml_last_error(_ctx));
}

std::shared_ptr<Tensor> Device::create_tensor(const std::vector<u32>& shape, DataType dtype, bool host_visible) {
    return std::make_shared<Tensor>(this, shape, dtype, host_visible);
}

void Device::set_fusion(bool on) { _fusion = on; }

void Device::set_overlap(bool on) { check(qsml_set_overlap(_ctx, on ? 1 : 0)); }

void Device::begin_batch() {
    QS_ASSERT(!_in_batch, "Already in batch");
    _in_batch = true;
}

void Device::end_batch() {
    QS_ASSERT(_in_batch, "Not in batch");
    _in_batch = false;
}

void Device::flush_pending() { synchronize(); }

void Device::synchronize() {
    if (_ctx) check(qsml_synchronize(_ctx));
}

void Device::wait_idle() { synchronize(); }

// ---------------------------------------------------------------------------
// DeviceManager
// ---------------------------------------------------------------------------
DeviceManager& DeviceManager::instance() {
    static DeviceManager mgr;
    return mgr;
}

DeviceManager::DeviceManager() {
    int32_t n = 0;
    if (qsml_device_count(&n) == QSML_OK && n > 0) _device_count = static_cast<u32>(n);
}

DeviceManager::~DeviceManager() { shutdown(); }

Device* DeviceManager::get(u32 device_id) {
    std::lock_guard<std::mutex> lock(_mutex);
    if (_shutdown || device_id >= _device_count) return nullptr;
    auto it = _devices.find(device_id);
    if (it != _devices.end()) return it->second.get();
    auto device = std::make_unique<Device>("QuasarML", device_id);
    if (!device->is_valid()) return nullptr;
    Device* ptr = device.get();
    _devices[device_id] = std::move(device);
    return ptr;
}

std::vector<std::string> DeviceManager::device_names() const {
    std::vector<std::string> names;
    char buf[256];
    for (u32 i = 0; i < _device_count; ++i) {
        if (qsml_device_name(static_cast<int32_t>(i), buf, sizeof(buf)) == QSML_OK) names.emplace_back(buf);
    }
    return names;
}

void DeviceManager::set_default(u32 device_id) {
    if (device_id < _device_count) _default_device = device_id;
}

void DeviceManager::shutdown() {
    Ops::release_device_groups();  // groups hold the devices' contexts
    std::lock_guard<std::mutex> lock(_mutex);
    if (_shutdown) return;
    _shutdown = true;
    _devices.clear();
}

}  // namespace QuasarML
