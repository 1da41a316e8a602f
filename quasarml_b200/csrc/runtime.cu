// Context, caching allocator, copies and error model of libqsml_cuda.
//
// The reference's equivalents are the Vulkan device/queue setup
// (Backend/Vulkan/VulkanDevice.cpp:42-113), VMA buffers
// (Backend/Vulkan/VulkanBackend.cpp:254-325), staged blocking copies
// (VulkanBackend.cpp:327-373) and fence waits (VulkanBackend.cpp:613-658).
// Here: one CUDA stream per context, a size-binned caching allocator and
// cudaMemcpyAsync on that stream.
#include "qsml_internal.cuh"

#include <cstdlib>
#include <vector>

namespace qsml {

static thread_local std::string g_global_error = "no error";

qsml_status_t set_error(Context* ctx, qsml_status_t st, const std::string& msg) {
    if (ctx) {
        std::lock_guard<std::mutex> lk(ctx->err_mu);
        ctx->last_error = msg;
    } else {
        g_global_error = msg;
    }
    return st;
}

qsml_status_t check_cuda(Context* ctx, cudaError_t e, const char* what) {
    if (e == cudaSuccess) return QSML_OK;
    cudaGetLastError();  // clear a non-sticky error
    if (ctx) {
        // a launch planned but refused: forget the plan and the window
        ctx->planned_for = 0;
        end_window(ctx->stream);
    }
    std::string m = std::string(what) + ": " + cudaGetErrorString(e);
    return set_error(ctx, e == cudaErrorMemoryAllocation ? QSML_E_OOM : QSML_E_CUDA, m);
}

qsml_status_t after_launch(Context* ctx, const char* kernel) {
    // a launch that plan_launch did not see closes the stream's window
    const bool planned = ctx->planned_for != 0 && ctx->planned_for == ctx->launches + 1;
    ctx->planned_for = 0;
    ctx->launches++;
    ctx->last_kernel = kernel;
    cudaError_t e = cudaGetLastError();
    if (!planned || e != cudaSuccess) end_window(ctx->stream);
    if (e != cudaSuccess) {
        return set_error(ctx, QSML_E_CUDA,
                         std::string("launch of ") + kernel + " failed: " + cudaGetErrorString(e));
    }
    return QSML_OK;
}

// ---------------------------------------------------------------------------
// Windows of kernels that may run together on a stream (see plan_launch in
// qsml_internal.cuh).
// ---------------------------------------------------------------------------
namespace {

constexpr size_t kMaxWindow = 16;  // deferring kernels in flight behind one that waited

struct Window {
    bool open = false;
    std::vector<Footprint> kernels;
};

std::mutex g_window_mu;
std::unordered_map<cudaStream_t, Window> g_windows;

bool overlap(const Span& a, const Span& b) { return a.lo < b.hi && b.lo < a.hi; }

// True if kernel n may not run beside kernel r.
bool conflict(const Footprint& n, const Footprint& r) {
    for (int i = 0; i < n.nw; ++i) {
        for (int j = 0; j < r.nr; ++j)
            if (overlap(n.writes[i], r.reads[j])) return true;
        for (int j = 0; j < r.nw; ++j)
            if (overlap(n.writes[i], r.writes[j])) return true;
    }
    for (int i = 0; i < n.nr; ++i)
        for (int j = 0; j < r.nw; ++j)
            if (overlap(n.reads[i], r.writes[j])) return true;
    return false;
}

}  // namespace

int plan_launch(Context* ctx, const Footprint& f) {
    std::lock_guard<std::mutex> lk(g_window_mu);
    Window& w = g_windows[ctx->stream];
    bool defer = ctx->overlap && w.open && w.kernels.size() < kMaxWindow;
    for (size_t i = 0; defer && i < w.kernels.size(); ++i) defer = !conflict(f, w.kernels[i]);
    if (!defer) w.kernels.clear();  // this kernel waits: nothing before it is still running
    w.kernels.push_back(f);
    w.open = true;
    ctx->planned_for = ctx->launches + 1;
    ctx->planned++;
    if (defer) ctx->deferred++;
    return defer ? 1 : 0;
}

void end_window(cudaStream_t stream) {
    std::lock_guard<std::mutex> lk(g_window_mu);
    auto it = g_windows.find(stream);
    if (it != g_windows.end()) {
        it->second.open = false;
        it->second.kernels.clear();
    }
}

Span view_span(const qsml_tdesc* d) {
    const int64_t es = static_cast<int64_t>(dtype_size(d->dtype));
    int64_t lo = 0, hi = 0;
    for (int i = 0; i < d->ndim; ++i) {
        if (d->shape[i] == 0) return Span{};
        const int64_t e = (d->shape[i] - 1) * d->stride[i];
        if (e < 0) lo += e; else hi += e;
    }
    const uintptr_t base = reinterpret_cast<uintptr_t>(d->data);
    return Span{base + static_cast<uintptr_t>(lo * es), base + static_cast<uintptr_t>((hi + 1) * es)};
}

qsml_status_t check_desc(Context* ctx, const qsml_tdesc* d, const char* name) {
    if (!d) return set_error(ctx, QSML_E_INVALID, std::string(name) + ": null descriptor");
    if (d->ndim < 0 || d->ndim > kMaxDims)
        return set_error(ctx, QSML_E_SHAPE, std::string(name) + ": ndim out of range");
    if (dtype_size(d->dtype) == 0)
        return set_error(ctx, QSML_E_DTYPE, std::string(name) + ": unknown dtype");
    for (int i = 0; i < d->ndim; ++i)
        if (d->shape[i] < 0) return set_error(ctx, QSML_E_SHAPE, std::string(name) + ": negative extent");
    if (numel(d) > 0 && d->data == nullptr)
        return set_error(ctx, QSML_E_INVALID, std::string(name) + ": null data pointer");
    return QSML_OK;
}

qsml_status_t plan_reduction(Context* ctx, const qsml_tdesc* a, int32_t axis, int32_t keepdims,
                             const qsml_tdesc* out, const char* what, int64_t* outer, int64_t* k,
                             int64_t* inner) {
    *outer = 1;
    *k = 1;
    *inner = 1;
    if (axis == QSML_AXIS_ALL) {
        *k = numel(a);
        if (numel(out) != 1)
            return set_error(ctx, QSML_E_SHAPE, std::string(what) + ": full reduction needs a 1-element out");
        return QSML_OK;
    }
    const int ax = axis < 0 ? axis + a->ndim : axis;
    if (ax < 0 || ax >= a->ndim) return set_error(ctx, QSML_E_SHAPE, std::string(what) + ": invalid axis");
    int64_t expect[kMaxDims];
    int en = 0;
    for (int i = 0; i < a->ndim; ++i) {
        if (i < ax) *outer *= a->shape[i];
        if (i > ax) *inner *= a->shape[i];
        if (i == ax) {
            *k = a->shape[i];
            if (keepdims) expect[en++] = 1;
        } else {
            expect[en++] = a->shape[i];
        }
    }
    bool ok = true;
    if (en == 0) {
        ok = numel(out) == 1 && out->ndim <= 1;
    } else {
        ok = out->ndim == en;
        for (int i = 0; ok && i < en; ++i) ok = out->shape[i] == expect[i];
    }
    if (!ok) return set_error(ctx, QSML_E_SHAPE, std::string(what) + ": out shape does not match the reduced shape");
    return QSML_OK;
}

bool dense_view_plan(const qsml_tdesc* a, int32_t axis, int64_t* outer, int64_t* k, int64_t* inner) {
    const int64_t n = numel(a);
    if (n == 0) return false;
    int ax = -1;
    if (axis != QSML_AXIS_ALL) {
        ax = axis < 0 ? axis + a->ndim : axis;
        if (ax < 0 || ax >= a->ndim || a->shape[ax] == 1) return false;
    }
    // the non-unit dims, by stride ascending, must tile one block exactly
    int dims[kMaxDims];
    int nd = 0;
    for (int i = 0; i < a->ndim; ++i) {
        if (a->shape[i] == 1) continue;
        if (a->stride[i] <= 0) return false;
        int j = nd++;
        while (j > 0 && a->stride[dims[j - 1]] > a->stride[i]) {
            dims[j] = dims[j - 1];
            --j;
        }
        dims[j] = i;
    }
    int64_t expect = 1;
    for (int j = 0; j < nd; ++j) {
        if (a->stride[dims[j]] != expect) return false;
        expect *= a->shape[dims[j]];
    }
    if (ax < 0) {
        *outer = 1;
        *k = n;
        *inner = 1;
        return true;
    }
    // kept dims in memory order along the view
    int64_t prev = INT64_MAX;
    for (int i = 0; i < a->ndim; ++i) {
        if (i == ax || a->shape[i] == 1) continue;
        if (a->stride[i] >= prev) return false;
        prev = a->stride[i];
    }
    *k = a->shape[ax];
    *inner = a->stride[ax];
    *outer = n / (*k * *inner);
    return true;
}

// ---------------------------------------------------------------------------
// Caching allocator
// ---------------------------------------------------------------------------

// Small requests round to 512 B, large ones to 2 MiB; a cached block is
// reused for a request of at most its size and at least half of it.
size_t CachingAllocator::round_size(size_t bytes) {
    if (bytes == 0) bytes = 1;
    const size_t small = 512, large = size_t(2) << 20;
    if (bytes <= (size_t(1) << 20)) return (bytes + small - 1) / small * small;
    return (bytes + large - 1) / large * large;
}

// Host-side fault injection for tests: QSML_FAULT_ALLOC_N=n makes the n-th
// driver allocation of the process report out-of-memory.
static int64_t fault_alloc_n() {
    static int64_t n = [] {
        const char* s = std::getenv("QSML_FAULT_ALLOC_N");
        return s ? std::atoll(s) : int64_t(0);
    }();
    return n;
}

qsml_status_t CachingAllocator::alloc(size_t bytes, void** ptr, std::string* err) {
    size_t r = round_size(bytes);
    std::lock_guard<std::mutex> lk(mu_);
    auto it = free_.lower_bound(r);
    if (it != free_.end() && it->first <= 2 * r) {
        void* p = it->second;
        size_t sz = it->first;
        free_.erase(it);
        live_[p] = sz;
        live_bytes_ += sz;
        hits_++;
        *ptr = p;
        return QSML_OK;
    }
    malloc_calls_++;
    int64_t fault = fault_alloc_n();
    void* p = nullptr;
    cudaError_t e;
    if (fault > 0 && int64_t(malloc_calls_) == fault) {
        e = cudaErrorMemoryAllocation;
    } else {
        e = cudaMalloc(&p, r);
        if (e == cudaErrorMemoryAllocation) {
            // Give the cache back to the driver and retry once.
            cudaGetLastError();
            for (auto& kv : free_) {
                cudaFree(kv.second);
                reserved_ -= kv.first;
            }
            free_.clear();
            e = cudaMalloc(&p, r);
        }
    }
    if (e != cudaSuccess) {
        cudaGetLastError();
        *err = "device allocation of " + std::to_string(r) + " bytes failed: " + cudaGetErrorString(e);
        return QSML_E_OOM;
    }
    misses_++;
    reserved_ += r;
    live_[p] = r;
    live_bytes_ += r;
    *ptr = p;
    return QSML_OK;
}

qsml_status_t CachingAllocator::free(void* ptr, std::string* err) {
    if (!ptr) return QSML_OK;
    std::lock_guard<std::mutex> lk(mu_);
    auto it = live_.find(ptr);
    if (it == live_.end()) {
        *err = "free of a pointer this allocator does not own";
        return QSML_E_INVALID;
    }
    size_t sz = it->second;
    live_.erase(it);
    live_bytes_ -= sz;
    free_.emplace(sz, ptr);
    return QSML_OK;
}

void CachingAllocator::release_cached() {
    std::lock_guard<std::mutex> lk(mu_);
    for (auto& kv : free_) {
        cudaFree(kv.second);
        reserved_ -= kv.first;
    }
    free_.clear();
}

void CachingAllocator::stats(uint64_t* misses, uint64_t* hits, uint64_t* reserved, uint64_t* live) {
    std::lock_guard<std::mutex> lk(mu_);
    if (misses) *misses = misses_;
    if (hits) *hits = hits_;
    if (reserved) *reserved = reserved_;
    if (live) *live = live_bytes_;
}

CachingAllocator::~CachingAllocator() {
    for (auto& kv : free_) cudaFree(kv.second);
    for (auto& kv : live_) cudaFree(kv.first);
}

qsml_status_t get_scratch(Context* ctx, size_t bytes, void** ptr) {
    bytes += 256;
    bytes = (bytes + 255) & ~size_t(255);
    // kScratchSlots slots of scratch_bytes / kScratchSlots each, in turn
    if (ctx->scratch_bytes / kScratchSlots < bytes) {
        if (ctx->scratch) {
            // The old scratch may still be read by enqueued kernels.
            QSML_TRY_STATUS(check_cuda(ctx, cudaStreamSynchronize(ctx->stream), "scratch resize sync"));
            cudaFree(ctx->scratch);
            ctx->scratch = nullptr;
            ctx->scratch_bytes = 0;
        }
        size_t slot = CachingAllocator::round_size(bytes < (size_t(1) << 20) ? (size_t(1) << 20) : bytes);
        const size_t sz = slot * kScratchSlots;
        QSML_TRY_STATUS(check_cuda(ctx, cudaMalloc(&ctx->scratch, sz), "scratch allocation"));
        QSML_TRY_STATUS(check_cuda(ctx, cudaMemsetAsync(ctx->scratch, 0, sz, ctx->stream), "scratch clear"));
        ctx->scratch_bytes = sz;
        ctx->scratch_slot = 0;
        end_window(ctx->stream);  // the memset: kernels after it wait for it
    }
    const size_t slot = ctx->scratch_bytes / kScratchSlots;
    *ptr = static_cast<char*>(ctx->scratch) + static_cast<size_t>(ctx->scratch_slot) * slot;
    ctx->scratch_slot = (ctx->scratch_slot + 1) % kScratchSlots;
    return QSML_OK;
}

__global__ void k_set_wait_limit(int* status, long long cycles) {
    *reinterpret_cast<long long*>(status + 2) = cycles;
}

}  // namespace qsml

using qsml::Context;

// ---------------------------------------------------------------------------
// extern "C" entry points
// ---------------------------------------------------------------------------

extern "C" {

qsml_status_t qsml_device_count(int32_t* count) {
    if (!count) return QSML_E_INVALID;
    int n = 0;
    cudaError_t e = cudaGetDeviceCount(&n);
    if (e != cudaSuccess) {
        cudaGetLastError();
        *count = 0;
        if (e == cudaErrorNoDevice || e == cudaErrorInsufficientDriver) return QSML_OK;
        return qsml::set_error(nullptr, QSML_E_CUDA, std::string("cudaGetDeviceCount: ") + cudaGetErrorString(e));
    }
    *count = n;
    return QSML_OK;
}

qsml_status_t qsml_device_name(int32_t device, char* buf, size_t len) {
    if (!buf || len == 0) return QSML_E_INVALID;
    cudaDeviceProp p;
    cudaError_t e = cudaGetDeviceProperties(&p, device);
    if (e != cudaSuccess) {
        cudaGetLastError();
        return qsml::set_error(nullptr, QSML_E_CUDA, std::string("cudaGetDeviceProperties: ") + cudaGetErrorString(e));
    }
    std::snprintf(buf, len, "%s", p.name);
    return QSML_OK;
}

qsml_status_t qsml_init(int32_t device, qsml_ctx** out) {
    if (!out) return QSML_E_INVALID;
    *out = nullptr;
    int n = 0;
    cudaError_t e = cudaGetDeviceCount(&n);
    if (e != cudaSuccess || device < 0 || device >= n) {
        cudaGetLastError();
        return qsml::set_error(nullptr, QSML_E_INVALID, "qsml_init: no CUDA device " + std::to_string(device));
    }
    if ((e = cudaSetDevice(device)) != cudaSuccess) {
        cudaGetLastError();
        return qsml::set_error(nullptr, QSML_E_CUDA, std::string("cudaSetDevice: ") + cudaGetErrorString(e));
    }
    int major = 0, minor = 0;
    cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, device);
    cudaDeviceGetAttribute(&minor, cudaDevAttrComputeCapabilityMinor, device);
    if (major != 10 || minor != 0) {
        return qsml::set_error(nullptr, QSML_E_UNSUPPORTED,
                               "qsml_init: this library is built for sm_100a (B200); device " +
                                   std::to_string(device) + " is sm_" + std::to_string(major) +
                                   std::to_string(minor));
    }
    Context* ctx = new Context();
    ctx->device = device;
    cudaDeviceGetAttribute(&ctx->num_sms, cudaDevAttrMultiProcessorCount, device);
    if ((e = cudaStreamCreateWithFlags(&ctx->own_stream, cudaStreamNonBlocking)) != cudaSuccess) {
        cudaGetLastError();
        delete ctx;
        return qsml::set_error(nullptr, QSML_E_CUDA, std::string("cudaStreamCreate: ") + cudaGetErrorString(e));
    }
    ctx->stream = ctx->own_stream;
    if ((e = cudaMalloc(&ctx->status, 256)) != cudaSuccess ||
        (e = cudaMemsetAsync(ctx->status, 0, 256, ctx->own_stream)) != cudaSuccess ||
        (e = cudaStreamSynchronize(ctx->own_stream)) != cudaSuccess) {
        cudaGetLastError();
        if (ctx->status) cudaFree(ctx->status);
        cudaStreamDestroy(ctx->own_stream);
        delete ctx;
        return qsml::set_error(nullptr, QSML_E_CUDA, std::string("qsml_init: status word: ") + cudaGetErrorString(e));
    }
    ctx->allocator = new qsml::CachingAllocator(device);
    *out = reinterpret_cast<qsml_ctx*>(ctx);
    return QSML_OK;
}

qsml_status_t qsml_destroy(qsml_ctx* handle) {
    QSML_CTX(handle);
    cudaStreamSynchronize(C_->stream);
    if (C_->stream != C_->own_stream) cudaStreamSynchronize(C_->own_stream);
    qsml::end_window(C_->stream);
    qsml::end_window(C_->own_stream);
    qsml::staging_free(C_);
    delete C_->allocator;
    if (C_->scratch) cudaFree(C_->scratch);
    if (C_->status) cudaFree(C_->status);
    cudaStreamDestroy(C_->own_stream);
    delete C_;
    return QSML_OK;
}

qsml_status_t qsml_set_overlap(qsml_ctx* handle, int32_t enable) {
    QSML_CTX(handle);
    C_->overlap = enable != 0;
    return QSML_OK;
}

qsml_status_t qsml_overlap_stats(qsml_ctx* handle, uint64_t* planned, uint64_t* deferred) {
    QSML_CTX(handle);
    if (planned) *planned = C_->planned;
    if (deferred) *deferred = C_->deferred;
    return QSML_OK;
}

qsml_status_t qsml_set_stream(qsml_ctx* handle, void* stream) {
    QSML_CTX(handle);
    // NULL is the CUDA legacy default stream (what a framework reports as
    // stream 0); the context's own stream is available from qsml_get_stream
    // on a fresh context.
    cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
    if (s == C_->stream) return QSML_OK;
    QSML_TRY_STATUS(qsml::check_cuda(C_, cudaStreamSynchronize(C_->stream), "qsml_set_stream"));
    C_->stream = s;
    return QSML_OK;
}

qsml_status_t qsml_get_stream(qsml_ctx* handle, void** stream) {
    QSML_CTX(handle);
    if (!stream) return QSML_E_INVALID;
    *stream = reinterpret_cast<void*>(C_->stream);
    return QSML_OK;
}

qsml_status_t qsml_synchronize(qsml_ctx* handle) {
    QSML_CTX(handle);
    QSML_TRY_STATUS(qsml::check_cuda(C_, cudaStreamSynchronize(C_->stream), "qsml_synchronize"));
    // A kernel whose bounded device-side wait expired left a code here.
    int code = 0;
    QSML_TRY_STATUS(qsml::check_cuda(C_, cudaMemcpy(&code, C_->status, sizeof(int), cudaMemcpyDeviceToHost),
                                     "qsml_synchronize status"));
    if (code != 0) {
        cudaMemset(C_->status, 0, sizeof(int));
        return qsml::set_error(C_, code, "a kernel's bounded device-side wait expired (status " +
                                             std::to_string(code) + ")");
    }
    return QSML_OK;
}

qsml_status_t qsml_set_wait_limit(qsml_ctx* handle, int64_t cycles) {
    QSML_CTX(handle);
    if (cycles < 0) return qsml::set_error(C_, QSML_E_INVALID, "qsml_set_wait_limit: negative limit");
    // stream-ordered: kernels enqueued after this call see the new limit
    qsml::k_set_wait_limit<<<1, 1, 0, C_->stream>>>(C_->status, static_cast<long long>(cycles));
    return qsml::after_launch(C_, "k_set_wait_limit");
}

const char* qsml_last_error(qsml_ctx* handle) {
    Context* ctx = reinterpret_cast<Context*>(handle);
    if (!ctx) return qsml::g_global_error.c_str();
    std::lock_guard<std::mutex> lk(ctx->err_mu);
    return ctx->last_error.empty() ? "no error" : ctx->last_error.c_str();
}

qsml_status_t qsml_alloc(qsml_ctx* handle, size_t bytes, void** ptr) {
    QSML_CTX(handle);
    if (!ptr) return qsml::set_error(C_, QSML_E_INVALID, "qsml_alloc: null out pointer");
    std::string err;
    qsml_status_t st = C_->allocator->alloc(bytes, ptr, &err);
    if (st != QSML_OK) return qsml::set_error(C_, st, err);
    return QSML_OK;
}

qsml_status_t qsml_free(qsml_ctx* handle, void* ptr) {
    QSML_CTX(handle);
    std::string err;
    qsml_status_t st = C_->allocator->free(ptr, &err);
    if (st != QSML_OK) return qsml::set_error(C_, st, err);
    return QSML_OK;
}

qsml_status_t qsml_empty_cache(qsml_ctx* handle) {
    QSML_CTX(handle);
    QSML_TRY_STATUS(qsml::check_cuda(C_, cudaStreamSynchronize(C_->stream), "qsml_empty_cache"));
    C_->allocator->release_cached();
    return QSML_OK;
}

qsml_status_t qsml_h2d(qsml_ctx* handle, void* dst, const void* src, size_t bytes) {
    QSML_CTX(handle);
    if (bytes == 0) return QSML_OK;
    if (!dst || !src) return qsml::set_error(C_, QSML_E_INVALID, "qsml_h2d: null pointer");
    return qsml::copy_h2d(C_, dst, src, bytes);
}

qsml_status_t qsml_d2h_async(qsml_ctx* handle, void* dst, const void* src, size_t bytes) {
    QSML_CTX(handle);
    if (bytes == 0) return QSML_OK;
    if (!dst || !src) return qsml::set_error(C_, QSML_E_INVALID, "qsml_d2h: null pointer");
    return qsml::check_cuda(C_, cudaMemcpyAsync(dst, src, bytes, cudaMemcpyDeviceToHost, C_->stream), "qsml_d2h");
}

qsml_status_t qsml_d2h(qsml_ctx* handle, void* dst, const void* src, size_t bytes) {
    QSML_CTX(handle);
    if (bytes == 0) return QSML_OK;
    if (!dst || !src) return qsml::set_error(C_, QSML_E_INVALID, "qsml_d2h: null pointer");
    return qsml::copy_d2h(C_, dst, src, bytes);
}

qsml_status_t qsml_d2d(qsml_ctx* handle, void* dst, const void* src, size_t bytes) {
    QSML_CTX(handle);
    if (bytes == 0) return QSML_OK;
    if (!dst || !src) return qsml::set_error(C_, QSML_E_INVALID, "qsml_d2d: null pointer");
    return qsml::check_cuda(C_, cudaMemcpyAsync(dst, src, bytes, cudaMemcpyDeviceToDevice, C_->stream), "qsml_d2d");
}

qsml_status_t qsml_host_alloc(size_t bytes, void** ptr) {
    if (!ptr) return QSML_E_INVALID;
    cudaError_t e = cudaHostAlloc(ptr, bytes ? bytes : 1, cudaHostAllocDefault);
    if (e != cudaSuccess) {
        cudaGetLastError();
        *ptr = nullptr;
        return qsml::set_error(nullptr, QSML_E_OOM, std::string("cudaHostAlloc: ") + cudaGetErrorString(e));
    }
    return QSML_OK;
}

qsml_status_t qsml_host_free(void* ptr) {
    if (!ptr) return QSML_OK;
    cudaError_t e = cudaFreeHost(ptr);
    if (e != cudaSuccess) {
        cudaGetLastError();
        return qsml::set_error(nullptr, QSML_E_CUDA, std::string("cudaFreeHost: ") + cudaGetErrorString(e));
    }
    return QSML_OK;
}

qsml_status_t qsml_launch_count(qsml_ctx* handle, uint64_t* count) {
    QSML_CTX(handle);
    if (!count) return QSML_E_INVALID;
    *count = C_->launches;
    return QSML_OK;
}

qsml_status_t qsml_last_kernel(qsml_ctx* handle, char* buf, size_t len) {
    QSML_CTX(handle);
    if (!buf || len == 0) return QSML_E_INVALID;
    std::snprintf(buf, len, "%s", C_->last_kernel);
    return QSML_OK;
}

qsml_status_t qsml_cpu_fallback_count(qsml_ctx* handle, uint64_t* count) {
    QSML_CTX(handle);
    if (!count) return QSML_E_INVALID;
    *count = 0;
    return QSML_OK;
}

qsml_status_t qsml_allocator_stats(qsml_ctx* handle, uint64_t* misses, uint64_t* hits,
                                   uint64_t* reserved_bytes, uint64_t* live_bytes) {
    QSML_CTX(handle);
    C_->allocator->stats(misses, hits, reserved_bytes, live_bytes);
    return QSML_OK;
}

}  // extern "C"
