// Internal declarations shared by the libqsml_cuda translation units.
#pragma once

#include <cuda_runtime.h>
#include <cuda_fp16.h>

#include <cstdint>
#include <cstdio>
#include <cstring>
#include <map>
#include <mutex>
#include <utility>
#include <string>
#include <unordered_map>

#include "qsml_cuda.h"

namespace qsml {

// ---------------------------------------------------------------------------
// Caching allocator: size-binned blocks reused in the order of the context's
// single stream.  Replaces one VMA allocation per tensor
// (Backend/Vulkan/VulkanBackend.cpp:254-281 in the reference), which has no
// pooling at all.
// ---------------------------------------------------------------------------
class CachingAllocator {
public:
    explicit CachingAllocator(int device) : device_(device) {}
    ~CachingAllocator();
    qsml_status_t alloc(size_t bytes, void** ptr, std::string* err);
    qsml_status_t free(void* ptr, std::string* err);
    void release_cached();
    void stats(uint64_t* misses, uint64_t* hits, uint64_t* reserved, uint64_t* live);
    static size_t round_size(size_t bytes);

private:
    int device_;
    std::mutex mu_;
    std::multimap<size_t, void*> free_;          // rounded size -> block
    std::unordered_map<void*, size_t> live_;     // block -> rounded size
    uint64_t misses_ = 0, hits_ = 0, reserved_ = 0, live_bytes_ = 0;
    uint64_t malloc_calls_ = 0;
};

struct Staging;  // pinned staging buffers for pageable copies (transfer.cu)

// Per-device execution context: what a reference Device owned through its
// Backend (queue, allocator, kernel cache), on CUDA.
struct Context {
    int device = 0;
    cudaStream_t own_stream = nullptr;
    cudaStream_t stream = nullptr;
    int num_sms = 148;
    CachingAllocator* allocator = nullptr;
    // Scratch space for multi-CTA reductions: partials + a self-resetting
    // ticket counter.  Grown on demand, zero-initialised once.
    void* scratch = nullptr;
    size_t scratch_bytes = 0;
    // Device word where kernels with bounded waits report QSML_E_TIMEOUT;
    // qsml_synchronize reads and clears it.  Layout of the 256-byte block:
    // int at [0] the status code; int64 at byte 8 the wait limit in SM
    // cycles (0 = kDefaultWaitCycles), set with qsml_set_wait_limit.
    int* status = nullptr;
    // Overlap of independent reductions on the stream (qsml_set_overlap) and
    // the launch count the last plan_launch was made for.
    bool overlap = false;
    uint64_t planned_for = 0;
    uint64_t planned = 0, deferred = 0;  // plan_launch calls, and those that deferred
    // Scratch is handed out in kScratchSlots slots in turn, so that kernels
    // in flight together do not share ticket counters or partials.
    int scratch_slot = 0;
    uint64_t launches = 0;
    const char* last_kernel = "";  // a string literal of the launch site
    // Fused elementwise expressions: QSML_FUSE_MODE_* and which kernel ran.
    int fuse_mode = 0;
    uint64_t fuse_jit_launches = 0, fuse_interp_launches = 0;
    Staging* staging = nullptr;
    std::mutex err_mu;
    std::string last_error;
};

// Bounded device-side waits ---------------------------------------------------
// A kernel that waits on an mbarrier for data (a TMA or bulk copy, an MMA, a
// peer warp) gives up after this many SM clock cycles (~1 s at 2 GHz),
// records QSML_E_TIMEOUT in the context's status word and returns.  The
// context may lower the limit (qsml_set_wait_limit); the waits that only let
// a kernel's own copies and MMAs finish before it exits always keep this one.
constexpr long long kDefaultWaitCycles = 2000000000LL;

__device__ __forceinline__ long long wait_limit(const int* status) {
    const long long v = *reinterpret_cast<const volatile long long*>(status + 2);
    return v > 0 ? v : kDefaultWaitCycles;
}

// Error recording helpers ----------------------------------------------------
qsml_status_t set_error(Context* ctx, qsml_status_t st, const std::string& msg);
qsml_status_t check_cuda(Context* ctx, cudaError_t e, const char* what);
// Checks the launch that was just enqueued and counts it.
qsml_status_t after_launch(Context* ctx, const char* kernel);

// Overlap of independent kernels on one stream --------------------------------
// A kernel launched with programmatic dependent launch normally starts with
// pdl_begin(): it waits for the previous kernel on the stream to finish before
// touching memory.  Between reductions that share no buffer that wait only
// costs time: each short launch then pays its predecessor's drain and its own
// ramp.  plan_launch() therefore tracks, per stream, the library kernels that
// may still be running (the window: every kernel since the last one that
// waited at its start), each with the address ranges it reads and writes.  A
// kernel whose writes overlap nothing the window reads or writes, and whose
// reads overlap nothing the window writes, may "defer": it triggers its own
// dependents and reads at once (pdl_start(1)), and waits for its predecessor
// only at its end (pdl_end(1)), so kernels still complete in stream order and
// a later kernel that waits at its start still sees every write before it.
// Any other library launch on the stream closes the window (after_launch),
// and a context defers only after qsml_set_overlap(ctx, 1): the window knows
// the library's kernels only, not a foreign kernel that triggers early.
struct Span {
    uintptr_t lo = 0, hi = 0;  // [lo, hi)
};
inline Span span_of(const void* p, size_t bytes) {
    const uintptr_t a = reinterpret_cast<uintptr_t>(p);
    return Span{a, a + bytes};
}
// The bytes a strided view touches (its lowest to its highest element).
Span view_span(const qsml_tdesc* d);
struct Footprint {
    static constexpr int kMax = 3;
    Span reads[kMax], writes[kMax];
    int nr = 0, nw = 0;
    Footprint& read(Span s) { return add(reads, nr, s); }
    Footprint& write(Span s) { return add(writes, nw, s); }

private:
    // a fourth range widens the third (a larger footprint is only more
    // conservative)
    Footprint& add(Span* v, int& n, Span s) {
        if (s.hi <= s.lo) return *this;
        if (n < kMax) {
            v[n++] = s;
        } else {
            v[kMax - 1].lo = s.lo < v[kMax - 1].lo ? s.lo : v[kMax - 1].lo;
            v[kMax - 1].hi = s.hi > v[kMax - 1].hi ? s.hi : v[kMax - 1].hi;
        }
        return *this;
    }
};
// The defer flag (0 or 1) for the kernel about to be launched on ctx->stream
// with footprint f; records f in the stream's window.  The launch must follow
// at once and be checked with after_launch.
int plan_launch(Context* ctx, const Footprint& f);
// Forgets the stream's window (the next kernel waits at its start).
void end_window(cudaStream_t stream);

__device__ __forceinline__ void pdl_start(int defer) {
    if (!defer) asm volatile("griddepcontrol.wait;" ::: "memory");
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}
__device__ __forceinline__ void pdl_end(int defer) {
    if (defer) asm volatile("griddepcontrol.wait;" ::: "memory");
}

// Programmatic dependent launch for short memory-bound kernels that run back
// to back: the kernel is launched with programmatic stream serialization, so
// its CTAs may become resident while the previous kernel on the stream drains;
// it must begin with pdl_begin(), which waits until that kernel has completed
// and its writes are visible (griddepcontrol.wait) before touching memory, and
// then lets the next such kernel launch early.  Correct whatever the previous
// kernel on the stream is; without the launch attribute the wait returns at
// once.
__device__ __forceinline__ void pdl_begin() {
    asm volatile("griddepcontrol.wait;" ::: "memory");
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}

// Prefetch of `bytes` bytes (a multiple of 16, from a 16-byte aligned address)
// into L2.  A hint: it moves no data into the thread and does not take part
// in memory ordering (L2 is where global writes become coherent), so a kernel
// may issue it before pdl_begin() to start its first DRAM reads while the
// previous kernel on the stream drains; its loads after pdl_begin() still see
// every write that kernel made.
__device__ __forceinline__ void prefetch_l2(const void* p, uint32_t bytes) {
    asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(p), "r"(bytes) : "memory");
}

template <typename... KArgs, typename... Args>
cudaError_t launch_pdl(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t stream,
                       Args&&... args) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.dynamicSmemBytes = smem;
    cfg.stream = stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, kernel, std::forward<Args>(args)...);
}

constexpr int kScratchSlots = 4;
// Scratch of at least `bytes`.  Its first kScratchCounterBytes hold the
// reductions' ticket counters, which every kernel that uses them leaves at
// zero; other users place their data after that region.
constexpr size_t kScratchCounterBytes = size_t(64) << 10;
qsml_status_t get_scratch(Context* ctx, size_t bytes, void** ptr);

// Host <-> device copies (transfer.cu): pageable host memory of 8 MiB and
// more goes through pinned staging with multi-threaded host copies.
// copy_h2d returns once the source may be reused; copy_d2h once the data is
// in dst.
qsml_status_t copy_h2d(Context* ctx, void* dst, const void* src, size_t bytes);
qsml_status_t copy_d2h(Context* ctx, void* dst, const void* src, size_t bytes);
void staging_free(Context* ctx);

// Descriptor helpers ---------------------------------------------------------
inline int dtype_size(int32_t dt) {
    switch (dt) {
        case QSML_F32: case QSML_I32: case QSML_U32: return 4;
        case QSML_F16: case QSML_I16: case QSML_U16: return 2;
        case QSML_I8: case QSML_U8: return 1;
    }
    return 0;
}

inline int64_t numel(const qsml_tdesc* d) {
    int64_t n = 1;
    for (int i = 0; i < d->ndim; ++i) n *= d->shape[i];
    return n;
}

inline bool is_contiguous(const qsml_tdesc* d) {
    if (numel(d) == 0) return true;  // no element is addressed
    int64_t s = 1;
    for (int i = d->ndim - 1; i >= 0; --i) {
        if (d->shape[i] != 1 && d->stride[i] != s) return false;
        s *= d->shape[i];
    }
    return true;
}

// Validates ndim, shape and dtype; data may be null only when empty.
qsml_status_t check_desc(Context* ctx, const qsml_tdesc* d, const char* name);

inline bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

// A reduction of `a` over `axis` (QSML_AXIS_ALL = every element) viewed as
// [outer, k, inner] (Ops/Reduction.cpp:310-312).  Checks that `out` has the
// reduced shape: the axis dropped, or kept as 1 with keepdims, and shape [1]
// (or a 1-element rank <= 1 tensor) when nothing is left, like
// Reduction.cpp:297-305.  `what` prefixes the error message.
qsml_status_t plan_reduction(Context* ctx, const qsml_tdesc* a, int32_t axis, int32_t keepdims,
                             const qsml_tdesc* out, const char* what, int64_t* outer, int64_t* k,
                             int64_t* inner);

constexpr int kMaxDims = QSML_MAX_DIMS;

// A view whose elements fill one contiguous block in another dim order (a
// transpose or permutation of a contiguous tensor; strides >= 0), reduced
// over `axis`, is the contiguous reduction [outer, k, inner] of that block
// when the kept dims appear in the view in memory order (strides decreasing),
// so that the results come out in the view's order.  True (and the block's
// [outer, k, inner], base = a->data) in that case, and for QSML_AXIS_ALL on
// any such view; false for every other view, and when the reduced dim has
// extent 1.
bool dense_view_plan(const qsml_tdesc* a, int32_t axis, int64_t* outer, int64_t* k, int64_t* inner);

}  // namespace qsml

// Every entry point validates its context with this.
#define QSML_CTX(ctx_)                                                   \
    qsml::Context* C_ = reinterpret_cast<qsml::Context*>(ctx_);          \
    if (!C_) return QSML_E_INVALID;                                      \
    if (cudaSetDevice(C_->device) != cudaSuccess)                        \
        return qsml::set_error(C_, QSML_E_CUDA, "cudaSetDevice failed");

#define QSML_TRY_STATUS(expr)                \
    do {                                     \
        qsml_status_t st__ = (expr);         \
        if (st__ != QSML_OK) return st__;    \
    } while (0)
