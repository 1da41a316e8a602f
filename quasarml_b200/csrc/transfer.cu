// Host <-> device copies from ordinary (pageable) host memory.
//
// Reference: Backend/Vulkan/VulkanBackend.cpp:327-373 uploads and downloads
// through a staging buffer created per call, with a blocking fence wait.  A
// pageable cudaMemcpy is the CUDA counterpart and is limited by the driver's
// single-threaded staging (about 12 GB/s up, 21 GB/s down on this machine).
// Here large pageable copies go through two pinned 16 MiB staging buffers per
// context, and the host-side memcpy into or out of them is split across a
// small pool of threads, so the host copy of one chunk overlaps the DMA of
// the other:
//   * upload: memcpy chunk i into buffer i%2 (after that buffer's previous
//     DMA finished), enqueue its DMA on the context stream, record an event;
//     the call returns once every chunk is staged -- the source may be reused,
//     the DMAs stay ordered on the stream;
//   * download: the DMA of chunk i+1 is enqueued before chunk i is copied out
//     of its buffer; the call returns when the data is in place.
// Pinned host memory and small copies go straight to cudaMemcpyAsync.
#include <condition_variable>
#include <thread>
#include <vector>

#include "qsml_internal.cuh"

namespace qsml {
namespace {

constexpr size_t kStageChunk = size_t(16) << 20;   // bytes per staging buffer
constexpr size_t kStageMin = size_t(8) << 20;      // smaller copies go direct
constexpr size_t kPartMin = size_t(1) << 20;       // bytes per memcpy task

// Process-wide pool of memcpy threads; copy() splits one copy over them and
// the calling thread and returns when all parts are done.
class CopyPool {
public:
    static CopyPool& get() {
        static CopyPool pool;
        return pool;
    }

    void copy(void* dst, const void* src, size_t n) {
        std::lock_guard<std::mutex> one(call_mu_);  // one batch at a time
        const size_t workers = threads_.size() + 1;
        size_t parts = n / kPartMin;
        if (parts > workers) parts = workers;
        if (parts <= 1) {
            std::memcpy(dst, src, n);
            return;
        }
        {
            std::lock_guard<std::mutex> lk(mu_);
            const size_t per = (n + parts - 1) / parts;
            jobs_.clear();
            for (size_t p = 0; p < parts; ++p) {
                const size_t off = p * per;
                if (off >= n) break;
                jobs_.push_back({static_cast<char*>(dst) + off, static_cast<const char*>(src) + off,
                                 off + per < n ? per : n - off});
            }
            next_ = 0;
            pending_ = jobs_.size();
        }
        cv_.notify_all();
        run_jobs();
        std::unique_lock<std::mutex> lk(mu_);
        done_cv_.wait(lk, [&] { return pending_ == 0; });
    }

private:
    struct Job {
        char* d;
        const char* s;
        size_t n;
    };

    CopyPool() {
        unsigned hw = std::thread::hardware_concurrency();
        unsigned n = hw / 2;
        if (n > 7) n = 7;
        for (unsigned i = 0; i < n; ++i) threads_.emplace_back([this] { worker(); });
    }

    ~CopyPool() {
        {
            std::lock_guard<std::mutex> lk(mu_);
            stop_ = true;
        }
        cv_.notify_all();
        for (auto& t : threads_) t.join();
    }

    // Takes jobs until none is left; returns when the queue is empty.
    void run_jobs() {
        for (;;) {
            Job j;
            {
                std::lock_guard<std::mutex> lk(mu_);
                if (next_ >= jobs_.size()) return;
                j = jobs_[next_++];
            }
            std::memcpy(j.d, j.s, j.n);
            std::lock_guard<std::mutex> lk(mu_);
            if (--pending_ == 0) done_cv_.notify_all();
        }
    }

    void worker() {
        for (;;) {
            {
                std::unique_lock<std::mutex> lk(mu_);
                cv_.wait(lk, [&] { return stop_ || next_ < jobs_.size(); });
                if (stop_) return;
            }
            run_jobs();
        }
    }

    std::vector<std::thread> threads_;
    std::mutex call_mu_, mu_;
    std::condition_variable cv_, done_cv_;
    std::vector<Job> jobs_;
    size_t next_ = 0, pending_ = 0;
    bool stop_ = false;
};

}  // namespace

// Two pinned buffers and the events of the DMAs that last used them.
struct Staging {
    std::mutex mu;
    void* buf[2] = {nullptr, nullptr};
    cudaEvent_t ev[2] = {nullptr, nullptr};
    bool used[2] = {false, false};
};

namespace {

qsml_status_t staging_of(Context* ctx, Staging** out) {
    if (!ctx->staging) {
        auto* s = new Staging;
        for (int b = 0; b < 2; ++b) {
            cudaError_t e = cudaHostAlloc(&s->buf[b], kStageChunk, cudaHostAllocDefault);
            if (e == cudaSuccess) e = cudaEventCreateWithFlags(&s->ev[b], cudaEventDisableTiming);
            if (e != cudaSuccess) {
                for (int k = 0; k <= b; ++k) {
                    if (s->buf[k]) cudaFreeHost(s->buf[k]);
                    if (s->ev[k]) cudaEventDestroy(s->ev[k]);
                }
                delete s;
                return check_cuda(ctx, e, "staging buffers");
            }
        }
        ctx->staging = s;
    }
    *out = ctx->staging;
    return QSML_OK;
}

bool pageable(const void* p) {
    cudaPointerAttributes a;
    if (cudaPointerGetAttributes(&a, p) != cudaSuccess) {
        cudaGetLastError();
        return true;
    }
    return a.type == cudaMemoryTypeUnregistered;
}

// The buffer's previous DMA has finished.
qsml_status_t reclaim(Context* ctx, Staging* s, int b) {
    if (!s->used[b]) return QSML_OK;
    return check_cuda(ctx, cudaEventSynchronize(s->ev[b]), "staging wait");
}

}  // namespace

void staging_free(Context* ctx) {
    Staging* s = ctx->staging;
    if (!s) return;
    for (int b = 0; b < 2; ++b) {
        if (s->used[b]) cudaEventSynchronize(s->ev[b]);
        cudaEventDestroy(s->ev[b]);
        cudaFreeHost(s->buf[b]);
    }
    delete s;
    ctx->staging = nullptr;
}

qsml_status_t copy_h2d(Context* ctx, void* dst, const void* src, size_t bytes) {
    if (bytes < kStageMin || !pageable(src))
        return check_cuda(ctx, cudaMemcpyAsync(dst, src, bytes, cudaMemcpyHostToDevice, ctx->stream), "qsml_h2d");
    Staging* s = nullptr;
    QSML_TRY_STATUS(staging_of(ctx, &s));
    std::lock_guard<std::mutex> lk(s->mu);
    for (size_t off = 0, i = 0; off < bytes; off += kStageChunk, ++i) {
        const int b = static_cast<int>(i & 1);
        const size_t n = bytes - off < kStageChunk ? bytes - off : kStageChunk;
        QSML_TRY_STATUS(reclaim(ctx, s, b));
        CopyPool::get().copy(s->buf[b], static_cast<const char*>(src) + off, n);
        QSML_TRY_STATUS(check_cuda(
            ctx, cudaMemcpyAsync(static_cast<char*>(dst) + off, s->buf[b], n, cudaMemcpyHostToDevice, ctx->stream),
            "qsml_h2d"));
        QSML_TRY_STATUS(check_cuda(ctx, cudaEventRecord(s->ev[b], ctx->stream), "staging event"));
        s->used[b] = true;
    }
    return QSML_OK;
}

qsml_status_t copy_d2h(Context* ctx, void* dst, const void* src, size_t bytes) {
    if (bytes < kStageMin || !pageable(dst)) {
        QSML_TRY_STATUS(
            check_cuda(ctx, cudaMemcpyAsync(dst, src, bytes, cudaMemcpyDeviceToHost, ctx->stream), "qsml_d2h"));
        return check_cuda(ctx, cudaStreamSynchronize(ctx->stream), "qsml_d2h sync");
    }
    Staging* s = nullptr;
    QSML_TRY_STATUS(staging_of(ctx, &s));
    std::lock_guard<std::mutex> lk(s->mu);
    const size_t chunks = (bytes + kStageChunk - 1) / kStageChunk;
    auto enqueue = [&](size_t i) -> qsml_status_t {
        const int b = static_cast<int>(i & 1);
        const size_t off = i * kStageChunk;
        const size_t n = bytes - off < kStageChunk ? bytes - off : kStageChunk;
        QSML_TRY_STATUS(reclaim(ctx, s, b));
        QSML_TRY_STATUS(check_cuda(ctx,
                                   cudaMemcpyAsync(s->buf[b], static_cast<const char*>(src) + off, n,
                                                   cudaMemcpyDeviceToHost, ctx->stream),
                                   "qsml_d2h"));
        QSML_TRY_STATUS(check_cuda(ctx, cudaEventRecord(s->ev[b], ctx->stream), "staging event"));
        s->used[b] = true;
        return QSML_OK;
    };
    QSML_TRY_STATUS(enqueue(0));
    for (size_t i = 0; i < chunks; ++i) {
        if (i + 1 < chunks) QSML_TRY_STATUS(enqueue(i + 1));
        const int b = static_cast<int>(i & 1);
        const size_t off = i * kStageChunk;
        const size_t n = bytes - off < kStageChunk ? bytes - off : kStageChunk;
        QSML_TRY_STATUS(check_cuda(ctx, cudaEventSynchronize(s->ev[b]), "staging wait"));
        s->used[b] = false;
        CopyPool::get().copy(static_cast<char*>(dst) + off, s->buf[b], n);
    }
    return QSML_OK;
}

}  // namespace qsml
