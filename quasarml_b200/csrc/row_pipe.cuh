// Warp-per-row streaming through shared memory, for row-wise ops whose rows
// are a few KiB to a few tens of KiB (layer norm, softmax over the last axis).
//
// Each warp owns `slots` row buffers in dynamic shared memory and one
// mbarrier per buffer.  Lane 0 fills a buffer with one bulk copy
// (cp.async.bulk, completion counted in bytes on the buffer's mbarrier); the
// warp waits for it, runs the op on the row from shared memory, and refills
// the buffer with the warp's next-but-(slots-1) row.  The bytes in flight per
// SM are set by shared memory (one CTA per SM, up to ~220 KiB of rows), not by
// registers, and no barrier couples the warps: each row is reduced with warp
// shuffles only.
//
// Waits are bounded: a copy that has not landed after the context's wait
// limit (qsml_set_wait_limit; ~1 s by default) makes the warp stop, wait for
// every copy it still has in flight -- the late one included, each bounded
// by the full kWaitCycles -- and report failure; the kernel then records
// QSML_E_TIMEOUT in the context status word.
#pragma once

#include "qsml_internal.cuh"

namespace qsml {
namespace rowpipe {

constexpr int kMaxWarps = 16;
constexpr int kMaxSlots = 4;
constexpr long long kWaitCycles = kDefaultWaitCycles;  // ~1 s at 2 GHz
constexpr size_t kRingBudget = 220 * 1024;       // dynamic shared memory per CTA
constexpr uint32_t kMinRowBytes = 2048;

__device__ __forceinline__ uint32_t smem_addr(const void* p) {
    return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ bool bar_test(uint32_t bar, uint32_t parity) {
    uint32_t done;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(done)
        : "r"(bar), "r"(parity)
        : "memory");
    return done != 0;
}

// Never suspends the thread (mbarrier.try_wait, used above, may suspend it
// for a hardware-chosen time before it answers).
__device__ __forceinline__ bool bar_probe(uint32_t bar, uint32_t parity) {
    uint32_t done;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.test_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(done)
        : "r"(bar), "r"(parity)
        : "memory");
    return done != 0;
}

__device__ __forceinline__ bool bar_wait(uint32_t bar, uint32_t parity, long long limit) {
    if (limit < kWaitCycles) {
        // a lowered limit decides alone: poll without the hardware's suspend
        const long long t0 = clock64();
        while (!bar_probe(bar, parity))
            if (clock64() - t0 > limit) return false;
        return true;
    }
    if (bar_test(bar, parity)) return true;
    const long long t0 = clock64();
    while (!bar_test(bar, parity))
        if (clock64() - t0 > limit) return false;
    return true;
}

// Waits up to kWaitCycles for a copy this kernel issued, before it exits.
__device__ __forceinline__ void bar_drain(uint32_t bar, uint32_t parity) {
    const long long t0 = clock64();
    while (!bar_test(bar, parity) && clock64() - t0 < kWaitCycles) {
    }
}

// One bulk copy of `bytes` (a multiple of 16, both addresses 16-byte aligned)
// into shared memory, counted on `bar`.  Called by one lane.
__device__ __forceinline__ void fill(uint32_t dst, const void* src, uint32_t bytes, uint32_t bar) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(bar), "r"(bytes) : "memory");
    asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(dst),
                 "l"(src), "r"(bytes), "r"(bar)
                 : "memory");
}

// xor butterflies: every lane ends with the same bits
__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
    for (int m = 16; m >= 1; m >>= 1) v = __fadd_rn(v, __shfl_xor_sync(0xffffffffu, v, m));
    return v;
}

// Streams this warp's rows (warp g of G in the grid takes rows g, g + G, ...)
// through its buffers, calling body(row, buffer) with the whole warp.  `ring`
// is the CTA's row area (warp w's buffer s at (w * slots + s) * row_bytes) and
// `bars` the CTA's kMaxWarps * kMaxSlots mbarriers.  Returns false if a copy
// did not land within `limit` cycles.
template <class Body>
__device__ bool stream_rows(const unsigned char* src, int64_t rows, uint32_t row_bytes, int slots,
                            unsigned char* ring, uint64_t* bars, long long limit, Body&& body) {
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int64_t nwarps = static_cast<int64_t>(gridDim.x) * (blockDim.x >> 5);
    const int64_t first = static_cast<int64_t>(blockIdx.x) * (blockDim.x >> 5) + warp;
    unsigned char* mine = ring + static_cast<size_t>(warp) * slots * row_bytes;
    const uint32_t bar0 = smem_addr(bars + warp * kMaxSlots);
    if (lane == 0) {
        for (int s = 0; s < slots; ++s)
            asm volatile("mbarrier.init.shared::cta.b64 [%0], 1;" ::"r"(bar0 + 8u * s) : "memory");
        asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
        for (int s = 0; s < slots; ++s) {
            const int64_t r = first + s * nwarps;
            if (r < rows) fill(smem_addr(mine + s * row_bytes), src + r * row_bytes, row_bytes, bar0 + 8u * s);
        }
    }
    __syncwarp();
    bool ok = true;
    int64_t i = 0;
    for (int64_t row = first; row < rows; row += nwarps, ++i) {
        const int s = static_cast<int>(i % slots);
        const uint32_t parity = static_cast<uint32_t>((i / slots) & 1);
        int landed = 0;
        if (lane == 0) landed = bar_wait(bar0 + 8u * s, parity, limit) ? 1 : 0;
        landed = __shfl_sync(0xffffffffu, landed, 0);
        if (!landed) {
            ok = false;
            // every copy already issued -- the late one into buffer s and
            // those into the other buffers -- lands before the CTA exits
            if (lane == 0)
                for (int k = 0; k < slots; ++k) {
                    const int64_t j = i + k;
                    if (first + j * nwarps >= rows) break;
                    bar_drain(bar0 + 8u * static_cast<int>(j % slots), static_cast<uint32_t>((j / slots) & 1));
                }
            __syncwarp();
            break;
        }
        unsigned char* buf = mine + s * row_bytes;
        body(row, buf);
        __syncwarp();  // every lane is done with the buffer
        const int64_t next = row + static_cast<int64_t>(slots) * nwarps;
        if (lane == 0 && next < rows) {
            asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
            fill(smem_addr(buf), src + next * row_bytes, row_bytes, bar0 + 8u * s);
        }
    }
    return ok;
}

// Which rows go through the pipeline (measured on B200 with 16K-64K rows):
// binary16 rows of 2-8 KiB and binary32 rows of 2-4 KiB.  Wider rows leave too
// few warps per SM (one warp reduces a whole row), and binary32 rows of 8 KiB
// already reach ~0.95 of the copy bandwidth as one CTA per row.
inline bool use_pipe(uint64_t row_bytes, uint32_t elem_bytes) {
    const uint64_t max_bytes = elem_bytes == 2 ? 8192 : 4096;
    return row_bytes >= kMinRowBytes && row_bytes <= max_bytes;
}

// Wide rows (tens of KiB): the whole CTA works on one row at a time, held in
// one of two shared-memory buffers; while it reduces row i from one buffer,
// the bulk copy of its next row fills the other.  Same bounded waits as
// stream_rows; body(row, buffer) is called by every thread of the CTA and
// must end with the buffer no longer being read by any thread.
constexpr uint32_t kWideMinRowBytes = 32 * 1024 + 16;  // beyond the register kernels
constexpr size_t kWideMaxRowBytes = 108 * 1024;        // two buffers in ~216 KiB
// Widest row (16-byte packs) for which two CTAs' buffers share an SM.
constexpr int kWide256MaxPacks = 52 * 1024 / 16;

template <class Body>
__device__ bool stream_rows_cta(const unsigned char* src, int64_t rows, uint32_t row_bytes, unsigned char* ring,
                                uint64_t* bars, long long limit, Body&& body) {
    const int64_t G = gridDim.x;
    const uint32_t bar0 = smem_addr(bars);
    if (threadIdx.x == 0) {
        for (int s = 0; s < 2; ++s) asm volatile("mbarrier.init.shared::cta.b64 [%0], 1;" ::"r"(bar0 + 8u * s) : "memory");
        asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
        for (int s = 0; s < 2; ++s) {
            const int64_t r = blockIdx.x + s * G;
            if (r < rows) fill(smem_addr(ring + s * row_bytes), src + r * row_bytes, row_bytes, bar0 + 8u * s);
        }
    }
    __syncthreads();
    int64_t i = 0;
    for (int64_t row = blockIdx.x; row < rows; row += G, ++i) {
        const int s = static_cast<int>(i & 1);
        const uint32_t parity = static_cast<uint32_t>((i >> 1) & 1);
        const bool landed = bar_wait(bar0 + 8u * s, parity, limit);
        if (__syncthreads_or(!landed)) {
            // the late copy into buffer s and the other buffer's copy (if
            // any) land before the CTA exits
            if (threadIdx.x == 0) {
                bar_drain(bar0 + 8u * s, parity);
                if (row + G < rows) bar_drain(bar0 + 8u * (s ^ 1), static_cast<uint32_t>(((i + 1) >> 1) & 1));
            }
            __syncthreads();
            return false;
        }
        unsigned char* buf = ring + s * row_bytes;
        body(row, buf);
        __syncthreads();  // every thread is done with the buffer
        const int64_t next = row + 2 * G;
        if (threadIdx.x == 0 && next < rows) {
            asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
            fill(smem_addr(buf), src + next * row_bytes, row_bytes, bar0 + 8u * s);
        }
    }
    return true;
}

// Block-wide sum or max over the CTA (at most 32 warps): warp butterflies,
// one slot per warp, every thread combines the slots in warp order (same bits
// everywhere).  `slot` must not be reused before every thread has returned:
// callers alternate two slot arrays.
template <bool MAX>
__device__ __forceinline__ float cta_combine(float v, float* slot) {
    const int lane = threadIdx.x & 31, w = threadIdx.x >> 5, nw = blockDim.x >> 5;
#pragma unroll
    for (int m = 16; m >= 1; m >>= 1) {
        const float o = __shfl_xor_sync(0xffffffffu, v, m);
        if (MAX) {
            asm("max.NaN.f32 %0, %1, %2;" : "=f"(v) : "f"(v), "f"(o));
        } else {
            v = __fadd_rn(v, o);
        }
    }
    if (lane == 0) slot[w] = v;
    __syncthreads();
    float a = slot[0];
    for (int j = 1; j < nw; ++j) {
        if (MAX) {
            asm("max.NaN.f32 %0, %1, %2;" : "=f"(a) : "f"(a), "f"(slot[j]));
        } else {
            a = __fadd_rn(a, slot[j]);
        }
    }
    return a;
}

// binary16 rows from 8 KiB up (the register kernels are instruction-bound
// there), binary32 rows beyond what the register kernels hold.
inline bool use_wide(uint64_t row_bytes, uint32_t elem_bytes) {
    const uint64_t lo = elem_bytes == 2 ? 8192 + 16 : kWideMinRowBytes;
    return row_bytes >= lo && row_bytes <= kWideMaxRowBytes;
}

// Launch shape: one CTA per SM, `warps` warps with `slots` buffers each, the
// op's per-CTA parameters (`param_bytes`, e.g. gamma and beta) in front of
// the buffers.
struct Plan {
    int warps = 0, slots = 0;
    size_t smem = 0;
    unsigned grid = 0;
};

// Rows of `row_bytes` (16-byte multiple, at least kMinRowBytes) with every
// row start 16-byte aligned; false if the op should use another kernel.
inline bool plan(const Context* ctx, int64_t rows, uint64_t row_bytes, size_t param_bytes, Plan* p) {
    if (rows <= 0 || row_bytes < kMinRowBytes || row_bytes % 16 || param_bytes % 16) return false;
    if (param_bytes + 2 * row_bytes > kRingBudget) return false;
    const size_t nbuf = (kRingBudget - param_bytes) / row_bytes;
    // two buffers per warp (one row reduced, one in flight): more warps per
    // SM measured faster than deeper per-warp rings
    const int slots = 2;
    int warps = static_cast<int>(nbuf / slots);
    if (warps > kMaxWarps) warps = kMaxWarps;
    // no more warps in the grid than rows
    const int64_t per_cta = (rows + ctx->num_sms - 1) / ctx->num_sms;
    if (warps > per_cta) warps = static_cast<int>(per_cta);
    if (warps < 1) return false;
    int64_t grid = (rows + warps - 1) / warps;
    if (grid > ctx->num_sms) grid = ctx->num_sms;
    p->warps = warps;
    p->slots = slots;
    p->smem = param_bytes + static_cast<size_t>(warps) * slots * row_bytes;
    p->grid = static_cast<unsigned>(grid);
    return true;
}

}  // namespace rowpipe
}  // namespace qsml
