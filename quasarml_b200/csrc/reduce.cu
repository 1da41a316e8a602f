// Reductions: sum / mean / max / min over one axis or over all elements.
//
// Reference: Ops/Reduction.cpp.  Full reductions there loop a one-element-
// per-thread workgroup tree (or subgroup) shader until one value is left
// (Reduction.cpp:213-281), allocating and zero-uploading a tensor per pass;
// axis sums run one thread per output with a serial k loop
// (Reduction.cpp:293-345); axis max/min are stubs (Reduction.cpp:366-382).
//
// Here the input is viewed as [outer, k, inner] (Reduction.cpp:310-312) and
// one of these kernels runs, chosen from the shape alone:
//   * k_reduce_seg   -- inner == 1 with few long rows, including the full
//                       reduction (one row).  Each row is cut into a number
//                       of interleaved slices fixed by the shape; a slice is
//                       reduced by one CTA in a fixed order and its partial
//                       stored; the CTA that takes the last ticket of a row
//                       (atomic counter per row) combines that row's
//                       partials in slice order.  One launch, deterministic
//                       for a given shape whatever the grid size.
//   * k_reduce_rows  -- inner == 1 with many rows: one warp per row.
//   * k_reduce_cols  -- inner > 1: lanes own 16-byte column vectors (loads
//                       coalesced along inner), the CTA's warps split k into
//                       contiguous slices, slices combine in warp order;
//   * k_reduce_cols_split -- k_reduce_cols for fewer than 128 column tiles
//                       over a long k: k also cut over CTAs, partials combined
//                       in chunk order by the CTA taking the last ticket;
//   * k_reduce_cols_wide -- inner > 1 with 16-byte column vectors, k <= 64 and
//                       many columns: each warp one column span over all k,
//                       the CTA's 8 warps neighbouring spans of the same rows.
// The kernels are launched with programmatic dependent launch (launch_pdl):
// each waits for the previous kernel on the stream before touching memory, but
// its CTAs are already resident when that kernel drains.  For binary16 inputs
// (10-15 us launches) each warp first prefetches its first batch of loads into
// L2, so DRAM reads start during that drain (measured on B200: +2 to +8 % for
// binary16, a loss for the longer binary32 launches, which do not prefetch).
// Accumulation is binary32 (binary16 inputs widen exactly); max/min use PTX
// max.NaN/min.NaN, so the result is exact and order-free (IEEE 754-2019
// maximum/minimum: -0 < +0, NaN wins as 0x7fffffff).
// mean = sum * (1.0f / (float)k), a reciprocal multiply like
// Reduction.cpp:347-356; the reciprocal is rounded on the host.
#include "qsml_internal.cuh"

#include <cuda.h>

#include <climits>

namespace qsml {
namespace {

constexpr int kRT = 256;             // threads of the segment kernel
constexpr int kSegIters = 8;         // 16-byte loads in flight per thread
constexpr int64_t kSegMaxUnits = 8192;  // slices per launch, all rows together
constexpr int64_t kSegSliceElems = 32768;  // elements per slice of a long row
constexpr int64_t kWideMaxK = 64;       // longest k the wide column kernel takes
constexpr int64_t kSplitBelowTiles = 128;  // column tiles below which k is also split over CTAs
constexpr int kMaxSegments = 16384;  // ticket counters kept in scratch
constexpr size_t kCounterBytes = kMaxSegments * sizeof(unsigned);
static_assert(kCounterBytes == kScratchCounterBytes, "counters fill the reserved scratch region");

template <typename T> struct alignas(16) Pack {
    static constexpr int N = 16 / sizeof(T);
    T v[N];
};

__device__ __forceinline__ float to_f(float v) { return v; }
__device__ __forceinline__ float to_f(__half v) { return __half2float(v); }
__device__ __forceinline__ void from_f(float v, float* o) { *o = v; }
__device__ __forceinline__ void from_f(float v, __half* o) { *o = __float2half_rn(v); }

// Slices per row of the segment kernel, from the shape alone: about
// kSegSliceElems elements per slice (measured best on B200 for 33.5M-element
// rows in binary32 and binary16 alike), at most kSegMaxUnits slices in all.
inline int64_t seg_slices(int64_t rows, int64_t k) {
    int64_t P = (k + kSegSliceElems - 1) / kSegSliceElems;
    const int64_t cap = kSegMaxUnits / rows;
    if (P > cap) P = cap;
    if (P < 1) P = 1;
    return P;
}

template <int OP> struct Red;
template <> struct Red<QSML_RED_SUM> {
    using V = float;
    static __device__ __forceinline__ V ident() { return 0.0f; }
    static __device__ __forceinline__ V lift(float x) { return x; }
    static __device__ __forceinline__ V comb(V a, V b) { return __fadd_rn(a, b); }
    static __device__ __forceinline__ float fin(V a, float) { return a; }
    static __device__ __forceinline__ V shfl(V v, int m) { return __shfl_xor_sync(0xffffffffu, v, m); }
};
template <> struct Red<QSML_RED_MEAN> : Red<QSML_RED_SUM> {
    static __device__ __forceinline__ float fin(V a, float scale) { return __fmul_rn(a, scale); }
};
// max/min: PTX max.NaN / min.NaN return the canonical NaN 0x7fffffff when
// either operand is NaN and order -0 below +0, i.e. IEEE 754-2019
// maximum/minimum in one instruction; the result is independent of the
// combine order.
__device__ __forceinline__ float max_nan(float a, float b) {
    float r;
    asm("max.NaN.f32 %0, %1, %2;" : "=f"(r) : "f"(a), "f"(b));
    return r;
}
__device__ __forceinline__ float min_nan(float a, float b) {
    float r;
    asm("min.NaN.f32 %0, %1, %2;" : "=f"(r) : "f"(a), "f"(b));
    return r;
}
template <> struct Red<QSML_RED_MAX> {
    using V = float;
    static __device__ __forceinline__ V ident() { return -INFINITY; }
    static __device__ __forceinline__ V lift(float x) { return x; }
    static __device__ __forceinline__ V comb(V a, V b) { return max_nan(a, b); }
    static __device__ __forceinline__ float fin(V a, float) { return a; }
    static __device__ __forceinline__ V shfl(V v, int m) { return __shfl_xor_sync(0xffffffffu, v, m); }
};
template <> struct Red<QSML_RED_MIN> {
    using V = float;
    static __device__ __forceinline__ V ident() { return INFINITY; }
    static __device__ __forceinline__ V lift(float x) { return x; }
    static __device__ __forceinline__ V comb(V a, V b) { return min_nan(a, b); }
    static __device__ __forceinline__ float fin(V a, float) { return a; }
    static __device__ __forceinline__ V shfl(V v, int m) { return __shfl_xor_sync(0xffffffffu, v, m); }
};

// prod (Reduction.cpp:190-211: `shared_data[tid] *= ...`, identity 1).
template <> struct Red<QSML_RED_PROD> {
    using V = float;
    static __device__ __forceinline__ V ident() { return 1.0f; }
    static __device__ __forceinline__ V lift(float x) { return x; }
    static __device__ __forceinline__ V comb(V a, V b) { return __fmul_rn(a, b); }
    static __device__ __forceinline__ float fin(V a, float) { return a; }
    static __device__ __forceinline__ V shfl(V v, int m) { return __shfl_xor_sync(0xffffffffu, v, m); }
};

// One element into a column accumulator.  A binary16 sum uses the sm_100
// mixed-precision add (add.rn.f32.f16: the half widens exactly, one rounding),
// the same bits as widening first and adding in binary32, in one instruction
// (measured on B200: binary16 column launches 3-5 % shorter; the segment
// kernel's single accumulator chain measured slower with it, so it widens).
template <int OP>
__device__ __forceinline__ float accum(float acc, float v) {
    return Red<OP>::comb(acc, Red<OP>::lift(v));
}
template <int OP>
__device__ __forceinline__ float accum(float acc, __half v) {
    if constexpr (OP == QSML_RED_SUM || OP == QSML_RED_MEAN) {
        asm("add.rn.f32.f16 %0, %1, %0;" : "+f"(acc) : "h"(__half_as_ushort(v)));
        return acc;
    } else {
        return Red<OP>::comb(acc, Red<OP>::lift(__half2float(v)));
    }
}

// Butterfly: every lane ends with the same bits (each step combines the same
// two operands on both partner lanes, and the ops are commutative).
template <int OP>
__device__ __forceinline__ typename Red<OP>::V warp_reduce(typename Red<OP>::V v) {
#pragma unroll
    for (int m = 16; m >= 1; m >>= 1) v = Red<OP>::comb(v, Red<OP>::shfl(v, m));
    return v;
}

// Block of kRT threads; result valid in every thread.
template <int OP>
__device__ __forceinline__ typename Red<OP>::V block_reduce(typename Red<OP>::V v) {
    using R = Red<OP>;
    __shared__ typename R::V sh[kRT / 32];
    const int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
    v = warp_reduce<OP>(v);
    __syncthreads();  // sh may still be read by a previous call
    if (lane == 0) sh[w] = v;
    __syncthreads();
    typename R::V t = lane < kRT / 32 ? sh[lane] : R::ident();
    return warp_reduce<OP>(t);
}

// ---------------------------------------------------------------------------
// Segment kernel: x = [nseg rows, len] contiguous.  Each row is split into
// P interleaved slices (P depends on the shape only); work unit (s, j), one
// CTA, reduces slice j of row s with 16-byte loads, kSegIters in flight per
// thread, in a fixed order, then one block reduction gives partial (s, j).
// The unit that takes the row's last ticket combines its P partials in slice
// order.  The result depends on the shape alone, not on the grid size.
// ---------------------------------------------------------------------------
template <typename T, typename OT, int OP, bool VEC>
__global__ void __launch_bounds__(kRT) k_reduce_seg(const T* __restrict__ x, int64_t nseg, int64_t len,
                                                    int64_t P, OT* __restrict__ out, float scale,
                                                    unsigned* __restrict__ counters,
                                                    typename Red<OP>::V* __restrict__ partials, int defer) {
    using R = Red<OP>;
    using V = typename R::V;
    constexpr int PV = Pack<T>::N;
    __shared__ bool s_last;
    const int t = threadIdx.x;
    const int64_t units = nseg * P;
    if (VEC && sizeof(T) == 2 && t < kSegIters && blockIdx.x < units) {
        // the first batch of this CTA's first slice: kSegIters blocks of 256 packs
        const int64_t s = blockIdx.x / P, j = blockIdx.x - s * P;
        const int64_t npk = len / PV;
        const int64_t q = j * kRT + t * P * kRT;
        if (q < npk) {
            const int64_t n = npk - q < kRT ? npk - q : kRT;
            prefetch_l2(reinterpret_cast<const Pack<T>*>(x + s * len) + q, static_cast<uint32_t>(n * 16));
        }
    }
    pdl_start(defer);
    for (int64_t w = blockIdx.x; w < units; w += gridDim.x) {
        const int64_t s = w / P, j = w - s * P;
        const T* row = x + s * len;
        V acc = R::ident();
        // Slice j of a row is the interleaved set of 256-thread blocks
        // j, j + P, j + 2P, ...: at any moment the P units of a row stream
        // through one contiguous region (measured faster on B200 than
        // contiguous slices).
        const int64_t stride = P * kRT;
        if (VEC) {
            const int64_t npk = len / PV;
            const Pack<T>* p = reinterpret_cast<const Pack<T>*>(row);
            int64_t q = j * kRT + t;
            for (; q + (kSegIters - 1) * stride < npk; q += kSegIters * stride) {
                Pack<T> r[kSegIters];
#pragma unroll
                for (int i = 0; i < kSegIters; ++i) r[i] = p[q + i * stride];
#pragma unroll
                for (int i = 0; i < kSegIters; ++i)
#pragma unroll
                    for (int e = 0; e < PV; ++e) acc = R::comb(acc, R::lift(to_f(r[i].v[e])));
            }
            for (; q < npk; q += stride) {
                Pack<T> r = p[q];
#pragma unroll
                for (int e = 0; e < PV; ++e) acc = R::comb(acc, R::lift(to_f(r.v[e])));
            }
            // elements past the last whole pack belong to the last slice
            if (j == P - 1 && t < len - npk * PV) acc = R::comb(acc, R::lift(to_f(row[npk * PV + t])));
        } else {
            for (int64_t q = j * kRT + t; q < len; q += stride) acc = R::comb(acc, R::lift(to_f(row[q])));
        }
        acc = block_reduce<OP>(acc);
        if (t == 0) {
            partials[w] = acc;
            __threadfence();
            unsigned ticket = atomicAdd(&counters[s], 1u);
            s_last = ticket == static_cast<unsigned>(P - 1);
        }
        __syncthreads();
        if (s_last) {
            // This unit completed row s: combine its partials in slice order.
            __threadfence();
            V a = R::ident();
            for (int64_t i = t; i < P; i += kRT) a = R::comb(a, __ldcg(&partials[s * P + i]));
            a = block_reduce<OP>(a);
            if (t == 0) {
                from_f(R::fin(a, scale), &out[s]);
                counters[s] = 0;  // ready for the next launch on this stream
            }
        }
        __syncthreads();
    }
    pdl_end(defer);
}

// ---------------------------------------------------------------------------
// Row kernel: one warp per row of `len` contiguous elements.
// ---------------------------------------------------------------------------
template <typename T, typename OT, int OP, bool VEC>
__global__ void __launch_bounds__(256) k_reduce_rows(const T* __restrict__ x, int64_t rows, int64_t len,
                                                     OT* __restrict__ out, float scale, int defer) {
    using R = Red<OP>;
    using V = typename R::V;
    constexpr int PV = Pack<T>::N;
    constexpr int U = 4;
    const int lane = threadIdx.x & 31;
    if (VEC && sizeof(T) == 2 && lane == 0) {
        // this warp's first row, up to 16 KiB of it
        const int64_t r = static_cast<int64_t>(blockIdx.x) * (blockDim.x >> 5) + (threadIdx.x >> 5);
        const int64_t bytes = (len / PV) * 16;
        if (r < rows && bytes > 0) prefetch_l2(x + r * len, static_cast<uint32_t>(bytes < 16384 ? bytes : 16384));
    }
    pdl_start(defer);
    const int64_t warps = static_cast<int64_t>(gridDim.x) * (blockDim.x >> 5);
    for (int64_t r = static_cast<int64_t>(blockIdx.x) * (blockDim.x >> 5) + (threadIdx.x >> 5); r < rows; r += warps) {
        const T* row = x + r * len;
        V acc = R::ident();
        if (VEC) {
            const Pack<T>* p = reinterpret_cast<const Pack<T>*>(row);
            const int64_t np = len / PV;
            int64_t i = lane;
            for (; i + (U - 1) * 32 < np; i += U * 32) {
                Pack<T> v[U];
#pragma unroll
                for (int u = 0; u < U; ++u) v[u] = p[i + u * 32];
#pragma unroll
                for (int u = 0; u < U; ++u)
#pragma unroll
                    for (int e = 0; e < PV; ++e) acc = R::comb(acc, R::lift(to_f(v[u].v[e])));
            }
            for (; i < np; i += 32) {
                Pack<T> v = p[i];
#pragma unroll
                for (int e = 0; e < PV; ++e) acc = R::comb(acc, R::lift(to_f(v.v[e])));
            }
        } else {
            for (int64_t j = lane; j < len; j += 32) acc = R::comb(acc, R::lift(to_f(row[j])));
        }
        acc = warp_reduce<OP>(acc);
        if (lane == 0) from_f(R::fin(acc, scale), &out[r]);
    }
    pdl_end(defer);
}

// ---------------------------------------------------------------------------
// Column kernel: out[o, i] = reduce_k x[o, k, i]; block (32, W).
// ---------------------------------------------------------------------------
template <typename T, typename OT, int OP, bool VEC>
__global__ void k_reduce_cols(const T* __restrict__ x, int64_t outer, int64_t k, int64_t inner,
                              int64_t tiles_per_o, OT* __restrict__ out, float scale, int defer) {
    using R = Red<OP>;
    using V = typename R::V;
    constexpr int PV = VEC ? Pack<T>::N : 1;
    constexpr int U = 8;
    extern __shared__ unsigned char smem_raw[];
    V* red = reinterpret_cast<V*>(smem_raw);
    const int lane = threadIdx.x, w = threadIdx.y, W = blockDim.y;
    const int64_t tile = blockIdx.x;
    const int64_t o = tile / tiles_per_o;
    const int64_t tc0 = (tile - o * tiles_per_o) * (32 * PV);
    const int64_t c0 = tc0 + static_cast<int64_t>(lane) * PV;
    const int64_t kper = (k + W - 1) / W;
    const int64_t k0 = w * kper;
    const int64_t k1 = k0 + kper < k ? k0 + kper : k;
    if (VEC && sizeof(T) == 2 && lane < U && k0 + lane < k1 && o < outer) {
        // the warp's first batch: U rows of the tile's 32 x 16-byte span
        const int64_t span = inner - tc0 < 32 * PV ? inner - tc0 : 32 * PV;
        prefetch_l2(x + (o * k + k0 + lane) * inner + tc0, static_cast<uint32_t>(span * sizeof(T)));
    }
    pdl_start(defer);
    V acc[PV];
#pragma unroll
    for (int e = 0; e < PV; ++e) acc[e] = R::ident();
    if (o < outer && c0 < inner) {
        const T* base = x + (o * k) * inner + c0;
        int64_t kk = k0;
        if (VEC) {
            for (; kk + U <= k1; kk += U) {
                Pack<T> v[U];
#pragma unroll
                for (int u = 0; u < U; ++u) v[u] = *reinterpret_cast<const Pack<T>*>(base + (kk + u) * inner);
#pragma unroll
                for (int u = 0; u < U; ++u)
#pragma unroll
                    for (int e = 0; e < PV; ++e) acc[e] = accum<OP>(acc[e], v[u].v[e]);
            }
            for (; kk < k1; ++kk) {
                Pack<T> v = *reinterpret_cast<const Pack<T>*>(base + kk * inner);
#pragma unroll
                for (int e = 0; e < PV; ++e) acc[e] = accum<OP>(acc[e], v.v[e]);
            }
        } else {
            for (; kk + U <= k1; kk += U) {
                T v[U];
#pragma unroll
                for (int u = 0; u < U; ++u) v[u] = base[(kk + u) * inner];
#pragma unroll
                for (int u = 0; u < U; ++u) acc[0] = R::comb(acc[0], R::lift(to_f(v[u])));
            }
            for (; kk < k1; ++kk) acc[0] = R::comb(acc[0], R::lift(to_f(base[kk * inner])));
        }
    }
#pragma unroll
    for (int e = 0; e < PV; ++e) red[(w * 32 + lane) * PV + e] = acc[e];
    __syncthreads();
    // Combine the W slices in slice order, one output column per thread.
    const int tid = w * 32 + lane;
    for (int col = tid; col < 32 * PV; col += 32 * W) {
        V a = red[col];
        for (int ww = 1; ww < W; ++ww) a = R::comb(a, red[ww * 32 * PV + col]);
        const int64_t ci = (tile - o * tiles_per_o) * (32 * PV) + col;
        if (o < outer && ci < inner) from_f(R::fin(a, scale), &out[o * inner + ci]);
    }
    pdl_end(defer);
}

// ---------------------------------------------------------------------------
// Split column kernel, for few column tiles over a long k (X[8192,8192] over
// axis 0 has 64 tiles of fp32): k_reduce_cols with k also cut into S
// contiguous chunks over S CTAs (unit = (chunk s, tile), tiles fastest).
// CTA (s, tile) reduces its chunk like k_reduce_cols (warps take contiguous
// sub-chunks, combined in warp order) and stores one binary32 partial per
// column; the CTA taking the tile's last ticket combines the S partials in
// chunk order.  S comes from the shape alone.  (For the 256-512 tiles of
// X[64,512,1024] over axis 1 the unsplit kernel measured faster on B200.)
// ---------------------------------------------------------------------------
template <typename T, typename OT, int OP>
__global__ void k_reduce_cols_split(const T* __restrict__ x, int64_t outer, int64_t k, int64_t inner,
                                    int64_t tiles_per_o, int64_t S, OT* __restrict__ out, float scale,
                                    unsigned* __restrict__ counters, typename Red<OP>::V* __restrict__ partials,
                                    int defer) {
    using R = Red<OP>;
    using V = typename R::V;
    constexpr int PV = Pack<T>::N;
    constexpr int NC = 32 * PV;
    constexpr int U = 8;
    extern __shared__ unsigned char smem_raw[];
    V* red = reinterpret_cast<V*>(smem_raw);
    __shared__ bool s_last;
    const int lane = threadIdx.x, w = threadIdx.y, W = blockDim.y;
    const int64_t tiles = tiles_per_o * outer;
    const int64_t s = blockIdx.x / tiles;
    const int64_t tile = blockIdx.x - s * tiles;
    const int64_t o = tile / tiles_per_o;
    const int64_t tc0 = (tile - o * tiles_per_o) * NC;
    const int64_t c0 = tc0 + static_cast<int64_t>(lane) * PV;
    const int64_t kc = (k + S - 1) / S;
    const int64_t ks = s * kc, ke = ks + kc < k ? ks + kc : k;
    const int64_t kper = (kc + W - 1) / W;
    const int64_t k0 = ks + w * kper;
    const int64_t k1 = k0 + kper < ke ? k0 + kper : ke;
    pdl_start(defer);
    V acc[PV];
#pragma unroll
    for (int e = 0; e < PV; ++e) acc[e] = R::ident();
    if (c0 < inner) {
        const T* base = x + (o * k) * inner + c0;
        int64_t kk = k0;
        for (; kk + U <= k1; kk += U) {
            Pack<T> v[U];
#pragma unroll
            for (int u = 0; u < U; ++u) v[u] = *reinterpret_cast<const Pack<T>*>(base + (kk + u) * inner);
#pragma unroll
            for (int u = 0; u < U; ++u)
#pragma unroll
                for (int e = 0; e < PV; ++e) acc[e] = accum<OP>(acc[e], v[u].v[e]);
        }
        for (; kk < k1; ++kk) {
            Pack<T> v = *reinterpret_cast<const Pack<T>*>(base + kk * inner);
#pragma unroll
            for (int e = 0; e < PV; ++e) acc[e] = accum<OP>(acc[e], v.v[e]);
        }
    }
#pragma unroll
    for (int e = 0; e < PV; ++e) red[(w * 32 + lane) * PV + e] = acc[e];
    __syncthreads();
    const int tid = w * 32 + lane;
    for (int col = tid; col < NC; col += 32 * W) {
        V a = red[col];
        for (int ww = 1; ww < W; ++ww) a = R::comb(a, red[ww * NC + col]);
        partials[(tile * S + s) * NC + col] = a;
    }
    __threadfence();
    __syncthreads();
    if (tid == 0) s_last = atomicAdd(&counters[tile], 1u) == static_cast<unsigned>(S - 1);
    __syncthreads();
    if (s_last) {
        // This CTA completed the tile: combine its S partials in chunk order.
        __threadfence();
        for (int col = tid; col < NC; col += 32 * W) {
            V a = __ldcg(&partials[tile * S * NC + col]);
            for (int64_t j = 1; j < S; ++j) a = R::comb(a, __ldcg(&partials[(tile * S + j) * NC + col]));
            const int64_t ci = tc0 + col;
            if (ci < inner) from_f(R::fin(a, scale), &out[o * inner + ci]);
        }
        if (tid == 0) counters[tile] = 0;  // ready for the next launch on this stream
    }
    pdl_end(defer);
}

// ---------------------------------------------------------------------------
// Wide column kernel (16-byte column vectors, short k, many columns): a CTA
// takes 8 neighbouring spans (warp w: span w, 32 lanes x PV columns) over all
// k rows, so each of its load instructions reads 4 KiB of one row in one
// piece and the CTAs in flight together read whole rows.  Each lane's
// columns are reduced in k order.
// ---------------------------------------------------------------------------
template <typename T, typename OT, int OP>
__global__ void __launch_bounds__(256) k_reduce_cols_wide(const T* __restrict__ x, int64_t outer, int64_t k,
                                                          int64_t inner, int64_t tiles_per_o, int64_t groups_per_o,
                                                          OT* __restrict__ out, float scale, int defer) {
    using R = Red<OP>;
    using V = typename R::V;
    constexpr int PV = Pack<T>::N;
    constexpr int U = 8;
    constexpr int NCOL = 32 * PV;
    const int lane = threadIdx.x, w = threadIdx.y;
    const int64_t grp = blockIdx.x;
    const int64_t o = grp / groups_per_o;
    const int64_t span = (grp - o * groups_per_o) * 8 + w;  // tile within o
    const int64_t c0 = span * NCOL + static_cast<int64_t>(lane) * PV;
    if (sizeof(T) == 2 && lane < U && lane < k && span < tiles_per_o) {
        // the warp's first batch: U rows of its 32 x 16-byte span
        const int64_t n = inner - span * NCOL < NCOL ? inner - span * NCOL : NCOL;
        prefetch_l2(x + (o * k + lane) * inner + span * NCOL, static_cast<uint32_t>(n * sizeof(T)));
    }
    pdl_start(defer);
    if (span >= tiles_per_o || c0 >= inner) {
        pdl_end(defer);
        return;
    }
    V acc[PV];
#pragma unroll
    for (int e = 0; e < PV; ++e) acc[e] = R::ident();
    const T* base = x + (o * k) * inner + c0;
    int64_t kk = 0;
    for (; kk + U <= k; kk += U) {
        Pack<T> v[U];
#pragma unroll
        for (int u = 0; u < U; ++u) v[u] = *reinterpret_cast<const Pack<T>*>(base + (kk + u) * inner);
#pragma unroll
        for (int u = 0; u < U; ++u)
#pragma unroll
            for (int e = 0; e < PV; ++e) acc[e] = accum<OP>(acc[e], v[u].v[e]);
    }
    for (; kk < k; ++kk) {
        Pack<T> v = *reinterpret_cast<const Pack<T>*>(base + kk * inner);
#pragma unroll
        for (int e = 0; e < PV; ++e) acc[e] = accum<OP>(acc[e], v.v[e]);
    }
#pragma unroll
    for (int e = 0; e < PV; ++e)
        if (c0 + e < inner) from_f(R::fin(acc[e], scale), &out[o * inner + c0 + e]);
    pdl_end(defer);
}

// ---------------------------------------------------------------------------
// Host dispatch
// ---------------------------------------------------------------------------
// scale_override > 0 replaces a mean's 1/k (a mean over more elements than
// this call reduces, as in the second stage of a strided full reduction).
template <typename T, typename OT, int OP>
qsml_status_t run_reduce(Context* ctx, const T* x, int64_t outer, int64_t k, int64_t inner, OT* out,
                         float scale_override = 0.0f) {
    using V = typename Red<OP>::V;
    constexpr int PV = Pack<T>::N;
    const float scale = scale_override > 0.0f ? scale_override : 1.0f / static_cast<float>(k);
    const bool x_al = aligned16(x);
    // what the launch reads and writes, for overlap with the kernels before it
    Footprint fp;
    fp.read(span_of(x, static_cast<size_t>(outer * k * inner) * sizeof(T)))
        .write(span_of(out, static_cast<size_t>(outer * inner) * sizeof(OT)));
    if (inner == 1 && (outer == 1 || (outer < 592 && k >= 8192))) {
        // Segment kernel.
        if (outer > kMaxSegments) return set_error(ctx, QSML_E_UNSUPPORTED, "too many segments");
        // One row may end in a partial pack (handled in-kernel); several rows
        // need every row start 16-byte aligned.
        const bool vec = x_al && (outer == 1 || (k * static_cast<int64_t>(sizeof(T))) % 16 == 0);
        const int64_t P = seg_slices(outer, k);
        const int64_t units = outer * P;
        void* scratch = nullptr;
        QSML_TRY_STATUS(get_scratch(ctx, kCounterBytes + static_cast<size_t>(units) * sizeof(V), &scratch));
        unsigned* counters = static_cast<unsigned*>(scratch);
        V* partials = reinterpret_cast<V*>(static_cast<char*>(scratch) + kCounterBytes);
        const int64_t grid = units;  // one slice per CTA
        const int defer = plan_launch(ctx, fp.write(span_of(scratch, kCounterBytes + units * sizeof(V))));
        const cudaError_t e =
            vec ? launch_pdl(k_reduce_seg<T, OT, OP, true>, dim3(static_cast<unsigned>(grid)), dim3(kRT), 0,
                             ctx->stream, x, outer, k, P, out, scale, counters, partials, defer)
                : launch_pdl(k_reduce_seg<T, OT, OP, false>, dim3(static_cast<unsigned>(grid)), dim3(kRT), 0,
                             ctx->stream, x, outer, k, P, out, scale, counters, partials, defer);
        if (e != cudaSuccess) return check_cuda(ctx, e, "k_reduce_seg");
        return after_launch(ctx, "k_reduce_seg");
    }
    if (inner == 1) {
        const bool vec = x_al && (k * static_cast<int64_t>(sizeof(T))) % 16 == 0;
        int64_t grid = (outer + 7) / 8;  // 8 warps per CTA
        int64_t cap = static_cast<int64_t>(ctx->num_sms) * 32;
        if (grid > cap) grid = cap;
        const int defer = plan_launch(ctx, fp);
        const cudaError_t e =
            vec ? launch_pdl(k_reduce_rows<T, OT, OP, true>, dim3(static_cast<unsigned>(grid)), dim3(256), 0,
                             ctx->stream, x, outer, k, out, scale, defer)
                : launch_pdl(k_reduce_rows<T, OT, OP, false>, dim3(static_cast<unsigned>(grid)), dim3(256), 0,
                             ctx->stream, x, outer, k, out, scale, defer);
        if (e != cudaSuccess) return check_cuda(ctx, e, "k_reduce_rows");
        return after_launch(ctx, "k_reduce_rows");
    }
    const bool vec = x_al && (inner * static_cast<int64_t>(sizeof(T))) % 16 == 0;
    if (vec && inner >= 8 * 32 * PV && k <= kWideMaxK) {
        // Wide column kernel, when its CTAs are enough to fill the SMs twice.
        const int64_t tiles_per_o = (inner + 32 * PV - 1) / (32 * PV);
        const int64_t groups_per_o = (tiles_per_o + 7) / 8;
        const int64_t groups = groups_per_o * outer;
        if (groups >= 2 * static_cast<int64_t>(ctx->num_sms) && groups <= INT32_MAX) {
            const int defer = plan_launch(ctx, fp);
            const cudaError_t e = launch_pdl(k_reduce_cols_wide<T, OT, OP>, dim3(static_cast<unsigned>(groups)),
                                             dim3(32, 8), 0, ctx->stream, x, outer, k, inner, tiles_per_o,
                                             groups_per_o, out, scale, defer);
            if (e != cudaSuccess) return check_cuda(ctx, e, "k_reduce_cols_wide");
            return after_launch(ctx, "k_reduce_cols_wide");
        }
    }
    const int pv = vec ? PV : 1;
    const int64_t tiles_per_o = (inner + 32 * pv - 1) / (32 * pv);
    const int64_t tiles = tiles_per_o * outer;
    if (vec && tiles < kSplitBelowTiles) {
        // Few tiles over a long k: 16 warps a CTA, k cut over S CTAs (about
        // 2 * kSplitBelowTiles CTAs, at least 32 rows per warp).
        const int64_t W = 16;
        int64_t S = (2 * kSplitBelowTiles + tiles - 1) / tiles;
        const int64_t cap = k / (W * 32);
        if (S > cap) S = cap;
        if (S > 1) {
            void* scratch = nullptr;
            QSML_TRY_STATUS(get_scratch(ctx, kCounterBytes + static_cast<size_t>(tiles * S) * 32 * PV * sizeof(V),
                                        &scratch));
            unsigned* counters = static_cast<unsigned*>(scratch);
            V* partials = reinterpret_cast<V*>(static_cast<char*>(scratch) + kCounterBytes);
            const int defer = plan_launch(
                ctx, fp.write(span_of(scratch, kCounterBytes + static_cast<size_t>(tiles * S) * 32 * PV * sizeof(V))));
            const cudaError_t e =
                launch_pdl(k_reduce_cols_split<T, OT, OP>, dim3(static_cast<unsigned>(tiles * S)),
                           dim3(32, static_cast<unsigned>(W)), static_cast<size_t>(W) * 32 * PV * sizeof(V),
                           ctx->stream, x, outer, k, inner, tiles_per_o, S, out, scale, counters, partials, defer);
            if (e != cudaSuccess) return check_cuda(ctx, e, "k_reduce_cols_split");
            return after_launch(ctx, "k_reduce_cols_split");
        }
    }
    // about 4096 warps per launch (4 KiB of loads in flight each): measured on
    // B200 best for both axes of X[64,512,1024] in binary32 and binary16
    int64_t W = (4096 + tiles - 1) / tiles;
    if (W > 16) W = 16;
    if (W > k) W = k;
    if (W < 1) W = 1;
    dim3 block(32, static_cast<unsigned>(W));
    size_t smem = static_cast<size_t>(W) * 32 * pv * sizeof(V);
    if (tiles > INT32_MAX) return set_error(ctx, QSML_E_UNSUPPORTED, "reduction too large");
    const int defer = plan_launch(ctx, fp);
    const cudaError_t e =
        vec ? launch_pdl(k_reduce_cols<T, OT, OP, true>, dim3(static_cast<unsigned>(tiles)), block, smem, ctx->stream,
                         x, outer, k, inner, tiles_per_o, out, scale, defer)
            : launch_pdl(k_reduce_cols<T, OT, OP, false>, dim3(static_cast<unsigned>(tiles)), block, smem,
                         ctx->stream, x, outer, k, inner, tiles_per_o, out, scale, defer);
    if (e != cudaSuccess) return check_cuda(ctx, e, "k_reduce_cols");
    return after_launch(ctx, "k_reduce_cols");
}

// ---------------------------------------------------------------------------
// Strided inputs (views: slices with a step, transposes, broadcasts).  The
// view's dims other than the reduced one are collapsed -- neighbours merge
// where their strides chain -- into at most kStrMaxOut output dims, and the
// kernels read the view in place: a reduction of a view is one pass over the
// elements it covers, not a gather copy followed by a reduction.
//   * k_reduce_strided_lanes -- a warp per output, lanes striding over k:
//     when k is the view's more contiguous direction (rows of a slice);
//   * k_reduce_strided_cols  -- a lane per output, warps (and, for few
//     outputs, CTAs) splitting k into contiguous chunks combined in order:
//     when neighbouring outputs are the more contiguous direction (columns
//     of a slice).
// A view that is a transposed or permuted contiguous block does not come
// here: qsml_reduce gives it to the contiguous kernels (dense_view_plan).
// A full reduction of a view first reduces its most contiguous dim into
// binary32 scratch (lanes kernel), then the scratch with the segment kernel.
// ---------------------------------------------------------------------------
constexpr int kStrMaxOut = 4;
constexpr int64_t kStrTargetWarps = 8192;  // warps of a column-block launch

struct StridedPlan {
    int nd;                              // output dims, outermost first
    int64_t oshape[kStrMaxOut], ostride[kStrMaxOut];  // extents, strides in elements
    int64_t k, sk;                       // reduced extent and stride
    int64_t tail_k;                      // k of the last output (a split 1-D view's ragged end)
};

__device__ __forceinline__ int64_t strided_base(const StridedPlan& p, int64_t o) {
    int64_t base = 0;
#pragma unroll
    for (int d = kStrMaxOut - 1; d >= 0; --d) {
        if (d < p.nd) {
            const int64_t e = p.oshape[d];
            const int64_t q = o / e;
            base += (o - q * e) * p.ostride[d];
            o = q;
        }
    }
    return base;
}

template <typename T, typename OT, int OP>
__global__ void __launch_bounds__(256) k_reduce_strided_lanes(const T* __restrict__ x, StridedPlan p, int64_t nout,
                                                              OT* __restrict__ out, float scale, int defer) {
    using R = Red<OP>;
    pdl_start(defer);
    const int lane = threadIdx.x & 31;
    const int64_t nw = static_cast<int64_t>(gridDim.x) * (blockDim.x >> 5);
    for (int64_t o = static_cast<int64_t>(blockIdx.x) * (blockDim.x >> 5) + (threadIdx.x >> 5); o < nout; o += nw) {
        const T* row = x + strided_base(p, o);
        const int64_t kn = o == nout - 1 ? p.tail_k : p.k;
        typename R::V acc = R::ident();
        int64_t kk = lane;
        for (; kk + 7 * 32 < kn; kk += 8 * 32) {  // eight loads in flight, used in k order
            T v[8];
#pragma unroll
            for (int u = 0; u < 8; ++u) v[u] = row[(kk + u * 32) * p.sk];
#pragma unroll
            for (int u = 0; u < 8; ++u) acc = R::comb(acc, R::lift(to_f(v[u])));
        }
        for (; kk < kn; kk += 32) acc = R::comb(acc, R::lift(to_f(row[kk * p.sk])));
        acc = warp_reduce<OP>(acc);
        if (lane == 0) from_f(R::fin(acc, scale), &out[o]);
    }
    pdl_end(defer);
}

// Column-block kernel: block (32, W); lane l owns output 32 g + l of the
// plan's order, the W warps split the CTA's k range into contiguous chunks
// (each ascending, eight loads in flight), combined in warp order.  With S > 1
// the k range is also cut into S contiguous chunks over S CTAs (unit = (chunk,
// group), groups fastest); each stores a binary32 partial per output and the
// CTA taking the group's last ticket combines the S partials in chunk order.
// W and S come from the shape alone.
template <typename T, typename OT, int OP>
__global__ void __launch_bounds__(512) k_reduce_strided_cols(const T* __restrict__ x, StridedPlan p, int64_t nout,
                                                             int64_t S, OT* __restrict__ out, float scale,
                                                             unsigned* __restrict__ counters,
                                                             typename Red<OP>::V* __restrict__ partials, int defer) {
    using R = Red<OP>;
    using V = typename R::V;
    constexpr int U = 8;
    __shared__ V red[16][32];
    __shared__ bool s_last;
    const int lane = threadIdx.x, w = threadIdx.y, W = blockDim.y;
    const int64_t groups = (nout + 31) / 32;
    const int64_t s = blockIdx.x / groups, g = blockIdx.x - s * groups;
    const int64_t o = g * 32 + lane;
    const int64_t kc = (p.k + S - 1) / S;
    const int64_t ks = s * kc, ke = ks + kc < p.k ? ks + kc : p.k;
    const int64_t kper = (kc + W - 1) / W;
    const int64_t k0 = ks + w * kper, k1 = k0 + kper < ke ? k0 + kper : ke;
    pdl_start(defer);
    V acc = R::ident();
    if (o < nout) {
        const T* col = x + strided_base(p, o);
        int64_t kk = k0;
        for (; kk + U <= k1; kk += U) {
            T v[U];
#pragma unroll
            for (int u = 0; u < U; ++u) v[u] = col[(kk + u) * p.sk];
#pragma unroll
            for (int u = 0; u < U; ++u) acc = accum<OP>(acc, v[u]);
        }
        for (; kk < k1; ++kk) acc = accum<OP>(acc, col[kk * p.sk]);
    }
    red[w][lane] = acc;
    __syncthreads();
    if (w == 0) {
        V a = red[0][lane];
        for (int ww = 1; ww < W; ++ww) a = R::comb(a, red[ww][lane]);
        if (S == 1) {
            if (o < nout) from_f(R::fin(a, scale), &out[o]);
        } else {
            partials[(g * S + s) * 32 + lane] = a;
        }
    }
    if (S > 1) {
        __threadfence();
        __syncthreads();
        if (w == 0 && lane == 0) s_last = atomicAdd(&counters[g], 1u) == static_cast<unsigned>(S - 1);
        __syncthreads();
        if (s_last && w == 0) {
            // This CTA completed the group: combine its S partials in chunk order.
            __threadfence();
            V a = __ldcg(&partials[g * S * 32 + lane]);
            for (int64_t j = 1; j < S; ++j) a = R::comb(a, __ldcg(&partials[(g * S + j) * 32 + lane]));
            if (o < nout) from_f(R::fin(a, scale), &out[o]);
            if (lane == 0) counters[g] = 0;  // ready for the next launch on this stream
        }
    }
    pdl_end(defer);
}

// The plan of a reduction of view `a` over dim `ax`: false if its other dims
// do not collapse into kStrMaxOut.
bool strided_plan(const qsml_tdesc* a, int ax, StridedPlan* p) {
    int64_t sh[kMaxDims], st[kMaxDims];
    int n = 0;
    for (int i = 0; i < a->ndim; ++i) {
        if (i == ax || a->shape[i] == 1) continue;
        if (n > 0 && st[n - 1] == a->stride[i] * a->shape[i]) {
            sh[n - 1] *= a->shape[i];
            st[n - 1] = a->stride[i];
            continue;
        }
        sh[n] = a->shape[i];
        st[n] = a->stride[i];
        ++n;
    }
    if (n > kStrMaxOut) return false;
    if (n == 0) {
        sh[0] = 1;
        st[0] = 0;
        n = 1;
    }
    p->nd = n;
    for (int d = 0; d < n; ++d) {
        p->oshape[d] = sh[d];
        p->ostride[d] = st[d];
    }
    p->k = a->shape[ax];
    p->sk = a->stride[ax];
    p->tail_k = p->k;
    return true;
}

inline int64_t iabs64(int64_t v) { return v < 0 ? -v : v; }

template <typename T, typename OT, int OP>
qsml_status_t launch_strided(Context* ctx, const T* x, const StridedPlan& p, int64_t nout, OT* out, float scale,
                             bool lanes) {
    int64_t grid;
    cudaError_t e;
    // the bytes the plan can touch (its lowest to its highest element)
    int64_t lo = 0, hi = 0;
    for (int d = 0; d < p.nd; ++d) {
        const int64_t ext = (p.oshape[d] - 1) * p.ostride[d];
        if (ext < 0) lo += ext; else hi += ext;
    }
    const int64_t ext_k = (p.k - 1) * p.sk;
    if (ext_k < 0) lo += ext_k; else hi += ext_k;
    Footprint fp;
    fp.read(Span{reinterpret_cast<uintptr_t>(x + lo), reinterpret_cast<uintptr_t>(x + hi + 1)})
        .write(span_of(out, static_cast<size_t>(nout) * sizeof(OT)));
    if (lanes) {
        grid = (nout + 7) / 8;
        const int64_t cap = static_cast<int64_t>(ctx->num_sms) * 32;
        if (grid > cap) grid = cap;
        const int defer = plan_launch(ctx, fp);
        e = launch_pdl(k_reduce_strided_lanes<T, OT, OP>, dim3(static_cast<unsigned>(grid)), dim3(256), 0, ctx->stream,
                       x, p, nout, out, scale, defer);
        if (e != cudaSuccess) return check_cuda(ctx, e, "k_reduce_strided_lanes");
        return after_launch(ctx, "k_reduce_strided_lanes");
    }
    // Column blocks: up to 16 warps of at least 16 rows each per CTA, and k cut
    // over more CTAs until about kStrTargetWarps warps read (eight loads in
    // flight each), keeping at least 16 rows per warp.
    using V = typename Red<OP>::V;
    const int64_t groups = (nout + 31) / 32;
    int64_t W = p.k / 16;
    if (W > 16) W = 16;
    if (W < 1) W = 1;
    int64_t S = 1;
    if (groups * W < kStrTargetWarps && groups <= kMaxSegments) {
        S = (kStrTargetWarps + groups * W - 1) / (groups * W);
        const int64_t cap = p.k / (W * 16);
        if (S > cap) S = cap;
        if (S < 1) S = 1;
    }
    if (groups * S > INT32_MAX) return set_error(ctx, QSML_E_UNSUPPORTED, "reduction too large");
    unsigned* counters = nullptr;
    V* partials = nullptr;
    if (S > 1) {
        void* scratch = nullptr;
        QSML_TRY_STATUS(get_scratch(ctx, kCounterBytes + static_cast<size_t>(groups * S) * 32 * sizeof(V), &scratch));
        counters = static_cast<unsigned*>(scratch);
        partials = reinterpret_cast<V*>(static_cast<char*>(scratch) + kCounterBytes);
        fp.write(span_of(scratch, kCounterBytes + static_cast<size_t>(groups * S) * 32 * sizeof(V)));
    }
    const int defer = plan_launch(ctx, fp);
    e = launch_pdl(k_reduce_strided_cols<T, OT, OP>, dim3(static_cast<unsigned>(groups * S)),
                   dim3(32, static_cast<unsigned>(W)), 0, ctx->stream, x, p, nout, S, out, scale, counters, partials,
                   defer);
    if (e != cudaSuccess) return check_cuda(ctx, e, "k_reduce_strided_cols");
    return after_launch(ctx, "k_reduce_strided_cols");
}

// One axis of a view.
template <typename T, typename OT, int OP>
qsml_status_t run_reduce_strided(Context* ctx, const qsml_tdesc* a, int ax, OT* out) {
    StridedPlan p;
    if (!strided_plan(a, ax, &p))
        return set_error(ctx, QSML_E_UNSUPPORTED, "qsml_reduce: view has too many non-mergeable dims");
    int64_t nout = 1;
    for (int d = 0; d < p.nd; ++d) nout *= p.oshape[d];
    // read along k when k is the view's more contiguous direction
    const bool lanes = iabs64(p.sk) <= iabs64(p.ostride[p.nd - 1]);
    return launch_strided<T, OT, OP>(ctx, static_cast<const T*>(a->data), p, nout, out,
                                     1.0f / static_cast<float>(p.k), lanes);
}

// All elements of a view: its most contiguous dim into binary32 scratch, then
// the scratch (mean: divided by the view's element count).
template <typename T, typename OT, int OP>
qsml_status_t run_reduce_strided_all(Context* ctx, const qsml_tdesc* a, OT* out) {
    constexpr int OP1 = OP == QSML_RED_MEAN ? QSML_RED_SUM : OP;
    const int64_t n = numel(a);
    int ax = -1;
    for (int i = 0; i < a->ndim; ++i)
        if (a->shape[i] > 1 && (ax < 0 || iabs64(a->stride[i]) < iabs64(a->stride[ax]))) ax = i;
    StridedPlan p;
    if (ax < 0 || !strided_plan(a, ax, &p))
        return set_error(ctx, QSML_E_UNSUPPORTED, "qsml_reduce: view has too many non-mergeable dims");
    int64_t nout = 1;
    for (int d = 0; d < p.nd; ++d) nout *= p.oshape[d];
    if (nout == 1) {
        // one strided dim: rows of kRowSplit elements (the last one ragged)
        constexpr int64_t kRowSplit = 8192;
        const int64_t k = p.k;
        p.nd = 1;
        p.oshape[0] = (k + kRowSplit - 1) / kRowSplit;
        p.ostride[0] = kRowSplit * p.sk;
        p.k = k < kRowSplit ? k : kRowSplit;
        p.tail_k = k - (p.oshape[0] - 1) * kRowSplit;
        nout = p.oshape[0];
    }
    const float scale = 1.0f / static_cast<float>(n);
    if (nout == 1)
        return launch_strided<T, OT, OP>(ctx, static_cast<const T*>(a->data), p, 1, out, scale, true);
    void* part = nullptr;
    std::string err;
    qsml_status_t st = ctx->allocator->alloc(static_cast<size_t>(nout) * sizeof(float), &part, &err);
    if (st != QSML_OK) return set_error(ctx, st, "qsml_reduce: strided scratch: " + err);
    st = launch_strided<T, float, OP1>(ctx, static_cast<const T*>(a->data), p, nout, static_cast<float*>(part), 1.0f,
                                       true);
    if (st == QSML_OK) st = run_reduce<float, OT, OP>(ctx, static_cast<const float*>(part), 1, nout, 1, out, scale);
    ctx->allocator->free(part, &err);  // reused in stream order
    return st;
}

template <typename T, typename OT>
qsml_status_t reduce_strided_op(Context* ctx, int op, const qsml_tdesc* a, int axis, OT* out) {
    const int ax = axis == QSML_AXIS_ALL ? -1 : (axis < 0 ? axis + a->ndim : axis);
#define QSML_STRIDED(OPC)                                                                  \
    case OPC:                                                                              \
        return ax < 0 ? run_reduce_strided_all<T, OT, OPC>(ctx, a, out)                    \
                      : run_reduce_strided<T, OT, OPC>(ctx, a, ax, out);
    switch (op) {
        QSML_STRIDED(QSML_RED_SUM)
        QSML_STRIDED(QSML_RED_MEAN)
        QSML_STRIDED(QSML_RED_MAX)
        QSML_STRIDED(QSML_RED_MIN)
        QSML_STRIDED(QSML_RED_PROD)
    }
#undef QSML_STRIDED
    return set_error(ctx, QSML_E_INVALID, "qsml_reduce: unknown op");
}

template <typename T, typename OT>
qsml_status_t reduce_op(Context* ctx, int op, const T* x, int64_t outer, int64_t k, int64_t inner, OT* out) {
    switch (op) {
        case QSML_RED_SUM: return run_reduce<T, OT, QSML_RED_SUM>(ctx, x, outer, k, inner, out);
        case QSML_RED_MEAN: return run_reduce<T, OT, QSML_RED_MEAN>(ctx, x, outer, k, inner, out);
        case QSML_RED_MAX: return run_reduce<T, OT, QSML_RED_MAX>(ctx, x, outer, k, inner, out);
        case QSML_RED_MIN: return run_reduce<T, OT, QSML_RED_MIN>(ctx, x, outer, k, inner, out);
        case QSML_RED_PROD: return run_reduce<T, OT, QSML_RED_PROD>(ctx, x, outer, k, inner, out);
    }
    return set_error(ctx, QSML_E_INVALID, "qsml_reduce: unknown op");
}

template <typename T>
__global__ void k_fill_value(T* p, T v, int64_t n) {
    for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < n;
         i += static_cast<int64_t>(gridDim.x) * blockDim.x)
        p[i] = v;
}

}  // namespace
}  // namespace qsml

using namespace qsml;

extern "C" qsml_status_t qsml_reduce(qsml_ctx* handle, int32_t op, const qsml_tdesc* a, int32_t axis,
                                     int32_t keepdims, const qsml_tdesc* out) {
    QSML_CTX(handle);
    QSML_TRY_STATUS(check_desc(C_, a, "a"));
    QSML_TRY_STATUS(check_desc(C_, out, "out"));
    if (op < QSML_RED_SUM || op > QSML_RED_PROD) return set_error(C_, QSML_E_INVALID, "qsml_reduce: unknown op");
    if (a->dtype != QSML_F32 && a->dtype != QSML_F16)
        return set_error(C_, QSML_E_DTYPE, "qsml_reduce: input must be F32 or F16");
    if (out->dtype != a->dtype && out->dtype != QSML_F32)
        return set_error(C_, QSML_E_DTYPE, "qsml_reduce: out dtype must equal the input's or be F32");
    if (!is_contiguous(out)) return set_error(C_, QSML_E_SHAPE, "qsml_reduce: out must be contiguous");

    int64_t outer = 1, k = 1, inner = 1;
    QSML_TRY_STATUS(plan_reduction(C_, a, axis, keepdims, out, "qsml_reduce", &outer, &k, &inner));
    const int64_t nout = outer * inner;
    if (nout == 0) return QSML_OK;
    if (k == 0) {
        if (op == QSML_RED_MAX || op == QSML_RED_MIN)
            return set_error(C_, QSML_E_SHAPE, "qsml_reduce: max/min of an empty axis");
        // sum = 0, prod = 1; mean = 0 * (1/0) = NaN, like the reference's arithmetic.
        float v = op == QSML_RED_PROD ? 1.0f : 0.0f;
        if (op == QSML_RED_MEAN) {
            const uint32_t nan_bits = 0x7fffffffu;
            std::memcpy(&v, &nan_bits, 4);
        }
        int64_t blocks = (nout + 255) / 256;
        if (blocks > 4096) blocks = 4096;
        if (out->dtype == QSML_F32)
            k_fill_value<float><<<static_cast<unsigned>(blocks), 256, 0, C_->stream>>>(static_cast<float*>(out->data), v, nout);
        else
            k_fill_value<__half><<<static_cast<unsigned>(blocks), 256, 0, C_->stream>>>(static_cast<__half*>(out->data),
                                                                                         __float2half_rn(v), nout);
        return after_launch(C_, "k_fill_value");
    }
    // a transposed or permuted contiguous block: the contiguous kernels
    if (!is_contiguous(a) && !dense_view_plan(a, axis, &outer, &k, &inner)) {
        if (a->dtype == QSML_F32) return reduce_strided_op<float, float>(C_, op, a, axis, static_cast<float*>(out->data));
        if (out->dtype == QSML_F16)
            return reduce_strided_op<__half, __half>(C_, op, a, axis, static_cast<__half*>(out->data));
        return reduce_strided_op<__half, float>(C_, op, a, axis, static_cast<float*>(out->data));
    }
    if (a->dtype == QSML_F32)
        return reduce_op<float, float>(C_, op, static_cast<const float*>(a->data), outer, k, inner,
                                       static_cast<float*>(out->data));
    if (out->dtype == QSML_F16)
        return reduce_op<__half, __half>(C_, op, static_cast<const __half*>(a->data), outer, k, inner,
                                         static_cast<__half*>(out->data));
    return reduce_op<__half, float>(C_, op, static_cast<const __half*>(a->data), outer, k, inner,
                                    static_cast<float*>(out->data));
}

// ---------------------------------------------------------------------------
// Allocation-free entry point.
//
// Some callers cannot allocate device memory when they reduce:
// latency-critical serving paths that must not block on the driver's
// allocator (cudaMalloc and cudaFree can synchronise the device), host
// frameworks whose own allocator already owns every byte of HBM, and plugins
// that are handed only a stream and hold no qsml_ctx with its scratch
// buffer.  qsml_reduce_noalloc gives them the
// segment reduction with its scratch (ticket counters + partials) in the
// fixed device array below instead of the context's scratch buffer, and it
// needs no qsml_ctx at all -- only the caller's stream.
//
// The array is a file-scope __device__ object: every GPU that loads this
// library holds its kNoAllocScratchBytes until the process exits.  In host
// code its name is only a stand-in, so its device address is looked up with
// cudaGetSymbolAddress once per device (first call on that device, with the
// device current) and passed to the kernel.  The address is cached per CUDA
// context (its unique id from cuCtxGetId), so a host that resets the device
// (cudaDeviceReset) and gets a new primary context, in which this module is
// loaded afresh at another address, gets a fresh lookup on its next call.
// All calls share the array and it keeps the last call's contents, so the
// counters are cleared before every launch; calls on the same GPU whose work
// overlaps (on different streams, say) race on it.
// ---------------------------------------------------------------------------
namespace qsml {
namespace {

constexpr size_t kNoAllocScratchBytes = size_t(64) << 10;         // 64 KiB per device
constexpr int64_t kNoAllocMaxRows = 64;                           // ticket counters
constexpr size_t kNoAllocCounterBytes = 256;                      // 64 x u32
constexpr int64_t kNoAllocMaxUnits =
    static_cast<int64_t>((kNoAllocScratchBytes - kNoAllocCounterBytes) / 4);  // 4-byte partials
// The slicing rule caps every launch at kSegMaxUnits partials, so any request
// that passes the row limit fits the array.
static_assert(kNoAllocCounterBytes + kSegMaxUnits * 4 <= kNoAllocScratchBytes, "partials fit the array");
static_assert(kNoAllocMaxRows * 4 <= static_cast<int64_t>(kNoAllocCounterBytes), "counters fit their region");

static __device__ __align__(256) unsigned char g_noalloc_scratch[kNoAllocScratchBytes];

std::mutex g_noalloc_mu;
// (device, context id) -> device address of g_noalloc_scratch in that context
std::map<std::pair<int, unsigned long long>, void*> g_noalloc_addr;

// Unique id of the calling thread's current CUDA context (0 when the driver
// cannot say, which then keys the cache by device alone).
unsigned long long current_context_id() {
    using GetCurrent = CUresult (*)(CUcontext*);
    using GetId = CUresult (*)(CUcontext, unsigned long long*);
    static GetCurrent get_current = nullptr;
    static GetId get_id = nullptr;
    static std::once_flag once;
    std::call_once(once, [] {
        void* p = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuCtxGetCurrent", &p, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            get_current = reinterpret_cast<GetCurrent>(p);
        p = nullptr;
        if (cudaGetDriverEntryPoint("cuCtxGetId", &p, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            get_id = reinterpret_cast<GetId>(p);
        cudaGetLastError();
    });
    CUcontext c = nullptr;
    unsigned long long id = 0;
    if (get_current && get_id && get_current(&c) == CUDA_SUCCESS && c && get_id(c, &id) == CUDA_SUCCESS) return id;
    return 0;
}

qsml_status_t noalloc_scratch(void** ptr) {
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) {
        cudaGetLastError();
        return set_error(nullptr, QSML_E_CUDA, std::string("qsml_reduce_noalloc: cudaGetDevice: ") +
                                                   cudaGetErrorString(e));
    }
    std::lock_guard<std::mutex> lk(g_noalloc_mu);
    // With no context current yet (id 0) the lookup below creates the
    // device's primary context; the address is then filed under its id.
    const unsigned long long id = current_context_id();
    auto it = g_noalloc_addr.find(std::make_pair(dev, id));
    if (it != g_noalloc_addr.end()) {
        *ptr = it->second;
        return QSML_OK;
    }
    void* p = nullptr;
    e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
    if (e != cudaSuccess || p == nullptr) {
        cudaGetLastError();
        return set_error(nullptr, QSML_E_CUDA, std::string("qsml_reduce_noalloc: cudaGetSymbolAddress: ") +
                                                   cudaGetErrorString(e));
    }
    g_noalloc_addr[std::make_pair(dev, id != 0 ? id : current_context_id())] = p;
    *ptr = p;
    return QSML_OK;
}

template <typename T, typename OT, int OP>
qsml_status_t run_noalloc(cudaStream_t stream, const T* x, int64_t rows, int64_t k, OT* out, void* scratch) {
    using V = typename Red<OP>::V;
    static_assert(sizeof(V) == 4, "partials are 4 bytes");
    const float scale = 1.0f / static_cast<float>(k);
    const bool vec = aligned16(x) && (rows == 1 || (k * static_cast<int64_t>(sizeof(T))) % 16 == 0);
    // Same slicing rule as the context path, so both give identical bits.
    const int64_t P = seg_slices(rows, k);
    const int64_t units = rows * P;
    if (units > kNoAllocMaxUnits)
        return set_error(nullptr, QSML_E_UNSUPPORTED, "qsml_reduce_noalloc: needs more partials than its fixed scratch holds");
    unsigned* counters = static_cast<unsigned*>(scratch);
    V* partials = reinterpret_cast<V*>(static_cast<char*>(scratch) + kNoAllocCounterBytes);
    cudaError_t e = cudaMemsetAsync(counters, 0, static_cast<size_t>(rows) * sizeof(unsigned), stream);
    if (e != cudaSuccess) {
        cudaGetLastError();
        return set_error(nullptr, QSML_E_CUDA, std::string("qsml_reduce_noalloc: counter clear: ") + cudaGetErrorString(e));
    }
    const int64_t grid = units;  // one slice per CTA
    if (vec)
        k_reduce_seg<T, OT, OP, true><<<static_cast<unsigned>(grid), kRT, 0, stream>>>(x, rows, k, P, out, scale,
                                                                                        counters, partials, 0);
    else
        k_reduce_seg<T, OT, OP, false><<<static_cast<unsigned>(grid), kRT, 0, stream>>>(x, rows, k, P, out, scale,
                                                                                         counters, partials, 0);
    e = cudaGetLastError();
    if (e != cudaSuccess)
        return set_error(nullptr, QSML_E_CUDA, std::string("qsml_reduce_noalloc: launch: ") + cudaGetErrorString(e));
    return QSML_OK;
}

template <typename T, typename OT>
qsml_status_t noalloc_op(cudaStream_t s, int op, const T* x, int64_t rows, int64_t k, OT* out, void* scratch) {
    switch (op) {
        case QSML_RED_SUM: return run_noalloc<T, OT, QSML_RED_SUM>(s, x, rows, k, out, scratch);
        case QSML_RED_MEAN: return run_noalloc<T, OT, QSML_RED_MEAN>(s, x, rows, k, out, scratch);
        case QSML_RED_MAX: return run_noalloc<T, OT, QSML_RED_MAX>(s, x, rows, k, out, scratch);
        case QSML_RED_MIN: return run_noalloc<T, OT, QSML_RED_MIN>(s, x, rows, k, out, scratch);
    }
    return set_error(nullptr, QSML_E_INVALID, "qsml_reduce_noalloc: unknown op");
}

}  // namespace
}  // namespace qsml

extern "C" qsml_status_t qsml_reduce_noalloc(void* stream, int32_t op, const qsml_tdesc* a, int32_t axis,
                                             int32_t keepdims, const qsml_tdesc* out) {
    QSML_TRY_STATUS(check_desc(nullptr, a, "a"));
    QSML_TRY_STATUS(check_desc(nullptr, out, "out"));
    if (op < QSML_RED_SUM || op > QSML_RED_MIN) return set_error(nullptr, QSML_E_INVALID, "qsml_reduce_noalloc: unknown op");
    if (a->dtype != QSML_F32 && a->dtype != QSML_F16)
        return set_error(nullptr, QSML_E_DTYPE, "qsml_reduce_noalloc: input must be F32 or F16");
    if (out->dtype != a->dtype && out->dtype != QSML_F32)
        return set_error(nullptr, QSML_E_DTYPE, "qsml_reduce_noalloc: out dtype must equal the input's or be F32");
    if (!is_contiguous(a) || !is_contiguous(out))
        return set_error(nullptr, QSML_E_UNSUPPORTED, "qsml_reduce_noalloc: a and out must be contiguous");
    // Only reductions whose reduced elements are contiguous: all elements, or
    // an axis with nothing but unit dims after it.
    int64_t rows = 1, k = numel(a);
    if (axis != QSML_AXIS_ALL) {
        const int ax = axis < 0 ? axis + a->ndim : axis;
        if (ax < 0 || ax >= a->ndim) return set_error(nullptr, QSML_E_SHAPE, "qsml_reduce_noalloc: invalid axis");
        for (int i = ax + 1; i < a->ndim; ++i)
            if (a->shape[i] != 1)
                return set_error(nullptr, QSML_E_UNSUPPORTED,
                                 "qsml_reduce_noalloc: only all-element or last-axis reductions are supported");
        k = a->shape[ax];
        rows = k == 0 ? numel(out) : numel(a) / k;
        int64_t expect = 1;
        for (int i = 0; i < a->ndim; ++i)
            if (i != ax) expect *= a->shape[i];
        if (numel(out) != expect) return set_error(nullptr, QSML_E_SHAPE, "qsml_reduce_noalloc: out has the wrong size");
        (void)keepdims;
    } else if (numel(out) != 1) {
        return set_error(nullptr, QSML_E_SHAPE, "qsml_reduce_noalloc: full reduction needs a 1-element out");
    }
    if (k == 0 || rows == 0) return set_error(nullptr, QSML_E_SHAPE, "qsml_reduce_noalloc: empty reduction");
    if (rows > kNoAllocMaxRows)
        return set_error(nullptr, QSML_E_UNSUPPORTED, "qsml_reduce_noalloc: at most 64 rows (its fixed scratch holds 64 counters)");
    void* scratch = nullptr;
    QSML_TRY_STATUS(noalloc_scratch(&scratch));
    cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
    if (a->dtype == QSML_F32)
        return noalloc_op<float, float>(s, op, static_cast<const float*>(a->data), rows, k,
                                        static_cast<float*>(out->data), scratch);
    if (out->dtype == QSML_F16)
        return noalloc_op<__half, __half>(s, op, static_cast<const __half*>(a->data), rows, k,
                                          static_cast<__half*>(out->data), scratch);
    return noalloc_op<__half, float>(s, op, static_cast<const __half*>(a->data), rows, k,
                                     static_cast<float*>(out->data), scratch);
}
