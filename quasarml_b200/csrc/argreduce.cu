// argmax / argmin over one axis or over all elements.
//
// Reference: Ops::argmax / Ops::argmin (Ops/Reduction.cpp:388-396) are stubs
// that ignore the axis and return max / min values.  Here they return
// indices, with NumPy's conventions: first index among equal values, values
// compared numerically (-0 == +0), a NaN beyond every number (first NaN wins).
//
// The input is viewed as [outer, k, inner] like the value reductions and the
// same three shapes of kernel run:
//   * k_arg_seg  -- inner == 1 with few long rows (including the flattened
//                   tensor): slices of a row per CTA, per-slice partials, the
//                   CTA holding the row's last ticket combines them;
//   * k_arg_rows -- inner == 1 with many rows: one warp per row;
//   * k_arg_cols -- inner > 1: lanes own 16-byte column vectors, warps split
//                   k into contiguous ranges.
// All three are launched with programmatic dependent launch (launch_pdl).
// Each thread scans its elements in increasing index order keeping the first
// strictly better one, in the input's own arithmetic (float for F32/F16,
// integers for the integer dtypes; the column kernel compares binary16 two
// halves at a time, see HalfBest).  Threads then combine through a 64-bit
// key, (order-preserving 32-bit image of the value) << 32 | (2^32-1 - index),
// whose maximum is the wanted element whatever the combine order: larger
// value first, then smaller index.  Key 0 stands for "no element".
#include "qsml_internal.cuh"

#include <type_traits>

namespace qsml {
namespace {

constexpr int kAT = 256;                  // threads of the segment kernel
constexpr int64_t kArgSlots = 1184;       // slices per launch (148 SMs x 8 CTAs)
constexpr int64_t kArgMinSlice = 4096;    // elements: short rows use fewer slices
constexpr int kArgMaxSegments = 16384;    // ticket counters at the start of scratch
constexpr size_t kArgCounterBytes = kArgMaxSegments * sizeof(unsigned);
static_assert(kArgCounterBytes == kScratchCounterBytes, "counters fill the reserved scratch region");
constexpr uint32_t kNone = 0xFFFFFFFFu;   // per-thread "no element yet"

template <typename T> struct alignas(16) APack {
    static constexpr int N = 16 / sizeof(T);
    T v[N];
};

// Comparison type per storage type.
template <typename T> struct Cmp { using C = T; };
template <> struct Cmp<__half> { using C = float; };
template <> struct Cmp<int16_t> { using C = int32_t; };
template <> struct Cmp<int8_t> { using C = int32_t; };
template <> struct Cmp<uint16_t> { using C = uint32_t; };
template <> struct Cmp<uint8_t> { using C = uint32_t; };

__device__ __forceinline__ float cval(float v) { return v; }
__device__ __forceinline__ float cval(__half v) { return __half2float(v); }
__device__ __forceinline__ int32_t cval(int32_t v) { return v; }
__device__ __forceinline__ int32_t cval(int16_t v) { return v; }
__device__ __forceinline__ int32_t cval(int8_t v) { return v; }
__device__ __forceinline__ uint32_t cval(uint32_t v) { return v; }
__device__ __forceinline__ uint32_t cval(uint16_t v) { return v; }
__device__ __forceinline__ uint32_t cval(uint8_t v) { return v; }

// v beats the current best (strictly; the earlier index keeps ties).
template <int OP> __device__ __forceinline__ bool better(float v, float best) {
    const bool num = OP == QSML_ARG_MAX ? v > best : v < best;
    return num || (v != v && best == best);
}
template <int OP> __device__ __forceinline__ bool better(int32_t v, int32_t best) {
    return OP == QSML_ARG_MAX ? v > best : v < best;
}
template <int OP> __device__ __forceinline__ bool better(uint32_t v, uint32_t best) {
    return OP == QSML_ARG_MAX ? v > best : v < best;
}

// Order-preserving 32-bit image: larger image = better value.
template <int OP> __device__ __forceinline__ uint32_t image(float v) {
    if (v != v) return 0xFFFFFFFFu;  // above every number for both ops
    if (v == 0.0f) v = 0.0f;         // -0 compares equal to +0
    const uint32_t u = __float_as_uint(v);
    const uint32_t o = (u & 0x80000000u) ? ~u : (u | 0x80000000u);
    return OP == QSML_ARG_MAX ? o : ~o;
}
template <int OP> __device__ __forceinline__ uint32_t image(int32_t v) {
    const uint32_t o = static_cast<uint32_t>(v) ^ 0x80000000u;
    return OP == QSML_ARG_MAX ? o : ~o;
}
template <int OP> __device__ __forceinline__ uint32_t image(uint32_t v) {
    return OP == QSML_ARG_MAX ? v : ~v;
}

template <int OP, typename C>
__device__ __forceinline__ unsigned long long make_key(C best, uint32_t idx) {
    if (idx == kNone) return 0ull;
    return (static_cast<unsigned long long>(image<OP>(best)) << 32) | (0xFFFFFFFFu - idx);
}

__device__ __forceinline__ uint32_t key_index(unsigned long long key) {
    return 0xFFFFFFFFu - static_cast<uint32_t>(key & 0xFFFFFFFFull);
}

__device__ __forceinline__ unsigned long long kmax(unsigned long long a, unsigned long long b) {
    return a > b ? a : b;
}

__device__ __forceinline__ unsigned long long warp_kmax(unsigned long long v) {
#pragma unroll
    for (int m = 16; m >= 1; m >>= 1) v = kmax(v, __shfl_xor_sync(0xffffffffu, v, m));
    return v;
}

// Block of kAT threads; result valid in every thread.
__device__ __forceinline__ unsigned long long block_kmax(unsigned long long v) {
    __shared__ unsigned long long sh[kAT / 32];
    const int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
    v = warp_kmax(v);
    __syncthreads();  // sh may still be read by a previous call
    if (lane == 0) sh[w] = v;
    __syncthreads();
    unsigned long long t = lane < kAT / 32 ? sh[lane] : 0ull;
    return warp_kmax(t);
}

// Running best of one thread.
template <int OP, typename C> struct Best {
    C v;
    uint32_t i = kNone;
    __device__ __forceinline__ void see(C x, uint32_t j) {
        if (i == kNone || better<OP>(x, v)) {
            v = x;
            i = j;
        }
    }
    __device__ __forceinline__ unsigned long long key() const { return make_key<OP>(v, i); }
};

// Running bests of a thread's binary16 packs, two halves per instruction: for
// each of the 8 element positions of a pack, the best value so far (half2
// lanes) and the ordinal of the pack it came from (16 bits per half).  The
// update is branch-free -- one mask of "strictly better" per half2 (the
// numeric compare, or a NaN against a number), then two bitwise selects --
// about three instructions per element against a compare-and-select chain on
// binary32 conversions.  Each position sees its elements in increasing index
// order, so it keeps the first index of its best value.  The starting value is
// the worst number (-inf for argmax) at ordinal 0: a position whose elements
// are all that value reports its first one.  Pack ordinals must stay below
// 65536.  Used by the column kernel, where the 8 positions are 8 columns with
// their own results (binary16 X[64,512,1024] over axis 0 / 1: 3.5 -> 4.2 /
// 4.3 TB/s); in the row and segment kernels a thread would have to merge its
// 8 positions into one key, which at their usual few packs per thread cost
// more than the packed updates saved (measured slower there).
template <int OP> struct HalfBest {
    uint32_t v[4];  // __half2 bits
    uint32_t n[4];  // two 16-bit pack ordinals
    __device__ __forceinline__ void init() {
        const uint32_t worst = OP == QSML_ARG_MAX ? 0xFC00FC00u : 0x7C007C00u;  // -inf / +inf
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            v[j] = worst;
            n[j] = 0u;
        }
    }
    __device__ __forceinline__ void see(const APack<__half>& p, uint32_t ord) {
        const uint32_t o2 = ord | (ord << 16);
        const uint32_t* x = reinterpret_cast<const uint32_t*>(p.v);
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            const __half2 xh = *reinterpret_cast<const __half2*>(&x[j]);
            const __half2 bh = *reinterpret_cast<const __half2*>(&v[j]);
            const uint32_t num = OP == QSML_ARG_MAX ? __hgt2_mask(xh, bh) : __hlt2_mask(xh, bh);
            const uint32_t m = num | (__hneu2_mask(xh, xh) & __heq2_mask(bh, bh));
            v[j] = (x[j] & m) | (v[j] & ~m);
            n[j] = (o2 & m) | (n[j] & ~m);
        }
    }
};

// Column form: pack ordinal = row offset within the thread's k range, and each
// of the 8 positions is its own column.
template <int OP>
__device__ __forceinline__ void half_cols_to_best(const HalfBest<OP>& hb, int64_t k0, Best<OP, float> (&b)[8]) {
#pragma unroll
    for (int j = 0; j < 4; ++j)
#pragma unroll
        for (int h = 0; h < 2; ++h) {
            b[2 * j + h].v = __half2float(__ushort_as_half(static_cast<unsigned short>(hb.v[j] >> (16 * h))));
            b[2 * j + h].i = static_cast<uint32_t>(k0 + ((hb.n[j] >> (16 * h)) & 0xFFFFu));
        }
}

// ---------------------------------------------------------------------------
// Segment kernel: x = [nseg rows, len] contiguous, P slices per row (slice j
// = 256-thread pack blocks j, j+P, j+2P, ...).
// ---------------------------------------------------------------------------
template <typename T, int OP, bool VEC>
__global__ void __launch_bounds__(kAT) k_arg_seg(const T* __restrict__ x, int64_t nseg, int64_t len, int64_t P,
                                                 uint32_t* __restrict__ out, unsigned* __restrict__ counters,
                                                 unsigned long long* __restrict__ partials, int defer) {
    pdl_start(defer);
    using C = typename Cmp<T>::C;
    constexpr int PV = APack<T>::N;
    __shared__ bool s_last;
    const int t = threadIdx.x;
    const int64_t units = nseg * P;
    for (int64_t w = blockIdx.x; w < units; w += gridDim.x) {
        const int64_t s = w / P, j = w - s * P;
        const T* row = x + s * len;
        Best<OP, C> b;
        const int64_t stride = P * kAT;
        if (VEC) {
            const int64_t npk = len / PV;
            const APack<T>* p = reinterpret_cast<const APack<T>*>(row);
            int64_t q = j * kAT + t;
            constexpr int U = 4;
            for (; q + (U - 1) * stride < npk; q += U * stride) {
                APack<T> r[U];
#pragma unroll
                for (int u = 0; u < U; ++u) r[u] = p[q + u * stride];
#pragma unroll
                for (int u = 0; u < U; ++u)
#pragma unroll
                    for (int e = 0; e < PV; ++e)
                        b.see(cval(r[u].v[e]), static_cast<uint32_t>((q + u * stride) * PV + e));
            }
            for (; q < npk; q += stride) {
                APack<T> r = p[q];
#pragma unroll
                for (int e = 0; e < PV; ++e) b.see(cval(r.v[e]), static_cast<uint32_t>(q * PV + e));
            }
            // elements past the last whole pack belong to the last slice
            if (j == P - 1 && t < len - npk * PV)
                b.see(cval(row[npk * PV + t]), static_cast<uint32_t>(npk * PV + t));
        } else {
            for (int64_t q = j * kAT + t; q < len; q += stride) b.see(cval(row[q]), static_cast<uint32_t>(q));
        }
        const unsigned long long key = block_kmax(b.key());
        if (t == 0) {
            partials[w] = key;
            __threadfence();
            const unsigned ticket = atomicAdd(&counters[s], 1u);
            s_last = ticket == static_cast<unsigned>(P - 1);
        }
        __syncthreads();
        if (s_last) {
            __threadfence();
            unsigned long long a = 0ull;
            for (int64_t i = t; i < P; i += kAT) a = kmax(a, __ldcg(&partials[s * P + i]));
            a = block_kmax(a);
            if (t == 0) {
                out[s] = key_index(a);
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
template <typename T, int OP, bool VEC>
__global__ void __launch_bounds__(256) k_arg_rows(const T* __restrict__ x, int64_t rows, int64_t len,
                                                  uint32_t* __restrict__ out, int defer) {
    pdl_start(defer);
    using C = typename Cmp<T>::C;
    constexpr int PV = APack<T>::N;
    const int lane = threadIdx.x & 31;
    const int64_t warps = static_cast<int64_t>(gridDim.x) * (blockDim.x >> 5);
    for (int64_t r = static_cast<int64_t>(blockIdx.x) * (blockDim.x >> 5) + (threadIdx.x >> 5); r < rows;
         r += warps) {
        const T* row = x + r * len;
        Best<OP, C> b;
        if (VEC) {
            const APack<T>* p = reinterpret_cast<const APack<T>*>(row);
            const int64_t np = len / PV;
            constexpr int U = 4;
            int64_t i = lane;
            for (; i + (U - 1) * 32 < np; i += U * 32) {
                APack<T> v[U];
#pragma unroll
                for (int u = 0; u < U; ++u) v[u] = p[i + u * 32];
#pragma unroll
                for (int u = 0; u < U; ++u)
#pragma unroll
                    for (int e = 0; e < PV; ++e) b.see(cval(v[u].v[e]), static_cast<uint32_t>((i + u * 32) * PV + e));
            }
            for (; i < np; i += 32) {
                APack<T> v = p[i];
#pragma unroll
                for (int e = 0; e < PV; ++e) b.see(cval(v.v[e]), static_cast<uint32_t>(i * PV + e));
            }
        } else {
            for (int64_t i = lane; i < len; i += 32) b.see(cval(row[i]), static_cast<uint32_t>(i));
        }
        const unsigned long long key = warp_kmax(b.key());
        if (lane == 0) out[r] = key_index(key);
    }
}

// ---------------------------------------------------------------------------
// Column kernel: out[o, i] = arg_k x[o, k, i]; block (32, W).  Lane owns PV
// consecutive columns, warp w owns k range [w*kper, (w+1)*kper).
// ---------------------------------------------------------------------------
template <typename T, int OP, bool VEC>
__global__ void k_arg_cols(const T* __restrict__ x, int64_t outer, int64_t k, int64_t inner, int64_t tiles_per_o,
                           uint32_t* __restrict__ out, int defer) {
    pdl_start(defer);
    using C = typename Cmp<T>::C;
    constexpr int PV = VEC ? APack<T>::N : 1;
    extern __shared__ unsigned long long red[];
    const int lane = threadIdx.x, w = threadIdx.y, W = blockDim.y;
    const int64_t tile = blockIdx.x;
    const int64_t o = tile / tiles_per_o;
    const int64_t c0 = (tile - o * tiles_per_o) * (32 * PV) + static_cast<int64_t>(lane) * PV;
    const int64_t kper = (k + W - 1) / W;
    const int64_t k0 = w * kper;
    const int64_t k1 = k0 + kper < k ? k0 + kper : k;
    Best<OP, C> b[PV];
    if (o < outer && c0 < inner) {
        const T* base = x + (o * k) * inner + c0;
        // U rows of loads in flight before they are consumed in k order.
        constexpr int U = 8;
        int64_t kk = k0;
        if constexpr (std::is_same<T, __half>::value && VEC) {
            if (k1 > k0 && k1 - k0 <= 65535) {  // row offsets fit 16 bits
                HalfBest<OP> hb;
                hb.init();
                for (; kk + U <= k1; kk += U) {
                    APack<T> v[U];
#pragma unroll
                    for (int u = 0; u < U; ++u) v[u] = *reinterpret_cast<const APack<T>*>(base + (kk + u) * inner);
#pragma unroll
                    for (int u = 0; u < U; ++u) hb.see(v[u], static_cast<uint32_t>(kk + u - k0));
                }
                for (; kk < k1; ++kk)
                    hb.see(*reinterpret_cast<const APack<T>*>(base + kk * inner), static_cast<uint32_t>(kk - k0));
                half_cols_to_best<OP>(hb, k0, b);
            }
        }
        if (VEC) {
            for (; kk + U <= k1; kk += U) {
                APack<T> v[U];
#pragma unroll
                for (int u = 0; u < U; ++u) v[u] = *reinterpret_cast<const APack<T>*>(base + (kk + u) * inner);
#pragma unroll
                for (int u = 0; u < U; ++u)
#pragma unroll
                    for (int e = 0; e < PV; ++e) b[e].see(cval(v[u].v[e]), static_cast<uint32_t>(kk + u));
            }
            for (; kk < k1; ++kk) {
                APack<T> v = *reinterpret_cast<const APack<T>*>(base + kk * inner);
#pragma unroll
                for (int e = 0; e < PV; ++e) b[e].see(cval(v.v[e]), static_cast<uint32_t>(kk));
            }
        } else {
            for (; kk + U <= k1; kk += U) {
                T v[U];
#pragma unroll
                for (int u = 0; u < U; ++u) v[u] = base[(kk + u) * inner];
#pragma unroll
                for (int u = 0; u < U; ++u) b[0].see(cval(v[u]), static_cast<uint32_t>(kk + u));
            }
            for (; kk < k1; ++kk) b[0].see(cval(base[kk * inner]), static_cast<uint32_t>(kk));
        }
    }
#pragma unroll
    for (int e = 0; e < PV; ++e) red[(w * 32 + lane) * PV + e] = b[e].key();
    __syncthreads();
    const int tid = w * 32 + lane;
    for (int col = tid; col < 32 * PV; col += 32 * W) {
        unsigned long long a = red[col];
        for (int ww = 1; ww < W; ++ww) a = kmax(a, red[ww * 32 * PV + col]);
        const int64_t ci = (tile - o * tiles_per_o) * (32 * PV) + col;
        if (o < outer && ci < inner) out[o * inner + ci] = key_index(a);
    }
    pdl_end(defer);
}

// ---------------------------------------------------------------------------
// Host dispatch
// ---------------------------------------------------------------------------
template <typename T, int OP>
qsml_status_t run_arg(Context* ctx, const T* x, int64_t outer, int64_t k, int64_t inner, uint32_t* out) {
    constexpr int PV = APack<T>::N;
    const bool x_al = aligned16(x);
    // what the launch reads and writes, for overlap with the kernels before it
    Footprint fp;
    fp.read(span_of(x, static_cast<size_t>(outer * k * inner) * sizeof(T)))
        .write(span_of(out, static_cast<size_t>(outer * inner) * sizeof(uint32_t)));
    if (inner == 1 && (outer == 1 || (outer < 592 && k >= 8192))) {
        if (outer > kArgMaxSegments) return set_error(ctx, QSML_E_UNSUPPORTED, "qsml_arg_reduce: too many segments");
        const bool vec = x_al && (outer == 1 || (k * static_cast<int64_t>(sizeof(T))) % 16 == 0);
        int64_t P = kArgSlots / outer;
        const int64_t by_size = (k + kArgMinSlice - 1) / kArgMinSlice;
        if (P > by_size) P = by_size;
        if (P < 1) P = 1;
        const int64_t units = outer * P;
        void* scratch = nullptr;
        QSML_TRY_STATUS(get_scratch(ctx, kArgCounterBytes + static_cast<size_t>(units) * 8, &scratch));
        unsigned* counters = static_cast<unsigned*>(scratch);
        auto* partials = reinterpret_cast<unsigned long long*>(static_cast<char*>(scratch) + kArgCounterBytes);
        int64_t grid = static_cast<int64_t>(ctx->num_sms) * 8;
        if (grid > units) grid = units;
        const int defer = plan_launch(ctx, fp.write(span_of(scratch, kArgCounterBytes + static_cast<size_t>(units) * 8)));
        const cudaError_t e =
            vec ? launch_pdl(k_arg_seg<T, OP, true>, dim3(static_cast<unsigned>(grid)), dim3(kAT), 0, ctx->stream, x,
                             outer, k, P, out, counters, partials, defer)
                : launch_pdl(k_arg_seg<T, OP, false>, dim3(static_cast<unsigned>(grid)), dim3(kAT), 0, ctx->stream, x,
                             outer, k, P, out, counters, partials, defer);
        if (e != cudaSuccess) return check_cuda(ctx, e, "k_arg_seg");
        return after_launch(ctx, "k_arg_seg");
    }
    if (inner == 1) {
        const bool vec = x_al && (k * static_cast<int64_t>(sizeof(T))) % 16 == 0;
        int64_t grid = (outer + 7) / 8;  // 8 warps per CTA
        const int64_t cap = static_cast<int64_t>(ctx->num_sms) * 32;
        if (grid > cap) grid = cap;
        const int defer = plan_launch(ctx, fp);
        const cudaError_t e =
            vec ? launch_pdl(k_arg_rows<T, OP, true>, dim3(static_cast<unsigned>(grid)), dim3(256), 0, ctx->stream, x,
                             outer, k, out, defer)
                : launch_pdl(k_arg_rows<T, OP, false>, dim3(static_cast<unsigned>(grid)), dim3(256), 0, ctx->stream, x,
                             outer, k, out, defer);
        if (e != cudaSuccess) return check_cuda(ctx, e, "k_arg_rows");
        return after_launch(ctx, "k_arg_rows");
    }
    const bool vec = x_al && (inner * static_cast<int64_t>(sizeof(T))) % 16 == 0;
    const int pv = vec ? PV : 1;
    const int64_t tiles_per_o = (inner + 32 * pv - 1) / (32 * pv);
    const int64_t tiles = tiles_per_o * outer;
    if (tiles > INT32_MAX) return set_error(ctx, QSML_E_UNSUPPORTED, "qsml_arg_reduce: too large");
    // about 4096 warps per launch for 4-byte elements and binary16 (compared
    // two halves at a time), more for the narrower integers (more
    // comparisons per 16-byte load); keys in at most 32 KiB of shared memory
    const int64_t target = std::is_same<T, __half>::value
                               ? 4096
                               : 4096 * (4 / static_cast<int64_t>(sizeof(T) < 4 ? sizeof(T) : 4));
    int64_t W = (target + tiles - 1) / tiles;
    const int64_t w_smem = 32768 / (32 * pv * 8);
    if (W > 16) W = 16;
    if (W > w_smem) W = w_smem;
    if (W > k) W = k;
    if (W < 1) W = 1;
    dim3 block(32, static_cast<unsigned>(W));
    const size_t smem = static_cast<size_t>(W) * 32 * pv * 8;
    const int defer = plan_launch(ctx, fp);
    const cudaError_t e =
        vec ? launch_pdl(k_arg_cols<T, OP, true>, dim3(static_cast<unsigned>(tiles)), block, smem, ctx->stream, x,
                         outer, k, inner, tiles_per_o, out, defer)
            : launch_pdl(k_arg_cols<T, OP, false>, dim3(static_cast<unsigned>(tiles)), block, smem, ctx->stream, x,
                         outer, k, inner, tiles_per_o, out, defer);
    if (e != cudaSuccess) return check_cuda(ctx, e, "k_arg_cols");
    return after_launch(ctx, "k_arg_cols");
}

template <typename T>
qsml_status_t arg_op(Context* ctx, int op, const void* x, int64_t outer, int64_t k, int64_t inner, void* out) {
    const T* xt = static_cast<const T*>(x);
    uint32_t* o = static_cast<uint32_t*>(out);
    if (op == QSML_ARG_MAX) return run_arg<T, QSML_ARG_MAX>(ctx, xt, outer, k, inner, o);
    return run_arg<T, QSML_ARG_MIN>(ctx, xt, outer, k, inner, o);
}

}  // namespace
}  // namespace qsml

using namespace qsml;

extern "C" qsml_status_t qsml_arg_reduce(qsml_ctx* handle, int32_t op, const qsml_tdesc* a, int32_t axis,
                                         int32_t keepdims, const qsml_tdesc* out) {
    QSML_CTX(handle);
    QSML_TRY_STATUS(check_desc(C_, a, "a"));
    QSML_TRY_STATUS(check_desc(C_, out, "out"));
    if (op != QSML_ARG_MAX && op != QSML_ARG_MIN) return set_error(C_, QSML_E_INVALID, "qsml_arg_reduce: unknown op");
    if (out->dtype != QSML_I32 && out->dtype != QSML_U32)
        return set_error(C_, QSML_E_DTYPE, "qsml_arg_reduce: out must be I32 or U32");
    if (!is_contiguous(out)) return set_error(C_, QSML_E_SHAPE, "qsml_arg_reduce: out must be contiguous");
    int64_t outer = 1, k = 1, inner = 1;
    QSML_TRY_STATUS(plan_reduction(C_, a, axis, keepdims, out, "qsml_arg_reduce", &outer, &k, &inner));
    // A transposed or permuted contiguous block reduced over one axis is the
    // contiguous arg-reduction of that block (the index along the axis is the
    // same); a full arg-reduction's flat index follows the view's order, so
    // it needs a contiguous input.
    if (!is_contiguous(a) &&
        (axis == QSML_AXIS_ALL || !dense_view_plan(a, axis, &outer, &k, &inner)))
        return set_error(C_, QSML_E_UNSUPPORTED,
                         "qsml_arg_reduce: input must be contiguous or a permuted contiguous block reduced over one "
                         "axis (materialise other views with qsml_gather)");
    if (outer * inner == 0) return QSML_OK;
    if (k == 0) return set_error(C_, QSML_E_SHAPE, "qsml_arg_reduce: arg-reduction of an empty axis");
    const int64_t kmax_len = out->dtype == QSML_I32 ? int64_t(INT32_MAX) : int64_t(0xFFFFFFFEu);
    if (k > kmax_len)
        return set_error(C_, QSML_E_UNSUPPORTED, "qsml_arg_reduce: reduced axis too long for the index dtype");
    switch (a->dtype) {
        case QSML_F32: return arg_op<float>(C_, op, a->data, outer, k, inner, out->data);
        case QSML_F16: return arg_op<__half>(C_, op, a->data, outer, k, inner, out->data);
        case QSML_I32: return arg_op<int32_t>(C_, op, a->data, outer, k, inner, out->data);
        case QSML_I16: return arg_op<int16_t>(C_, op, a->data, outer, k, inner, out->data);
        case QSML_I8: return arg_op<int8_t>(C_, op, a->data, outer, k, inner, out->data);
        case QSML_U32: return arg_op<uint32_t>(C_, op, a->data, outer, k, inner, out->data);
        case QSML_U16: return arg_op<uint16_t>(C_, op, a->data, outer, k, inner, out->data);
        case QSML_U8: return arg_op<uint8_t>(C_, op, a->data, outer, k, inner, out->data);
    }
    return set_error(C_, QSML_E_DTYPE, "qsml_arg_reduce: unknown dtype");
}
