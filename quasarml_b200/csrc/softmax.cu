// Softmax over one axis: y = exp(x - max) / sum(exp(x - max)).
//
// Reference: Ops::softmax (Ops/Elementwise.cpp:395-417) runs one workgroup
// per row with the shader of Elementwise.cpp:98-135: a shared-memory tree for
// the row max, another for the sum of exp(x - max), then
// out = exp(x - max) / sum.  Its indexing (offset = row * axis_size) is right
// for the last axis only.  Here the same arithmetic (max, subtract, expf,
// binary32 sum; the division as a correctly rounded reciprocal per slice and
// one multiply per element, within 1.5 ulp of the quotient -- GLSL's `/` is
// not correctly rounded either) runs over any axis:
//   * k_softmax_rows -- last axis, row held in registers (16-byte loads):
//     persistent CTAs with the next two rows in flight, so x is read once and y
//     written once;
//   * k_softmax_rows_generic -- last axis, any width: one CTA per row, three
//     passes over global memory (max, sum, write);
//   * k_softmax_long_{max,sum,out} -- last axis, fewer rows than SMs and long
//     rows: slices of each row over many CTAs, three launches;
//   * k_softmax_cols -- inner dims after the axis: one thread per column of
//     the [outer, k, inner] view, three passes over k.
// The max is IEEE 754-2019 maximum (a NaN in the row makes the row NaN), and
// every combine order is fixed by the shape, so results are deterministic.
#include "qsml_internal.cuh"

namespace qsml {
namespace {

template <typename T> struct alignas(16) Pack {
    static constexpr int N = 16 / sizeof(T);
    T v[N];
};

__device__ __forceinline__ float to_f(float v) { return v; }
__device__ __forceinline__ float to_f(__half v) { return __half2float(v); }
__device__ __forceinline__ void from_f(float v, float* o) { *o = v; }
__device__ __forceinline__ void from_f(float v, __half* o) { *o = __float2half_rn(v); }

__device__ __forceinline__ float max_nan(float a, float b) {
    float r;
    asm("max.NaN.f32 %0, %1, %2;" : "=f"(r) : "f"(a), "f"(b));
    return r;
}

// Block-wide max or sum: xor butterflies inside warps (both partners hold
// identical bits), one slot per warp in `sh`, one barrier, then every thread
// combines the slots in warp order (the same bits everywhere).  Callers use a
// separate `sh` for the max and for the sum of a row: the max slots of row
// r+1 are written only after every thread passed row r's sum barrier (so
// after it read row r's max), and the sum slots of row r+1 only after row
// r+1's max barrier (so after every thread read row r's sum).
template <bool MAX>
__device__ __forceinline__ float block_combine(float v, float* sh) {
    const int lane = threadIdx.x & 31, w = threadIdx.x >> 5, nw = blockDim.x >> 5;
#pragma unroll
    for (int m = 16; m >= 1; m >>= 1) {
        const float o = __shfl_xor_sync(0xffffffffu, v, m);
        v = MAX ? max_nan(v, o) : __fadd_rn(v, o);
    }
    if (lane == 0) sh[w] = v;
    __syncthreads();
    float a = sh[0];
    for (int j = 1; j < nw; ++j) a = MAX ? max_nan(a, sh[j]) : __fadd_rn(a, sh[j]);
    return a;
}

template <typename T, int NV>
__global__ void __launch_bounds__(256) k_softmax_rows(const T* __restrict__ x, T* __restrict__ y, int64_t rows,
                                                      int cols) {
    constexpr int PV = Pack<T>::N;
    constexpr int E = NV * PV;
    __shared__ float sh_max[8], sh_sum[8];
    const int t = threadIdx.x, th = blockDim.x;
    // Two rows in flight beyond the one being reduced (cur <- nxt <- nxt2).
    Pack<T> cur[NV], nxt[NV], nxt2[NV];
    int64_t row = blockIdx.x;
    if (row < rows) {
        const Pack<T>* xr = reinterpret_cast<const Pack<T>*>(x + row * cols);
#pragma unroll
        for (int i = 0; i < NV; ++i) cur[i] = xr[t + i * th];
    }
    if (row + gridDim.x < rows) {
        const Pack<T>* xr = reinterpret_cast<const Pack<T>*>(x + (row + gridDim.x) * cols);
#pragma unroll
        for (int i = 0; i < NV; ++i) nxt[i] = xr[t + i * th];
    }
    for (; row < rows; row += gridDim.x) {
        const int64_t nrow = row + 2 * static_cast<int64_t>(gridDim.x);
        if (nrow < rows) {
            const Pack<T>* xn = reinterpret_cast<const Pack<T>*>(x + nrow * cols);
#pragma unroll
            for (int i = 0; i < NV; ++i) nxt2[i] = xn[t + i * th];
        }
        float v[E];
#pragma unroll
        for (int i = 0; i < NV; ++i)
#pragma unroll
            for (int e = 0; e < PV; ++e) v[i * PV + e] = to_f(cur[i].v[e]);
        float m = -INFINITY;
#pragma unroll
        for (int k = 0; k < E; ++k) m = max_nan(m, v[k]);
        m = block_combine<true>(m, sh_max);
        float s = 0.0f;
#pragma unroll
        for (int k = 0; k < E; ++k) {
            v[k] = expf(__fsub_rn(v[k], m));
            s = __fadd_rn(s, v[k]);
        }
        s = block_combine<false>(s, sh_sum);
        const float inv = __frcp_rn(s);
        Pack<T>* yr = reinterpret_cast<Pack<T>*>(y + row * cols);
#pragma unroll
        for (int i = 0; i < NV; ++i) {
            Pack<T> o;
#pragma unroll
            for (int e = 0; e < PV; ++e) from_f(__fmul_rn(v[i * PV + e], inv), &o.v[e]);
            yr[t + i * th] = o;
        }
#pragma unroll
        for (int i = 0; i < NV; ++i) {
            cur[i] = nxt[i];
            nxt[i] = nxt2[i];
        }
    }
}

template <typename T>
__global__ void __launch_bounds__(256) k_softmax_rows_generic(const T* __restrict__ x, T* __restrict__ y,
                                                              int64_t rows, int64_t cols) {
    __shared__ float sh_max[8], sh_sum[8];
    for (int64_t row = blockIdx.x; row < rows; row += gridDim.x) {
        const T* xr = x + row * cols;
        float m = -INFINITY;
        for (int64_t c = threadIdx.x; c < cols; c += blockDim.x) m = max_nan(m, to_f(xr[c]));
        m = block_combine<true>(m, sh_max);
        float s = 0.0f;
        for (int64_t c = threadIdx.x; c < cols; c += blockDim.x) s = __fadd_rn(s, expf(__fsub_rn(to_f(xr[c]), m)));
        s = block_combine<false>(s, sh_sum);
        const float inv = __frcp_rn(s);
        T* yr = y + row * cols;
        for (int64_t c = threadIdx.x; c < cols; c += blockDim.x)
            from_f(__fmul_rn(expf(__fsub_rn(to_f(xr[c]), m)), inv), &yr[c]);
    }
}

// One thread per (outer, inner) column; consecutive threads take consecutive
// inner indices, so every pass over k is coalesced.
template <typename T>
__global__ void __launch_bounds__(256) k_softmax_cols(const T* __restrict__ x, T* __restrict__ y, int64_t outer,
                                                      int64_t k, int64_t inner) {
    const int64_t ncol = outer * inner;
    for (int64_t c = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; c < ncol;
         c += static_cast<int64_t>(gridDim.x) * blockDim.x) {
        const int64_t o = c / inner, i = c - o * inner;
        const T* xc = x + o * k * inner + i;
        T* yc = y + o * k * inner + i;
        float m = -INFINITY;
        for (int64_t j = 0; j < k; ++j) m = max_nan(m, to_f(xc[j * inner]));
        float s = 0.0f;
        for (int64_t j = 0; j < k; ++j) s = __fadd_rn(s, expf(__fsub_rn(to_f(xc[j * inner]), m)));
        const float inv = __frcp_rn(s);
        for (int64_t j = 0; j < k; ++j) from_f(__fmul_rn(expf(__fsub_rn(to_f(xc[j * inner]), m)), inv), &yc[j * inner]);
    }
}

// ---------------------------------------------------------------------------
// Long rows (few rows, many elements): each row is cut into P slices, one CTA
// per (row, slice), in three launches -- slice maxima; slice sums of
// exp(x - m) with every CTA combining the row's maxima itself in slice order;
// then y = exp(x - m) * (1 / s) with m and s recombined the same way.  The
// combine orders depend on the shape only, so results are deterministic.
// ---------------------------------------------------------------------------
constexpr int kLongThreads = 256;

template <typename T>
__device__ __forceinline__ void slice_bounds(int64_t cols, int64_t P, int64_t j, int64_t* c0, int64_t* c1) {
    const int64_t per = (cols + P - 1) / P;
    *c0 = j * per;
    *c1 = *c0 + per < cols ? *c0 + per : cols;
}

template <typename T>
__global__ void __launch_bounds__(kLongThreads) k_softmax_long_max(const T* __restrict__ x, int64_t rows,
                                                                   int64_t cols, int64_t P, float* __restrict__ pmax) {
    __shared__ float sh[8];
    const int64_t unit = blockIdx.x, r = unit / P, j = unit - r * P;
    int64_t c0, c1;
    slice_bounds<T>(cols, P, j, &c0, &c1);
    const T* xr = x + r * cols;
    float m = -INFINITY;
    for (int64_t c = c0 + threadIdx.x; c < c1; c += kLongThreads) m = max_nan(m, to_f(xr[c]));
    m = block_combine<true>(m, sh);
    if (threadIdx.x == 0) pmax[unit] = m;
}

__device__ __forceinline__ float row_max(const float* pmax, int64_t r, int64_t P) {
    float m = -INFINITY;
    for (int64_t i = 0; i < P; ++i) m = max_nan(m, pmax[r * P + i]);
    return m;
}

template <typename T>
__global__ void __launch_bounds__(kLongThreads) k_softmax_long_sum(const T* __restrict__ x, int64_t rows,
                                                                   int64_t cols, int64_t P,
                                                                   const float* __restrict__ pmax,
                                                                   float* __restrict__ psum) {
    __shared__ float sh[8];
    const int64_t unit = blockIdx.x, r = unit / P, j = unit - r * P;
    int64_t c0, c1;
    slice_bounds<T>(cols, P, j, &c0, &c1);
    const float m = row_max(pmax, r, P);
    const T* xr = x + r * cols;
    float s = 0.0f;
    for (int64_t c = c0 + threadIdx.x; c < c1; c += kLongThreads) s = __fadd_rn(s, expf(__fsub_rn(to_f(xr[c]), m)));
    s = block_combine<false>(s, sh);
    if (threadIdx.x == 0) psum[unit] = s;
}

template <typename T>
__global__ void __launch_bounds__(kLongThreads) k_softmax_long_out(const T* __restrict__ x, T* __restrict__ y,
                                                                   int64_t rows, int64_t cols, int64_t P,
                                                                   const float* __restrict__ pmax,
                                                                   const float* __restrict__ psum) {
    const int64_t unit = blockIdx.x, r = unit / P, j = unit - r * P;
    int64_t c0, c1;
    slice_bounds<T>(cols, P, j, &c0, &c1);
    const float m = row_max(pmax, r, P);
    float s = 0.0f;
    for (int64_t i = 0; i < P; ++i) s = __fadd_rn(s, psum[r * P + i]);
    const float inv = __frcp_rn(s);
    const T* xr = x + r * cols;
    T* yr = y + r * cols;
    for (int64_t c = c0 + threadIdx.x; c < c1; c += kLongThreads)
        from_f(__fmul_rn(expf(__fsub_rn(to_f(xr[c]), m)), inv), &yr[c]);
}

template <typename T>
qsml_status_t run_long_rows(Context* ctx, const T* x, T* y, int64_t rows, int64_t cols) {
    // about 8 CTAs per SM over all rows, slices of at least 8192 elements
    int64_t P = (int64_t(ctx->num_sms) * 8 + rows - 1) / rows;
    const int64_t by_size = (cols + 8191) / 8192;
    if (P > by_size) P = by_size;
    if (P < 1) P = 1;
    const int64_t units = rows * P;
    if (units > INT32_MAX) return set_error(ctx, QSML_E_UNSUPPORTED, "qsml_softmax: too many slices");
    void* scratch = nullptr;
    QSML_TRY_STATUS(get_scratch(ctx, kScratchCounterBytes + static_cast<size_t>(units) * 2 * sizeof(float), &scratch));
    float* pmax = reinterpret_cast<float*>(static_cast<char*>(scratch) + kScratchCounterBytes);
    float* psum = pmax + units;
    const unsigned g = static_cast<unsigned>(units);
    k_softmax_long_max<T><<<g, kLongThreads, 0, ctx->stream>>>(x, rows, cols, P, pmax);
    QSML_TRY_STATUS(after_launch(ctx, "k_softmax_long_max"));
    k_softmax_long_sum<T><<<g, kLongThreads, 0, ctx->stream>>>(x, rows, cols, P, pmax, psum);
    QSML_TRY_STATUS(after_launch(ctx, "k_softmax_long_sum"));
    k_softmax_long_out<T><<<g, kLongThreads, 0, ctx->stream>>>(x, y, rows, cols, P, pmax, psum);
    return after_launch(ctx, "k_softmax_long_out");
}

template <typename T, int NV>
qsml_status_t launch_rows(Context* ctx, const T* x, T* y, int64_t rows, int cols, unsigned th) {
    static std::mutex mu;
    static std::map<unsigned, int> per_sm_cache;
    int per_sm = 0;
    {
        std::lock_guard<std::mutex> lk(mu);
        auto it = per_sm_cache.find(th);
        if (it == per_sm_cache.end()) {
            cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, k_softmax_rows<T, NV>, static_cast<int>(th), 0);
            if (per_sm < 1) per_sm = 1;
            per_sm_cache[th] = per_sm;
        } else {
            per_sm = it->second;
        }
    }
    int64_t grid = static_cast<int64_t>(ctx->num_sms) * per_sm;
    if (grid > rows) grid = rows;
    k_softmax_rows<T, NV><<<static_cast<unsigned>(grid), th, 0, ctx->stream>>>(x, y, rows, cols);
    return after_launch(ctx, "k_softmax_rows");
}

template <typename T>
qsml_status_t run_softmax(Context* ctx, const T* x, T* y, int64_t outer, int64_t k, int64_t inner) {
    constexpr int PV = Pack<T>::N;
    if (inner == 1) {
        const int64_t rows = outer, cols = k;
        if (cols % PV == 0 && aligned16(x) && aligned16(y) && cols <= INT32_MAX) {
            const int64_t packs = cols / PV;
            int nv = 0;
            for (int cand : {1, 2, 4, 8}) {
                if (packs % cand) continue;
                const int64_t th = packs / cand;
                if (th % 32 == 0 && th <= 256) {
                    nv = cand;
                    break;
                }
            }
            if (nv) {
                const unsigned th = static_cast<unsigned>(packs / nv);
                const int c = static_cast<int>(cols);
                switch (nv) {
                    case 1: return launch_rows<T, 1>(ctx, x, y, rows, c, th);
                    case 2: return launch_rows<T, 2>(ctx, x, y, rows, c, th);
                    case 4: return launch_rows<T, 4>(ctx, x, y, rows, c, th);
                    default: return launch_rows<T, 8>(ctx, x, y, rows, c, th);
                }
            }
        }
        // Few long rows: a CTA per row would leave most SMs idle.
        if (rows < ctx->num_sms && cols >= 16384) return run_long_rows<T>(ctx, x, y, rows, cols);
        int64_t grid = rows < int64_t(ctx->num_sms) * 16 ? rows : int64_t(ctx->num_sms) * 16;
        const unsigned th = cols >= 256 ? 256 : (cols >= 128 ? 128 : (cols >= 64 ? 64 : 32));
        k_softmax_rows_generic<T><<<static_cast<unsigned>(grid), th, 0, ctx->stream>>>(x, y, rows, cols);
        return after_launch(ctx, "k_softmax_rows_generic");
    }
    const int64_t ncol = outer * inner;
    int64_t blocks = (ncol + 255) / 256;
    if (blocks > int64_t(ctx->num_sms) * 32) blocks = int64_t(ctx->num_sms) * 32;
    k_softmax_cols<T><<<static_cast<unsigned>(blocks), 256, 0, ctx->stream>>>(x, y, outer, k, inner);
    return after_launch(ctx, "k_softmax_cols");
}

}  // namespace
}  // namespace qsml

using namespace qsml;

extern "C" qsml_status_t qsml_softmax(qsml_ctx* handle, const qsml_tdesc* x, int32_t axis, const qsml_tdesc* y) {
    QSML_CTX(handle);
    QSML_TRY_STATUS(check_desc(C_, x, "x"));
    QSML_TRY_STATUS(check_desc(C_, y, "y"));
    if (x->dtype != QSML_F32 && x->dtype != QSML_F16)
        return set_error(C_, QSML_E_DTYPE, "qsml_softmax: x must be F32 or F16");
    if (y->dtype != x->dtype) return set_error(C_, QSML_E_DTYPE, "qsml_softmax: y dtype must equal x dtype");
    if (y->ndim != x->ndim) return set_error(C_, QSML_E_SHAPE, "qsml_softmax: y shape must equal x shape");
    for (int d = 0; d < x->ndim; ++d)
        if (y->shape[d] != x->shape[d]) return set_error(C_, QSML_E_SHAPE, "qsml_softmax: y shape must equal x shape");
    if (!is_contiguous(x) || !is_contiguous(y))
        return set_error(C_, QSML_E_UNSUPPORTED, "qsml_softmax: x and y must be contiguous (materialise x with qsml_gather)");
    const int ax = axis < 0 ? axis + x->ndim : axis;
    if (x->ndim < 1 || ax < 0 || ax >= x->ndim) return set_error(C_, QSML_E_SHAPE, "qsml_softmax: invalid axis");
    int64_t outer = 1, k = x->shape[ax], inner = 1;
    for (int d = 0; d < ax; ++d) outer *= x->shape[d];
    for (int d = ax + 1; d < x->ndim; ++d) inner *= x->shape[d];
    if (outer * k * inner == 0) return QSML_OK;
    if (x->dtype == QSML_F32)
        return run_softmax<float>(C_, static_cast<const float*>(x->data), static_cast<float*>(y->data), outer, k, inner);
    return run_softmax<__half>(C_, static_cast<const __half*>(x->data), static_cast<__half*>(y->data), outer, k, inner);
}
