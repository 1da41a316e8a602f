// Layer norm over the last dim: y = (x - mean) / sqrt(var + eps) * gamma + beta
// with the biased (population) variance.  The reference snapshot has no
// layer norm; this is a new op of the same API family.
//
// k_layer_norm_reg: persistent CTAs, one row at a time held in registers
// (16-byte loads) with the next two rows already in flight, so x is read from HBM
// exactly once and y written once; gamma/beta stay in shared memory.  Each
// thread's values give a local (mean, M2); warps merge them with Chan's
// pairwise update (equal counts, written symmetrically so partner lanes hold
// identical bits), then the warps' results merge the same way.
// k_layer_norm_generic: any width or alignment, Welford over global memory
// (reads x twice).
#include "qsml_internal.cuh"

namespace qsml {
namespace {

template <typename T> struct alignas(16) Pack {
    static constexpr int N = 16 / sizeof(T);
    T v[N];
};

__device__ __forceinline__ float to_f(float v) { return v; }
__device__ __forceinline__ float to_f(__half v) { return __half2float(v); }
__device__ __forceinline__ float from_f_tag(float v, float*) { return v; }
__device__ __forceinline__ __half from_f_tag(float v, __half*) { return __float2half_rn(v); }

// Merge (mean, m2) statistics of two equal-count halves of n elements each.
__device__ __forceinline__ void chan_equal(float& mean, float& m2, float mo, float m2o, float n) {
    float d = __fsub_rn(mo, mean);
    float dd = __fmul_rn(d, d);  // (a-b)^2 == (b-a)^2 bit for bit
    mean = __fmul_rn(__fadd_rn(mean, mo), 0.5f);
    m2 = __fadd_rn(__fadd_rn(m2, m2o), __fmul_rn(dd, __fmul_rn(n, 0.5f)));
}

// PV consecutive gamma/beta values as binary32, with 16-byte loads.
template <typename GT, int PV>
__device__ __forceinline__ void load_params(const GT* p, float* out) {
    if constexpr (sizeof(GT) == 4) {
#pragma unroll
        for (int i = 0; i < PV; i += 4) {
            float4 v = *reinterpret_cast<const float4*>(p + i);
            out[i] = v.x; out[i + 1] = v.y; out[i + 2] = v.z; out[i + 3] = v.w;
        }
    } else {
#pragma unroll
        for (int i = 0; i < PV; i += 8) {
            Pack<__half> v = *reinterpret_cast<const Pack<__half>*>(p + i);
#pragma unroll
            for (int e = 0; e < 8; ++e) out[i + e] = __half2float(v.v[e]);
        }
    }
}

// Persistent CTAs; the next two rows' x are loaded before the current row is
// reduced, so each CTA always has a row in flight.  gamma/beta (as binary32)
// sit in dynamic shared memory, each thread holding exactly the columns it
// reads, so they need no barrier and no registers.  Per-warp statistics go to
// slots double-buffered by row parity; after one barrier every warp merges
// all slots itself (identical bits in every warp), so a row costs one
// barrier: row r+2 rewrites row r's slots only after every thread has passed
// row r+1's barrier, i.e. after it read row r's slots.
template <typename T, typename GT, int NV>
__global__ void __launch_bounds__(256) k_layer_norm_reg(const T* __restrict__ x, const GT* __restrict__ gamma,
                                                        const GT* __restrict__ beta, T* __restrict__ y,
                                                        int64_t rows, int cols, float eps) {
    constexpr int PV = Pack<T>::N;
    constexpr int E = NV * PV;  // elements per thread
    extern __shared__ float4 ln_smem[];
    float* sg = reinterpret_cast<float*>(ln_smem);
    float* sb = sg + cols;
    __shared__ float s_mean[2][8], s_m2[2][8];
    const int t = threadIdx.x, lane = t & 31, w = t >> 5, nw = blockDim.x >> 5;
    const int th = blockDim.x;
    const bool pow2 = (nw & (nw - 1)) == 0;
#pragma unroll
    for (int i = 0; i < NV; ++i) {
        const int c0 = (t + i * th) * PV;
        load_params<GT, PV>(gamma + c0, sg + c0);
        load_params<GT, PV>(beta + c0, sb + c0);
    }
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
    for (int parity = 0; row < rows; row += gridDim.x, parity ^= 1) {
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
        // Thread-local statistics (two passes over registers; E is a power
        // of two, so the multiply by 1/E is exact).
        float s = 0.0f;
#pragma unroll
        for (int i = 0; i < E; ++i) s = __fadd_rn(s, v[i]);
        float mean = __fmul_rn(s, 1.0f / static_cast<float>(E));
        float m2 = 0.0f;
#pragma unroll
        for (int i = 0; i < E; ++i) {
            float d = __fsub_rn(v[i], mean);
            m2 = __fmaf_rn(d, d, m2);
        }
        // Warp: butterfly merge, counts double each step.
        float n = static_cast<float>(E);
#pragma unroll
        for (int m = 1; m < 32; m <<= 1) {
            float mo = __shfl_xor_sync(0xffffffffu, mean, m);
            float m2o = __shfl_xor_sync(0xffffffffu, m2, m);
            chan_equal(mean, m2, mo, m2o, n);
            n = __fmul_rn(n, 2.0f);
        }
        if (lane == 0) {
            s_mean[parity][w] = mean;
            s_m2[parity][w] = m2;
        }
        __syncthreads();
        // Every warp merges the nw warp results the same way.
        float gm = lane < nw ? s_mean[parity][lane] : 0.0f, gm2 = lane < nw ? s_m2[parity][lane] : 0.0f;
        if (pow2) {
            // equal counts again: butterfly inside aligned groups of nw lanes
            float gn = n;
            for (int m = 1; m < nw; m <<= 1) {
                float mo = __shfl_xor_sync(0xffffffffu, gm, m);
                float m2o = __shfl_xor_sync(0xffffffffu, gm2, m);
                chan_equal(gm, gm2, mo, m2o, gn);
                gn = __fmul_rn(gn, 2.0f);
            }
        } else if (lane == 0) {
            float gn = n;
            for (int j = 1; j < nw; ++j) {
                float tot = __fadd_rn(gn, n);
                float d = __fsub_rn(s_mean[parity][j], gm);
                gm = __fadd_rn(gm, __fmul_rn(d, __fdiv_rn(n, tot)));
                gm2 = __fadd_rn(__fadd_rn(gm2, s_m2[parity][j]),
                                __fmul_rn(__fmul_rn(d, d), __fdiv_rn(__fmul_rn(gn, n), tot)));
                gn = tot;
            }
        }
        gm = __shfl_sync(0xffffffffu, gm, 0);
        gm2 = __shfl_sync(0xffffffffu, gm2, 0);
        const float var = __fdiv_rn(gm2, static_cast<float>(cols));
        const float rstd = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(var, eps)));
        Pack<T>* yr = reinterpret_cast<Pack<T>*>(y + row * cols);
#pragma unroll
        for (int i = 0; i < NV; ++i) {
            const int c0 = (t + i * th) * PV;
            float g[PV], b[PV];
#pragma unroll
            for (int e = 0; e < PV; e += 4) {
                const float4 gv = *reinterpret_cast<const float4*>(sg + c0 + e);
                const float4 bv = *reinterpret_cast<const float4*>(sb + c0 + e);
                g[e] = gv.x; g[e + 1] = gv.y; g[e + 2] = gv.z; g[e + 3] = gv.w;
                b[e] = bv.x; b[e + 1] = bv.y; b[e + 2] = bv.z; b[e + 3] = bv.w;
            }
            Pack<T> o;
#pragma unroll
            for (int e = 0; e < PV; ++e) {
                float z = __fmul_rn(__fsub_rn(v[i * PV + e], gm), rstd);
                o.v[e] = from_f_tag(__fmaf_rn(z, g[e], b[e]), static_cast<T*>(nullptr));
            }
            yr[t + i * th] = o;
        }
#pragma unroll
        for (int i = 0; i < NV; ++i) {
            cur[i] = nxt[i];
            nxt[i] = nxt2[i];
        }
    }
}

template <typename T, typename GT>
__global__ void __launch_bounds__(256) k_layer_norm_generic(const T* __restrict__ x, const GT* __restrict__ gamma,
                                                            const GT* __restrict__ beta, T* __restrict__ y,
                                                            int64_t rows, int64_t cols, float eps) {
    __shared__ float s_n[8], s_mean[8], s_m2[8];
    const int t = threadIdx.x, lane = t & 31, w = t >> 5;
    for (int64_t row = blockIdx.x; row < rows; row += gridDim.x) {
        const T* xr = x + row * cols;
        float n = 0.0f, mean = 0.0f, m2 = 0.0f;
        for (int64_t c = t; c < cols; c += 256) {
            float v = to_f(xr[c]);
            n = __fadd_rn(n, 1.0f);
            float d = __fsub_rn(v, mean);
            mean = __fadd_rn(mean, __fdiv_rn(d, n));
            m2 = __fmaf_rn(d, __fsub_rn(v, mean), m2);
        }
        // General Chan merge down a fixed tree (lane i absorbs lane i+m).
#pragma unroll
        for (int m = 16; m >= 1; m >>= 1) {
            float nb = __shfl_down_sync(0xffffffffu, n, m);
            float mb = __shfl_down_sync(0xffffffffu, mean, m);
            float m2b = __shfl_down_sync(0xffffffffu, m2, m);
            if (lane < m && nb > 0.0f) {
                float tot = __fadd_rn(n, nb);
                float d = __fsub_rn(mb, mean);
                mean = __fadd_rn(mean, __fmul_rn(d, __fdiv_rn(nb, tot)));
                m2 = __fadd_rn(__fadd_rn(m2, m2b), __fmul_rn(__fmul_rn(d, d), __fdiv_rn(__fmul_rn(n, nb), tot)));
                n = tot;
            }
        }
        __syncthreads();
        if (lane == 0) {
            s_n[w] = n;
            s_mean[w] = mean;
            s_m2[w] = m2;
        }
        __syncthreads();
        float gn = s_n[0], gm = s_mean[0], gm2 = s_m2[0];
        for (int j = 1; j < 8; ++j) {
            float nb = s_n[j];
            if (nb <= 0.0f) continue;
            float tot = __fadd_rn(gn, nb);
            float d = __fsub_rn(s_mean[j], gm);
            gm = __fadd_rn(gm, __fmul_rn(d, __fdiv_rn(nb, tot)));
            gm2 = __fadd_rn(__fadd_rn(gm2, s_m2[j]), __fmul_rn(__fmul_rn(d, d), __fdiv_rn(__fmul_rn(gn, nb), tot)));
            gn = tot;
        }
        const float var = __fdiv_rn(gm2, static_cast<float>(cols));
        const float rstd = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(var, eps)));
        T* yr = y + row * cols;
        for (int64_t c = t; c < cols; c += 256) {
            float z = __fmul_rn(__fsub_rn(to_f(xr[c]), gm), rstd);
            yr[c] = from_f_tag(__fmaf_rn(z, to_f(gamma[c]), to_f(beta[c])), static_cast<T*>(nullptr));
        }
    }
}

template <typename T, typename GT, int NV>
qsml_status_t launch_reg(Context* ctx, const T* x, const GT* g, const GT* b, T* y, int64_t rows, int cols,
                         float eps, unsigned th) {
    // gamma and beta as binary32 in dynamic shared memory: 8 bytes per column,
    // at most 128 KiB (fp16 rows of 256 threads x 8 packs x 8 = 16384 columns).
    const size_t smem = static_cast<size_t>(cols) * 2 * sizeof(float);
    // Resident CTAs per SM for this block size and width, queried once per
    // kernel variant (later calls, graph capture included, make no runtime
    // query); the attribute for more than 48 KiB is set at the same time.
    static std::mutex mu;
    static std::map<std::pair<unsigned, int>, int> per_sm_cache;
    int per_sm = 0;
    {
        std::lock_guard<std::mutex> lk(mu);
        auto key = std::make_pair(th, cols);
        auto it = per_sm_cache.find(key);
        if (it == per_sm_cache.end()) {
            if (smem > 48 * 1024)
                QSML_TRY_STATUS(check_cuda(ctx,
                                           cudaFuncSetAttribute(k_layer_norm_reg<T, GT, NV>,
                                                                cudaFuncAttributeMaxDynamicSharedMemorySize,
                                                                static_cast<int>(smem)),
                                           "layer norm: shared-memory attribute"));
            cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, k_layer_norm_reg<T, GT, NV>, static_cast<int>(th),
                                                          smem);
            if (per_sm < 1) per_sm = 1;
            per_sm_cache[key] = per_sm;
        } else {
            per_sm = it->second;
        }
    }
    int64_t grid = static_cast<int64_t>(ctx->num_sms) * per_sm;
    if (grid > rows) grid = rows;
    k_layer_norm_reg<T, GT, NV><<<static_cast<unsigned>(grid), th, smem, ctx->stream>>>(x, g, b, y, rows, cols, eps);
    return after_launch(ctx, "k_layer_norm_reg");
}

template <typename T, typename GT>
qsml_status_t run_ln(Context* ctx, const T* x, const GT* g, const GT* b, T* y, int64_t rows, int64_t cols, float eps) {
    constexpr int PV = Pack<T>::N;
    if (cols % PV == 0 && aligned16(x) && aligned16(y) && aligned16(g) && aligned16(b) && cols <= INT32_MAX) {
        const int64_t packs = cols / PV;
        int nv = 0;
        for (int cand : {1, 2, 4, 8}) {
            if (packs % cand) continue;
            int64_t th = packs / cand;
            // 256-thread CTAs: measured faster than 512 for 4096-wide rows
            if (th % 32 == 0 && th <= 256) {
                nv = cand;
                break;
            }
        }
        if (nv) {
            const unsigned th = static_cast<unsigned>(packs / nv);
            const int c = static_cast<int>(cols);
            switch (nv) {
                case 1: return launch_reg<T, GT, 1>(ctx, x, g, b, y, rows, c, eps, th);
                case 2: return launch_reg<T, GT, 2>(ctx, x, g, b, y, rows, c, eps, th);
                case 4: return launch_reg<T, GT, 4>(ctx, x, g, b, y, rows, c, eps, th);
                default: return launch_reg<T, GT, 8>(ctx, x, g, b, y, rows, c, eps, th);
            }
        }
    }
    int64_t grid = rows < 65535 * 16 ? rows : 65535 * 16;
    k_layer_norm_generic<T, GT><<<static_cast<unsigned>(grid), 256, 0, ctx->stream>>>(x, g, b, y, rows, cols, eps);
    return after_launch(ctx, "k_layer_norm_generic");
}

}  // namespace
}  // namespace qsml

using namespace qsml;

extern "C" qsml_status_t qsml_layer_norm(qsml_ctx* handle, const qsml_tdesc* x, const qsml_tdesc* gamma,
                                         const qsml_tdesc* beta, float eps, const qsml_tdesc* y) {
    QSML_CTX(handle);
    QSML_TRY_STATUS(check_desc(C_, x, "x"));
    QSML_TRY_STATUS(check_desc(C_, gamma, "gamma"));
    QSML_TRY_STATUS(check_desc(C_, beta, "beta"));
    QSML_TRY_STATUS(check_desc(C_, y, "y"));
    if (x->ndim < 1) return set_error(C_, QSML_E_SHAPE, "qsml_layer_norm: x needs at least one dim");
    if (x->dtype != QSML_F32 && x->dtype != QSML_F16)
        return set_error(C_, QSML_E_DTYPE, "qsml_layer_norm: x must be F32 or F16");
    if (y->dtype != x->dtype) return set_error(C_, QSML_E_DTYPE, "qsml_layer_norm: y dtype must equal x dtype");
    if (gamma->dtype != beta->dtype || (gamma->dtype != QSML_F32 && gamma->dtype != x->dtype))
        return set_error(C_, QSML_E_DTYPE, "qsml_layer_norm: gamma/beta must be F32 or x's dtype");
    if (!is_contiguous(x) || !is_contiguous(y) || !is_contiguous(gamma) || !is_contiguous(beta))
        return set_error(C_, QSML_E_UNSUPPORTED, "qsml_layer_norm: x, y, gamma and beta must be contiguous");
    const int64_t cols = x->shape[x->ndim - 1];
    if (numel(gamma) != cols || numel(beta) != cols)
        return set_error(C_, QSML_E_SHAPE, "qsml_layer_norm: gamma/beta must have the last dim's size");
    if (y->ndim != x->ndim) return set_error(C_, QSML_E_SHAPE, "qsml_layer_norm: y shape must equal x shape");
    for (int d = 0; d < x->ndim; ++d)
        if (y->shape[d] != x->shape[d]) return set_error(C_, QSML_E_SHAPE, "qsml_layer_norm: y shape must equal x shape");
    const int64_t n = numel(x);
    if (n == 0) return QSML_OK;
    const int64_t rows = n / cols;
    if (x->dtype == QSML_F32)
        return run_ln<float, float>(C_, static_cast<const float*>(x->data), static_cast<const float*>(gamma->data),
                                    static_cast<const float*>(beta->data), static_cast<float*>(y->data), rows, cols, eps);
    if (gamma->dtype == QSML_F32)
        return run_ln<__half, float>(C_, static_cast<const __half*>(x->data), static_cast<const float*>(gamma->data),
                                     static_cast<const float*>(beta->data), static_cast<__half*>(y->data), rows, cols, eps);
    return run_ln<__half, __half>(C_, static_cast<const __half*>(x->data), static_cast<const __half*>(gamma->data),
                                  static_cast<const __half*>(beta->data), static_cast<__half*>(y->data), rows, cols, eps);
}
