// Layer norm over the last dim: y = (x - mean) / sqrt(var + eps) * gamma + beta
// with the biased (population) variance.  The reference snapshot has no
// layer norm; this is a new op of the same API family.
//
// k_layer_norm_pipe: rows of 2-8 KiB, one warp per row, rows streamed through
// shared memory by bulk copies (row_pipe.cuh); x is read from HBM once and y
// written once.
// k_layer_norm_reg: wider rows, persistent CTAs, one row at a time held in
// registers (16-byte loads) with the next two rows already in flight, so x is
// read once and y written once; gamma/beta stay in shared memory.  The row
// statistics are two block sums (row sum, then squared deviations from the
// mean), so the variance is a true two-pass variance.
// k_layer_norm_wide: binary16 rows of 8-108 KiB and binary32 rows of 32-108
// KiB, one CTA per row, rows streamed through two shared-memory buffers.
// k_layer_norm_generic: any width or alignment, Welford over global memory
// (reads x twice).
#include "qsml_internal.cuh"
#include "row_pipe.cuh"

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

// gamma/beta live in shared memory as binary32 in a split layout: for pack p
// (columns p*PV .. p*PV+PV-1) and k < PV/4, the float4 of columns
// p*PV+4k .. +3 sits at float4 index k*packs + p, so lanes reading
// consecutive packs read consecutive 16-byte words (no bank conflicts for
// binary16 packs of 8 columns).
template <int PV>
__device__ __forceinline__ int param_slot(int p, int k, int packs) {
    return k * packs + p;
}

// Columns p*PV .. p*PV+PV-1 of a gamma/beta vector into the split layout.
template <typename GT, int PV>
__device__ __forceinline__ void load_params(const GT* src, float4* dst, int p, int packs) {
    const GT* q = src + static_cast<int64_t>(p) * PV;
    if constexpr (sizeof(GT) == 4) {
#pragma unroll
        for (int k = 0; k < PV / 4; ++k)
            dst[param_slot<PV>(p, k, packs)] = *reinterpret_cast<const float4*>(q + 4 * k);
    } else {
#pragma unroll
        for (int k = 0; k < PV / 4; ++k) {
            float4 f;
            f.x = __half2float(q[4 * k]);
            f.y = __half2float(q[4 * k + 1]);
            f.z = __half2float(q[4 * k + 2]);
            f.w = __half2float(q[4 * k + 3]);
            dst[param_slot<PV>(p, k, packs)] = f;
        }
    }
}

// Binary32 values to a pack (binary16: two at a time).
template <typename T>
__device__ __forceinline__ Pack<T> to_pack(const float* z) {
    Pack<T> o;
    if constexpr (sizeof(T) == 4) {
#pragma unroll
        for (int e = 0; e < Pack<T>::N; ++e) o.v[e] = z[e];
    } else {
#pragma unroll
        for (int e = 0; e < Pack<T>::N; e += 2) {
            const __half2 h = __floats2half2_rn(z[e], z[e + 1]);
            o.v[e] = __low2half(h);
            o.v[e + 1] = __high2half(h);
        }
    }
    return o;
}

// PV consecutive gamma/beta values as binary32, with 16-byte loads from global
// memory (read-only path).
template <typename GT, int PV>
__device__ __forceinline__ void load_pack_params(const GT* p, float* out) {
    if constexpr (sizeof(GT) == 4) {
#pragma unroll
        for (int i = 0; i < PV; i += 4) {
            const float4 v = __ldg(reinterpret_cast<const float4*>(p + i));
            out[i] = v.x; out[i + 1] = v.y; out[i + 2] = v.z; out[i + 3] = v.w;
        }
    } else {
#pragma unroll
        for (int i = 0; i < PV; i += 8) {
            const uint4 u = __ldg(reinterpret_cast<const uint4*>(p + i));
            const __half* h = reinterpret_cast<const __half*>(&u);
#pragma unroll
            for (int e = 0; e < 8; ++e) out[i + e] = __half2float(h[e]);
        }
    }
}

// Block-wide binary32 sum: xor butterflies inside warps, one slot per warp,
// one barrier, then every thread adds the slots in a fixed order (a butterfly
// over the slots when the warp count is a power of two), so every thread
// holds the same bits.
__device__ __forceinline__ float block_sum(float v, float* slot) {
    const int lane = threadIdx.x & 31, w = threadIdx.x >> 5, nw = blockDim.x >> 5;
#pragma unroll
    for (int m = 16; m >= 1; m >>= 1) v = __fadd_rn(v, __shfl_xor_sync(0xffffffffu, v, m));
    if (lane == 0) slot[w] = v;
    __syncthreads();
    if ((nw & (nw - 1)) == 0) {
        float a = slot[lane & (nw - 1)];
        for (int m = 1; m < nw; m <<= 1) a = __fadd_rn(a, __shfl_xor_sync(0xffffffffu, a, m));
        return a;
    }
    float a = slot[0];
    for (int j = 1; j < nw; ++j) a = __fadd_rn(a, slot[j]);
    return a;
}

// Persistent CTAs, one row at a time held in registers (16-byte loads) with
// the next two rows in flight; the loop body is unrolled three times so the
// three row buffers change roles without register copies.  gamma/beta (as
// binary32) sit in dynamic shared memory, each thread holding exactly the
// columns it reads.  Statistics are two block sums per row: the row sum
// (mean = sum * (1/n)), then the sum of squared deviations from that mean
// (var = sum * (1/n)); rstd = rsqrtf(var + eps).  Each sum has its own slots:
// a thread rewrites the sum slots of the next row only after passing this
// row's second barrier, which every thread reaches after reading them, and
// the deviation slots only after the next row's first barrier, likewise.
template <typename T, typename GT, int NV>
__global__ void __launch_bounds__(256) k_layer_norm_reg(const T* __restrict__ x, const GT* __restrict__ gamma,
                                                        const GT* __restrict__ beta, T* __restrict__ y,
                                                        int64_t rows, int cols, float eps, int defer) {
    pdl_start(defer);
    constexpr int PV = Pack<T>::N;
    constexpr int E = NV * PV;  // elements per thread
    extern __shared__ float4 ln_smem[];
    const int packs = cols / PV;
    float4* sg = ln_smem;
    float4* sb = ln_smem + cols / 4;
    __shared__ float s_sum[8], s_dev[8];
    const int t = threadIdx.x, th = blockDim.x;
#pragma unroll
    for (int i = 0; i < NV; ++i) {
        load_params<GT, PV>(gamma, sg, t + i * th, packs);
        load_params<GT, PV>(beta, sb, t + i * th, packs);
    }
    const float inv_n = __frcp_rn(static_cast<float>(cols));
    auto load_row = [&](Pack<T>(&buf)[NV], int64_t r) {
        if (r < rows) {
            const Pack<T>* xr = reinterpret_cast<const Pack<T>*>(x + r * cols);
#pragma unroll
            for (int i = 0; i < NV; ++i) buf[i] = xr[t + i * th];
        }
    };
    auto process = [&](const Pack<T>(&buf)[NV], int64_t r) {
        float v[E];
#pragma unroll
        for (int i = 0; i < NV; ++i)
#pragma unroll
            for (int e = 0; e < PV; ++e) v[i * PV + e] = to_f(buf[i].v[e]);
        float s0 = 0.0f, s1 = 0.0f;
#pragma unroll
        for (int i = 0; i < E; i += 2) {
            s0 = __fadd_rn(s0, v[i]);
            s1 = __fadd_rn(s1, v[i + 1]);
        }
        const float mean = __fmul_rn(block_sum(__fadd_rn(s0, s1), s_sum), inv_n);
        float q0 = 0.0f, q1 = 0.0f;
#pragma unroll
        for (int i = 0; i < E; i += 2) {
            const float d0 = __fsub_rn(v[i], mean), d1 = __fsub_rn(v[i + 1], mean);
            q0 = __fmaf_rn(d0, d0, q0);
            q1 = __fmaf_rn(d1, d1, q1);
        }
        const float var = __fmul_rn(block_sum(__fadd_rn(q0, q1), s_dev), inv_n);
        const float rstd = rsqrtf(__fadd_rn(var, eps));
        Pack<T>* yr = reinterpret_cast<Pack<T>*>(y + r * cols);
#pragma unroll
        for (int i = 0; i < NV; ++i) {
            const int p = t + i * th;
            float z[PV];
#pragma unroll
            for (int e = 0; e < PV; e += 4) {
                const float4 gv = sg[param_slot<PV>(p, e / 4, packs)];
                const float4 bv = sb[param_slot<PV>(p, e / 4, packs)];
                const float g[4] = {gv.x, gv.y, gv.z, gv.w}, b[4] = {bv.x, bv.y, bv.z, bv.w};
#pragma unroll
                for (int k = 0; k < 4; ++k)
                    z[e + k] = __fmaf_rn(__fmul_rn(__fsub_rn(v[i * PV + e + k], mean), rstd), g[k], b[k]);
            }
            yr[t + i * th] = to_pack<T>(z);
        }
    };
    const int64_t G = gridDim.x;
    Pack<T> A[NV], B[NV], C[NV];
    int64_t row = blockIdx.x;
    load_row(A, row);
    load_row(B, row + G);
    while (row < rows) {
        load_row(C, row + 2 * G);
        process(A, row);
        if ((row += G) >= rows) break;
        load_row(A, row + 2 * G);
        process(B, row);
        if ((row += G) >= rows) break;
        load_row(B, row + 2 * G);
        process(C, row);
        row += G;
    }
    pdl_end(defer);
}

// Rows streamed through shared memory (row_pipe.cuh), one warp per row:
// gamma/beta as binary32 in front of the row buffers; per row three passes
// over the buffer -- the sum (PV interleaved partial sums per lane, then the
// warp), the squared deviations from the mean the same way, and the output.
template <typename T, typename GT>
__global__ void __launch_bounds__(rowpipe::kMaxWarps * 32, 1)
    k_layer_norm_pipe(const T* __restrict__ x, const GT* __restrict__ gamma, const GT* __restrict__ beta,
                      T* __restrict__ y, int64_t rows, int cols, float eps, int slots, int* status, int defer) {
    pdl_start(defer);
    constexpr int PV = Pack<T>::N;
    extern __shared__ float4 ln_pipe_smem[];
    __shared__ uint64_t bars[rowpipe::kMaxWarps * rowpipe::kMaxSlots];
    const int packs = cols / PV, lane = threadIdx.x & 31;
    float4* sg = ln_pipe_smem;
    float4* sb = ln_pipe_smem + cols / 4;
    unsigned char* ring = reinterpret_cast<unsigned char*>(sb + cols / 4);
    for (int p = threadIdx.x; p < packs; p += blockDim.x) {
        load_params<GT, PV>(gamma, sg, p, packs);
        load_params<GT, PV>(beta, sb, p, packs);
    }
    __syncthreads();
    const float n = static_cast<float>(cols);
    const bool ok = rowpipe::stream_rows(
        reinterpret_cast<const unsigned char*>(x), rows, static_cast<uint32_t>(cols * sizeof(T)), slots, ring, bars,
        wait_limit(status), [&](int64_t row, unsigned char* buf) {
            const Pack<T>* xs = reinterpret_cast<const Pack<T>*>(buf);
            float part[PV];
#pragma unroll
            for (int e = 0; e < PV; ++e) part[e] = 0.0f;
#pragma unroll 4
            for (int p = lane; p < packs; p += 32) {
                const Pack<T> v = xs[p];
#pragma unroll
                for (int e = 0; e < PV; ++e) part[e] = __fadd_rn(part[e], to_f(v.v[e]));
            }
            float s = part[0];
#pragma unroll
            for (int e = 1; e < PV; ++e) s = __fadd_rn(s, part[e]);
            const float mean = __fdiv_rn(rowpipe::warp_sum(s), n);
#pragma unroll
            for (int e = 0; e < PV; ++e) part[e] = 0.0f;
#pragma unroll 4
            for (int p = lane; p < packs; p += 32) {
                const Pack<T> v = xs[p];
#pragma unroll
                for (int e = 0; e < PV; ++e) {
                    const float d = __fsub_rn(to_f(v.v[e]), mean);
                    part[e] = __fmaf_rn(d, d, part[e]);
                }
            }
            float q = part[0];
#pragma unroll
            for (int e = 1; e < PV; ++e) q = __fadd_rn(q, part[e]);
            const float var = __fdiv_rn(rowpipe::warp_sum(q), n);
            const float rstd = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(var, eps)));
            Pack<T>* yr = reinterpret_cast<Pack<T>*>(y + row * cols);
#pragma unroll 2
            for (int p = lane; p < packs; p += 32) {
                const Pack<T> v = xs[p];
                float z[PV];
#pragma unroll
                for (int e = 0; e < PV; e += 4) {
                    const float4 gv = sg[param_slot<PV>(p, e / 4, packs)];
                    const float4 bv = sb[param_slot<PV>(p, e / 4, packs)];
                    const float g[4] = {gv.x, gv.y, gv.z, gv.w}, b[4] = {bv.x, bv.y, bv.z, bv.w};
#pragma unroll
                    for (int k = 0; k < 4; ++k)
                        z[e + k] = __fmaf_rn(__fmul_rn(__fsub_rn(to_f(v.v[e + k]), mean), rstd), g[k], b[k]);
                }
                yr[p] = to_pack<T>(z);
            }
        });
    if (!ok && lane == 0) atomicExch(status, QSML_E_TIMEOUT);
    pdl_end(defer);
}

// Binary16 rows of 8-108 KiB and binary32 rows of 32-108 KiB: one CTA of TH
// threads per row, rows streamed through two shared-memory buffers
// (row_pipe.cuh, stream_rows_cta): the sum, the squared deviations from the
// mean and the output as three passes over the buffer; gamma/beta are read
// from global memory (L2-resident after the first row) with 16-byte loads.
// With REG > 0 (rows of at most TH * REG packs) each thread keeps the
// gamma/beta of its packs in registers for all its rows instead.
template <typename T, typename GT, int REG, int TH>
__global__ void __launch_bounds__(TH) k_layer_norm_wide(const T* __restrict__ x, const GT* __restrict__ gamma,
                                                         const GT* __restrict__ beta, T* __restrict__ y,
                                                         int64_t rows, int cols, float eps, int* status, int defer) {
    pdl_start(defer);
    constexpr int PV = Pack<T>::N;
    float rg[REG > 0 ? REG : 1][PV], rb[REG > 0 ? REG : 1][PV];
    if constexpr (REG > 0) {
        const int packs = cols / PV;
#pragma unroll
        for (int j = 0; j < REG; ++j) {
            const int p = static_cast<int>(threadIdx.x) + j * static_cast<int>(blockDim.x);
            if (p < packs) {
                load_pack_params<GT, PV>(gamma + static_cast<int64_t>(p) * PV, rg[j]);
                load_pack_params<GT, PV>(beta + static_cast<int64_t>(p) * PV, rb[j]);
            }
        }
    }
    extern __shared__ float4 ln_wide_smem[];
    __shared__ uint64_t bars[2];
    __shared__ float s_sum[32], s_dev[32];
    const int packs = cols / PV, t = threadIdx.x, th = blockDim.x;
    const float n = static_cast<float>(cols);
    const bool ok = rowpipe::stream_rows_cta(
        reinterpret_cast<const unsigned char*>(x), rows, static_cast<uint32_t>(cols * sizeof(T)),
        reinterpret_cast<unsigned char*>(ln_wide_smem), bars, wait_limit(status),
        [&](int64_t row, unsigned char* buf) {
            const Pack<T>* xs = reinterpret_cast<const Pack<T>*>(buf);
            float part[PV];
#pragma unroll
            for (int e = 0; e < PV; ++e) part[e] = 0.0f;
#pragma unroll 2
            for (int p = t; p < packs; p += th) {
                const Pack<T> v = xs[p];
#pragma unroll
                for (int e = 0; e < PV; ++e) part[e] = __fadd_rn(part[e], to_f(v.v[e]));
            }
            float s = part[0];
#pragma unroll
            for (int e = 1; e < PV; ++e) s = __fadd_rn(s, part[e]);
            const float mean = __fdiv_rn(rowpipe::cta_combine<false>(s, s_sum), n);
#pragma unroll
            for (int e = 0; e < PV; ++e) part[e] = 0.0f;
#pragma unroll 2
            for (int p = t; p < packs; p += th) {
                const Pack<T> v = xs[p];
#pragma unroll
                for (int e = 0; e < PV; ++e) {
                    const float d = __fsub_rn(to_f(v.v[e]), mean);
                    part[e] = __fmaf_rn(d, d, part[e]);
                }
            }
            float q = part[0];
#pragma unroll
            for (int e = 1; e < PV; ++e) q = __fadd_rn(q, part[e]);
            const float var = __fdiv_rn(rowpipe::cta_combine<false>(q, s_dev), n);
            const float rstd = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(var, eps)));
            Pack<T>* yr = reinterpret_cast<Pack<T>*>(y + row * cols);
            if constexpr (REG > 0) {
#pragma unroll
                for (int j = 0; j < REG; ++j) {
                    const int p = t + j * th;
                    if (p < packs) {
                        const Pack<T> v = xs[p];
                        float z[PV];
#pragma unroll
                        for (int e = 0; e < PV; ++e)
                            z[e] = __fmaf_rn(__fmul_rn(__fsub_rn(to_f(v.v[e]), mean), rstd), rg[j][e], rb[j][e]);
                        yr[p] = to_pack<T>(z);
                    }
                }
            } else {
                for (int p = t; p < packs; p += th) {
                    const Pack<T> v = xs[p];
                    float g[PV], b[PV];
                    load_pack_params<GT, PV>(gamma + static_cast<int64_t>(p) * PV, g);
                    load_pack_params<GT, PV>(beta + static_cast<int64_t>(p) * PV, b);
                    float z[PV];
#pragma unroll
                    for (int e = 0; e < PV; ++e)
                        z[e] = __fmaf_rn(__fmul_rn(__fsub_rn(to_f(v.v[e]), mean), rstd), g[e], b[e]);
                    yr[p] = to_pack<T>(z);
                }
            }
        });
    if (!ok && t == 0) atomicExch(status, QSML_E_TIMEOUT);
    pdl_end(defer);
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

// What a layer-norm launch reads (x, gamma, beta) and writes (y), for overlap.
template <typename T, typename GT>
Footprint ln_footprint(const T* x, const GT* g, const GT* b, const T* y, int64_t rows, int cols) {
    Footprint f;
    const size_t n = static_cast<size_t>(rows) * cols * sizeof(T);
    f.read(span_of(x, n)).read(span_of(g, cols * sizeof(GT))).read(span_of(b, cols * sizeof(GT))).write(span_of(y, n));
    return f;
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
    {
        const int defer = plan_launch(ctx, ln_footprint(x, g, b, y, rows, cols));
        const cudaError_t e = launch_pdl(k_layer_norm_reg<T, GT, NV>, dim3(static_cast<unsigned>(grid)), dim3(th),
                                         smem, ctx->stream, x, g, b, y, rows, cols, eps, defer);
        if (e != cudaSuccess) return check_cuda(ctx, e, "k_layer_norm_reg");
    }
    return after_launch(ctx, "k_layer_norm_reg");
}

template <typename T, typename GT>
qsml_status_t launch_pipe(Context* ctx, const T* x, const GT* g, const GT* b, T* y, int64_t rows, int cols, float eps,
                          const rowpipe::Plan& p) {
    static std::mutex mu;
    static size_t attr_set = 0;  // largest dynamic shared memory opted in so far
    {
        std::lock_guard<std::mutex> lk(mu);
        if (p.smem > 48 * 1024 && p.smem > attr_set) {
            QSML_TRY_STATUS(check_cuda(ctx,
                                       cudaFuncSetAttribute(k_layer_norm_pipe<T, GT>,
                                                            cudaFuncAttributeMaxDynamicSharedMemorySize,
                                                            static_cast<int>(p.smem)),
                                       "layer norm: shared-memory attribute"));
            attr_set = p.smem;
        }
    }
    {
        const int defer = plan_launch(ctx, ln_footprint(x, g, b, y, rows, cols));
        const cudaError_t e = launch_pdl(k_layer_norm_pipe<T, GT>, dim3(p.grid), dim3(p.warps * 32), p.smem,
                                         ctx->stream, x, g, b, y, rows, cols, eps, p.slots, ctx->status, defer);
        if (e != cudaSuccess) return check_cuda(ctx, e, "k_layer_norm_pipe");
    }
    return after_launch(ctx, "k_layer_norm_pipe");
}

template <typename T, typename GT, int REG, int TH>
qsml_status_t launch_wide_as(Context* ctx, const T* x, const GT* g, const GT* b, T* y, int64_t rows, int cols,
                             float eps) {
    const size_t smem = 2 * static_cast<size_t>(cols) * sizeof(T);
    static std::mutex mu;
    static bool attr_set = false;
    int per_sm = 1;
    {
        std::lock_guard<std::mutex> lk(mu);
        if (!attr_set) {
            QSML_TRY_STATUS(check_cuda(ctx,
                                       cudaFuncSetAttribute(k_layer_norm_wide<T, GT, REG, TH>,
                                                            cudaFuncAttributeMaxDynamicSharedMemorySize,
                                                            static_cast<int>(2 * rowpipe::kWideMaxRowBytes)),
                                       "layer norm: shared-memory attribute"));
            attr_set = true;
        }
        if (TH < 512) {
            // several CTAs per SM when their buffers and registers fit (one
            // occupancy query per row width)
            static std::unordered_map<size_t, int> per_sm_by_smem;
            auto it = per_sm_by_smem.find(smem);
            if (it == per_sm_by_smem.end()) {
                cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, k_layer_norm_wide<T, GT, REG, TH>, TH, smem);
                if (per_sm < 1) per_sm = 1;
                per_sm_by_smem[smem] = per_sm;
            } else {
                per_sm = it->second;
            }
        }
    }
    int64_t grid = static_cast<int64_t>(ctx->num_sms) * per_sm;
    if (grid > rows) grid = rows;
    const int defer = plan_launch(ctx, ln_footprint(x, g, b, y, rows, cols));
    const cudaError_t e = launch_pdl(k_layer_norm_wide<T, GT, REG, TH>, dim3(static_cast<unsigned>(grid)), dim3(TH),
                                     smem, ctx->stream, x, g, b, y, rows, cols, eps, ctx->status, defer);
    if (e != cudaSuccess) return check_cuda(ctx, e, "k_layer_norm_wide");
    return after_launch(ctx, "k_layer_norm_wide");
}

// Thread count and gamma/beta placement by row width (measured on binary16
// rows of 12-80 KiB: these choices ran 15-45 % faster than the register
// kernel or the other thread counts there):
//   * up to 1024 packs: 128 threads, gamma/beta in registers (8 packs each);
//   * binary16 rows up to 2048 packs: binary32 gamma/beta in registers with
//     512 threads (4 packs each), binary16 gamma/beta from L1/L2 with 256
//     threads (several CTAs per SM);
//   * binary16 rows up to 52 KiB (two CTAs' buffers fit an SM): 256 threads,
//     gamma/beta from L1/L2;
//   * binary32 rows up to 4096 packs: 512 threads, registers (8 packs each);
//   * wider: 512 threads, gamma/beta from L1/L2 (16 gamma/beta values per
//     binary16 pack in registers would spill).
template <typename T, typename GT>
qsml_status_t launch_wide(Context* ctx, const T* x, const GT* g, const GT* b, T* y, int64_t rows, int cols,
                          float eps) {
    const int packs = cols / Pack<T>::N;
    if (packs <= 128 * 8) return launch_wide_as<T, GT, 8, 128>(ctx, x, g, b, y, rows, cols, eps);
    if constexpr (sizeof(T) == 2) {
        if (packs <= 512 * 4) {
            if constexpr (sizeof(GT) == 4) return launch_wide_as<T, GT, 4, 512>(ctx, x, g, b, y, rows, cols, eps);
            else return launch_wide_as<T, GT, 0, 256>(ctx, x, g, b, y, rows, cols, eps);
        }
        if (packs <= rowpipe::kWide256MaxPacks) return launch_wide_as<T, GT, 0, 256>(ctx, x, g, b, y, rows, cols, eps);
    } else {
        if (packs <= 512 * 8) return launch_wide_as<T, GT, 8, 512>(ctx, x, g, b, y, rows, cols, eps);
    }
    return launch_wide_as<T, GT, 0, 512>(ctx, x, g, b, y, rows, cols, eps);
}

template <typename T, typename GT>
qsml_status_t run_ln(Context* ctx, const T* x, const GT* g, const GT* b, T* y, int64_t rows, int64_t cols, float eps) {
    constexpr int PV = Pack<T>::N;
    rowpipe::Plan plan;
    if (rowpipe::use_pipe(cols * sizeof(T), sizeof(T)) && aligned16(x) && aligned16(y) && ctx->status && cols <= INT32_MAX &&
        rowpipe::plan(ctx, rows, static_cast<uint64_t>(cols) * sizeof(T), static_cast<size_t>(cols) * 8, &plan))
        return launch_pipe<T, GT>(ctx, x, g, b, y, rows, static_cast<int>(cols), eps, plan);
    const uint64_t row_bytes = static_cast<uint64_t>(cols) * sizeof(T);
    if (rowpipe::use_wide(row_bytes, sizeof(T)) && row_bytes % 16 == 0 && aligned16(x) && aligned16(y) &&
        aligned16(g) && aligned16(b) && ctx->status)
        return launch_wide<T, GT>(ctx, x, g, b, y, rows, static_cast<int>(cols), eps);
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
