// Softmax over one axis: y = exp(x - max) / sum(exp(x - max)).
//
// Reference: Ops::softmax (Ops/Elementwise.cpp:395-417) runs one workgroup
// per row with the shader of Elementwise.cpp:98-135: a shared-memory tree for
// the row max, another for the sum of exp(x - max), then
// out = exp(x - max) / sum.  Its indexing (offset = row * axis_size) is right
// for the last axis only.  Here the same arithmetic (max, subtract, exp,
// binary32 sum; the division as a correctly rounded reciprocal per slice and
// one multiply per element, within 1.5 ulp of the quotient -- GLSL's `/` is
// not correctly rounded either) runs over any axis.  exp is expf, except in
// the last-axis row kernels on binary16 rows, which use the hardware base-2
// exponential (relative error about 2^-22, far below binary16 resolution):
//   * k_softmax_pipe -- last axis, rows of 2-8 KiB (binary16: below 8 KiB):
//     one warp per row, rows streamed through shared memory by bulk copies
//     (row_pipe.cuh);
//   * k_softmax_rows -- last axis, wider rows held in registers (16-byte
//     loads): persistent CTAs with the next two rows in flight, so x is read
//     once and y written once;
//   * k_softmax_wide -- last axis, binary16 rows of 8-108 KiB (tried before
//     the other kernels) and binary32 rows of 32-108 KiB: one CTA per row, rows
//     streamed through two shared-memory buffers (row_pipe.cuh);
//   * k_softmax_rows_generic -- last axis, any width: one CTA per row, three
//     passes over global memory (max, sum, write);
//   * k_softmax_long_{max,sum,out} -- last axis, fewer rows than SMs and long
//     rows: slices of each row over many CTAs, three launches;
//   * k_softmax_cols -- inner dims after the axis: one thread per column of
//     the [outer, k, inner] view, three passes over k.
// The max is IEEE 754-2019 maximum (a NaN in the row makes the row NaN), and
// every combine order is fixed by the shape, so results are deterministic.
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

// exp(x - m) in the last-axis row kernels, given mk = m * log2(e): expf for
// binary32 rows; for binary16 rows 2^(x*log2(e) - mk), one fma and the
// hardware base-2 exponential (ex2.approx, relative error about 2^-22; the
// rounding of mk adds |m| * 2^-24 to the exponent), far below binary16
// resolution.
template <typename T>
__device__ __forceinline__ float row_exp(float x, float m, float mk) {
    if constexpr (sizeof(T) == 4) {
        return expf(__fsub_rn(x, m));
    } else {
        float r;
        asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(r) : "f"(__fmaf_rn(x, 1.4426950408889634f, -mk)));
        return r;
    }
}

// Binary16 rows two columns at a time: row_exp and the __fadd_rn /
// __fmul_rn around it issued as packed binary32 instructions
// (fma/add/mul.rn.f32x2, each lane rounded to nearest even exactly like the
// scalar instruction), so the results are bit-identical and the kernels,
// issue-bound on these rows, issue fewer instructions.
__device__ __forceinline__ uint64_t f2pack(float lo, float hi) {
    uint64_t r;
    asm("mov.b64 %0, {%1, %2};" : "=l"(r) : "f"(lo), "f"(hi));
    return r;
}
__device__ __forceinline__ void f2unpack(uint64_t v, float& lo, float& hi) {
    asm("mov.b64 {%0, %1}, %2;" : "=f"(lo), "=f"(hi) : "l"(v));
}
__device__ __forceinline__ uint64_t add2(uint64_t a, uint64_t b) {
    uint64_t r;
    asm("add.rn.f32x2 %0, %1, %2;" : "=l"(r) : "l"(a), "l"(b));
    return r;
}
__device__ __forceinline__ uint64_t mul2(uint64_t a, uint64_t b) {
    uint64_t r;
    asm("mul.rn.f32x2 %0, %1, %2;" : "=l"(r) : "l"(a), "l"(b));
    return r;
}
// {2^(x0*log2(e) - mk), 2^(x1*log2(e) - mk)} for the pair h = {x0, x1};
// l2e = {log2(e), log2(e)}, nmk = {-mk, -mk}.  Per lane row_exp<__half>.
__device__ __forceinline__ uint64_t exp_pair(__half2 h, uint64_t l2e, uint64_t nmk) {
    const float2 f = __half22float2(h);
    uint64_t a;
    asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(a) : "l"(f2pack(f.x, f.y)), "l"(l2e), "l"(nmk));
    float a0, a1, r0, r1;
    f2unpack(a, a0, a1);
    asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(r0) : "f"(a0));
    asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(r1) : "f"(a1));
    return f2pack(r0, r1);
}

// Sum pass of a binary16 row from shared memory: per-column partials (the
// same per-column order as the scalar loop), combined in column order.
__device__ __forceinline__ float half_exp_sum(const Pack<__half>* xs, int packs, int t, int stride, float mk) {
    constexpr int PV = Pack<__half>::N;
    const uint64_t l2e = f2pack(1.4426950408889634f, 1.4426950408889634f), nmk = f2pack(-mk, -mk);
    uint64_t part2[PV / 2];
#pragma unroll
    for (int e = 0; e < PV / 2; ++e) part2[e] = 0;  // both lanes +0.0f
#pragma unroll 4
    for (int p = t; p < packs; p += stride) {
        const Pack<__half> v = xs[p];
        const __half2* h = reinterpret_cast<const __half2*>(v.v);
#pragma unroll
        for (int e = 0; e < PV / 2; ++e) part2[e] = add2(part2[e], exp_pair(h[e], l2e, nmk));
    }
    float part[PV];
#pragma unroll
    for (int e = 0; e < PV / 2; ++e) f2unpack(part2[e], part[2 * e], part[2 * e + 1]);
    float s = part[0];
#pragma unroll
    for (int e = 1; e < PV; ++e) s = __fadd_rn(s, part[e]);
    return s;
}

// Output pass of a binary16 row: y = exp(x - m) * inv, rounded to binary16.
__device__ __forceinline__ void half_exp_out(const Pack<__half>* xs, Pack<__half>* yr, int packs, int t, int stride,
                                             float mk, float inv) {
    constexpr int PV = Pack<__half>::N;
    const uint64_t l2e = f2pack(1.4426950408889634f, 1.4426950408889634f), nmk = f2pack(-mk, -mk);
    const uint64_t inv2 = f2pack(inv, inv);
#pragma unroll 2
    for (int p = t; p < packs; p += stride) {
        const Pack<__half> v = xs[p];
        const __half2* h = reinterpret_cast<const __half2*>(v.v);
        Pack<__half> o;
        __half2* oh = reinterpret_cast<__half2*>(o.v);
#pragma unroll
        for (int e = 0; e < PV / 2; ++e) {
            float z0, z1;
            f2unpack(mul2(exp_pair(h[e], l2e, nmk), inv2), z0, z1);
            oh[e] = __floats2half2_rn(z0, z1);
        }
        yr[p] = o;
    }
}

// Binary16 rows of which each thread holds at most KP packs: the sum pass
// keeps its exponentials in registers (ex), and the output pass multiplies
// those instead of reading the row again and recomputing them -- the same
// values, so the same bits, with one pass over shared memory less.
template <int KP>
__device__ __forceinline__ float half_exp_sum_keep(const Pack<__half>* xs, int packs, int t, int stride, float mk,
                                                   uint64_t (&ex)[KP][Pack<__half>::N / 2]) {
    constexpr int PV = Pack<__half>::N;
    const uint64_t l2e = f2pack(1.4426950408889634f, 1.4426950408889634f), nmk = f2pack(-mk, -mk);
    uint64_t part2[PV / 2];
#pragma unroll
    for (int e = 0; e < PV / 2; ++e) part2[e] = 0;  // both lanes +0.0f
#pragma unroll
    for (int k = 0; k < KP; ++k) {
        const int p = t + k * stride;
        if (p < packs) {
            const Pack<__half> v = xs[p];
            const __half2* h = reinterpret_cast<const __half2*>(v.v);
#pragma unroll
            for (int e = 0; e < PV / 2; ++e) {
                ex[k][e] = exp_pair(h[e], l2e, nmk);
                part2[e] = add2(part2[e], ex[k][e]);
            }
        }
    }
    float part[PV];
#pragma unroll
    for (int e = 0; e < PV / 2; ++e) f2unpack(part2[e], part[2 * e], part[2 * e + 1]);
    float s = part[0];
#pragma unroll
    for (int e = 1; e < PV; ++e) s = __fadd_rn(s, part[e]);
    return s;
}

template <int KP>
__device__ __forceinline__ void half_exp_out_keep(Pack<__half>* yr, int packs, int t, int stride, float inv,
                                                  const uint64_t (&ex)[KP][Pack<__half>::N / 2]) {
    constexpr int PV = Pack<__half>::N;
    const uint64_t inv2 = f2pack(inv, inv);
#pragma unroll
    for (int k = 0; k < KP; ++k) {
        const int p = t + k * stride;
        if (p < packs) {
            Pack<__half> o;
            __half2* oh = reinterpret_cast<__half2*>(o.v);
#pragma unroll
            for (int e = 0; e < PV / 2; ++e) {
                float z0, z1;
                f2unpack(mul2(ex[k][e], inv2), z0, z1);
                oh[e] = __floats2half2_rn(z0, z1);
            }
            yr[p] = o;
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

// Persistent CTAs, one row at a time held in registers with the next two rows
// in flight; the loop body is unrolled three times so the three row buffers
// change roles without register copies.
template <typename T, int NV>
__global__ void __launch_bounds__(256) k_softmax_rows(const T* __restrict__ x, T* __restrict__ y, int64_t rows,
                                                      int cols, int defer) {
    pdl_start(defer);
    constexpr int PV = Pack<T>::N;
    constexpr int E = NV * PV;
    __shared__ float sh_max[8], sh_sum[8];
    const int t = threadIdx.x, th = blockDim.x;
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
        float m0 = -INFINITY, m1 = -INFINITY;
#pragma unroll
        for (int k = 0; k < E; k += 2) {
            m0 = max_nan(m0, v[k]);
            m1 = max_nan(m1, v[k + 1]);
        }
        const float m = block_combine<true>(max_nan(m0, m1), sh_max);
        float s0 = 0.0f, s1 = 0.0f;
        const float mk = __fmul_rn(m, 1.4426950408889634f);
#pragma unroll
        for (int k = 0; k < E; k += 2) {
            v[k] = row_exp<T>(v[k], m, mk);
            v[k + 1] = row_exp<T>(v[k + 1], m, mk);
            s0 = __fadd_rn(s0, v[k]);
            s1 = __fadd_rn(s1, v[k + 1]);
        }
        const float inv = __frcp_rn(block_combine<false>(__fadd_rn(s0, s1), sh_sum));
        Pack<T>* yr = reinterpret_cast<Pack<T>*>(y + r * cols);
#pragma unroll
        for (int i = 0; i < NV; ++i) {
            float z[PV];
#pragma unroll
            for (int e = 0; e < PV; ++e) z[e] = __fmul_rn(v[i * PV + e], inv);
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
// the max (interleaved partial maxima per lane -- binary16 rows as half2
// pairs, exact -- then the warp), the sum of exp(x - max) the same way, then
// the output.  binary32 rows keep exp(x - max) in the buffer between the sum
// and the output; binary16 rows recompute it (the same function in both
// passes, so the sum and the outputs agree).
template <typename T>
__device__ __forceinline__ float pack_max(const Pack<T>* xs, int packs, int lane, int stride = 32) {
    constexpr int PV = Pack<T>::N;
    if constexpr (sizeof(T) == 4) {
        float part[PV];
#pragma unroll
        for (int e = 0; e < PV; ++e) part[e] = -INFINITY;
#pragma unroll 4
        for (int p = lane; p < packs; p += stride) {
            const Pack<T> v = xs[p];
#pragma unroll
            for (int e = 0; e < PV; ++e) part[e] = max_nan(part[e], v.v[e]);
        }
        float m = part[0];
#pragma unroll
        for (int e = 1; e < PV; ++e) m = max_nan(m, part[e]);
        return m;
    } else {
        __half2 part[PV / 2];
#pragma unroll
        for (int e = 0; e < PV / 2; ++e) part[e] = __float2half2_rn(-INFINITY);
#pragma unroll 4
        for (int p = lane; p < packs; p += stride) {
            const Pack<T> v = xs[p];
            const __half2* h = reinterpret_cast<const __half2*>(v.v);
#pragma unroll
            for (int e = 0; e < PV / 2; ++e) part[e] = __hmax2_nan(part[e], h[e]);
        }
#pragma unroll
        for (int e = 1; e < PV / 2; ++e) part[0] = __hmax2_nan(part[0], part[e]);
        return max_nan(__low2float(part[0]), __high2float(part[0]));
    }
}

template <typename T>
__global__ void __launch_bounds__(rowpipe::kMaxWarps * 32, 1)
    k_softmax_pipe(const T* __restrict__ x, T* __restrict__ y, int64_t rows, int cols, int slots, int* status, int defer) {
    pdl_start(defer);
    constexpr int PV = Pack<T>::N;
    constexpr bool F32 = sizeof(T) == 4;
    extern __shared__ float4 sm_pipe_smem[];
    __shared__ uint64_t bars[rowpipe::kMaxWarps * rowpipe::kMaxSlots];
    unsigned char* ring = reinterpret_cast<unsigned char*>(sm_pipe_smem);
    const int packs = cols / PV, lane = threadIdx.x & 31;
    const bool ok = rowpipe::stream_rows(
        reinterpret_cast<const unsigned char*>(x), rows, static_cast<uint32_t>(cols * sizeof(T)), slots, ring, bars,
        wait_limit(status), [&](int64_t row, unsigned char* buf) {
            Pack<T>* xs = reinterpret_cast<Pack<T>*>(buf);
            float m = pack_max<T>(xs, packs, lane);
#pragma unroll
            for (int k = 16; k >= 1; k >>= 1) m = max_nan(m, __shfl_xor_sync(0xffffffffu, m, k));
            const float mk = __fmul_rn(m, 1.4426950408889634f);
            float s;
            if constexpr (F32) {
                float part[PV];
#pragma unroll
                for (int e = 0; e < PV; ++e) part[e] = 0.0f;
#pragma unroll 4
                for (int p = lane; p < packs; p += 32) {
                    Pack<T> v = xs[p];
#pragma unroll
                    for (int e = 0; e < PV; ++e) {
                        const float ex = row_exp<T>(to_f(v.v[e]), m, mk);
                        part[e] = __fadd_rn(part[e], ex);
                        from_f(ex, &v.v[e]);
                    }
                    xs[p] = v;
                }
                s = part[0];
#pragma unroll
                for (int e = 1; e < PV; ++e) s = __fadd_rn(s, part[e]);
            } else {
                s = half_exp_sum(xs, packs, lane, 32, mk);
            }
            const float inv = __frcp_rn(rowpipe::warp_sum(s));
            Pack<T>* yr = reinterpret_cast<Pack<T>*>(y + row * cols);
            if constexpr (F32) {
#pragma unroll 2
                for (int p = lane; p < packs; p += 32) {
                    const Pack<T> v = xs[p];
                    float z[PV];
#pragma unroll
                    for (int e = 0; e < PV; ++e) z[e] = __fmul_rn(to_f(v.v[e]), inv);
                    yr[p] = to_pack<T>(z);
                }
            } else {
                half_exp_out(xs, yr, packs, lane, 32, mk, inv);
            }
        });
    if (!ok && lane == 0) atomicExch(status, QSML_E_TIMEOUT);
    pdl_end(defer);
}

// Binary16 rows of 8-108 KiB and binary32 rows of 32-108 KiB: one CTA of TH
// threads per row, rows streamed through two shared-memory buffers
// (row_pipe.cuh, stream_rows_cta): the max, the sum of exp(x - max) and the
// output as three passes over the buffer, each thread striding over the row's
// 16-byte packs.
template <typename T, int TH>
__global__ void __launch_bounds__(TH) k_softmax_wide(const T* __restrict__ x, T* __restrict__ y, int64_t rows,
                                                      int cols, int* status, int defer) {
    pdl_start(defer);
    constexpr int PV = Pack<T>::N;
    constexpr bool F32 = sizeof(T) == 4;
    extern __shared__ float4 sm_wide_smem[];
    __shared__ uint64_t bars[2];
    __shared__ float s_max[32], s_sum[32];
    const int packs = cols / PV, t = threadIdx.x, th = blockDim.x;
    const bool ok = rowpipe::stream_rows_cta(
        reinterpret_cast<const unsigned char*>(x), rows, static_cast<uint32_t>(cols * sizeof(T)),
        reinterpret_cast<unsigned char*>(sm_wide_smem), bars, wait_limit(status),
        [&](int64_t row, unsigned char* buf) {
            Pack<T>* xs = reinterpret_cast<Pack<T>*>(buf);
            const float m = rowpipe::cta_combine<true>(pack_max<T>(xs, packs, t, th), s_max);
            const float mk = __fmul_rn(m, 1.4426950408889634f);
            // binary16 rows of at most KP packs per thread keep their exponentials
            constexpr int KP = 4;
            uint64_t ex[KP][Pack<__half>::N / 2];
            const bool keep = !F32 && packs <= KP * th;
            float s;
            if constexpr (F32) {
                float part[PV];
#pragma unroll
                for (int e = 0; e < PV; ++e) part[e] = 0.0f;
#pragma unroll 2
                for (int p = t; p < packs; p += th) {
                    Pack<T> v = xs[p];
#pragma unroll
                    for (int e = 0; e < PV; ++e) {
                        const float ex = row_exp<T>(to_f(v.v[e]), m, mk);
                        part[e] = __fadd_rn(part[e], ex);
                        from_f(ex, &v.v[e]);
                    }
                    xs[p] = v;
                }
                s = part[0];
#pragma unroll
                for (int e = 1; e < PV; ++e) s = __fadd_rn(s, part[e]);
            } else {
                s = keep ? half_exp_sum_keep<KP>(xs, packs, t, th, mk, ex) : half_exp_sum(xs, packs, t, th, mk);
            }
            const float inv = __frcp_rn(rowpipe::cta_combine<false>(s, s_sum));
            Pack<T>* yr = reinterpret_cast<Pack<T>*>(y + row * cols);
            if constexpr (F32) {
#pragma unroll 2
                for (int p = t; p < packs; p += th) {
                    const Pack<T> v = xs[p];
                    float z[PV];
#pragma unroll
                    for (int e = 0; e < PV; ++e) z[e] = __fmul_rn(to_f(v.v[e]), inv);
                    yr[p] = to_pack<T>(z);
                }
            } else if (keep) {
                half_exp_out_keep<KP>(yr, packs, t, th, inv, ex);
            } else {
                half_exp_out(xs, yr, packs, t, th, mk, inv);
            }
        });
    if (!ok && t == 0) atomicExch(status, QSML_E_TIMEOUT);
    pdl_end(defer);
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

// What a softmax launch reads (x) and writes (y), for overlap.
template <typename T>
Footprint sm_footprint(const T* x, const T* y, int64_t rows, int cols) {
    Footprint f;
    const size_t n = static_cast<size_t>(rows) * cols * sizeof(T);
    f.read(span_of(x, n)).write(span_of(y, n));
    return f;
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
    {
        const int defer = plan_launch(ctx, sm_footprint(x, y, rows, cols));
        const cudaError_t e = launch_pdl(k_softmax_rows<T, NV>, dim3(static_cast<unsigned>(grid)), dim3(th), 0,
                                         ctx->stream, x, y, rows, cols, defer);
        if (e != cudaSuccess) return check_cuda(ctx, e, "k_softmax_rows");
    }
    return after_launch(ctx, "k_softmax_rows");
}

template <typename T>
qsml_status_t launch_pipe(Context* ctx, const T* x, T* y, int64_t rows, int cols, const rowpipe::Plan& p) {
    static std::mutex mu;
    static size_t attr_set = 0;  // largest dynamic shared memory opted in so far
    {
        std::lock_guard<std::mutex> lk(mu);
        if (p.smem > 48 * 1024 && p.smem > attr_set) {
            QSML_TRY_STATUS(check_cuda(ctx,
                                       cudaFuncSetAttribute(k_softmax_pipe<T>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                                            static_cast<int>(p.smem)),
                                       "softmax: shared-memory attribute"));
            attr_set = p.smem;
        }
    }
    {
        const int defer = plan_launch(ctx, sm_footprint(x, y, rows, cols));
        const cudaError_t e = launch_pdl(k_softmax_pipe<T>, dim3(p.grid), dim3(p.warps * 32), p.smem, ctx->stream, x,
                                         y, rows, cols, p.slots, ctx->status, defer);
        if (e != cudaSuccess) return check_cuda(ctx, e, "k_softmax_pipe");
    }
    return after_launch(ctx, "k_softmax_pipe");
}

template <typename T, int TH>
qsml_status_t launch_wide_as(Context* ctx, const T* x, T* y, int64_t rows, int cols) {
    const size_t smem = 2 * static_cast<size_t>(cols) * sizeof(T);
    static std::mutex mu;
    static bool attr_set = false;
    int per_sm = 1;
    {
        std::lock_guard<std::mutex> lk(mu);
        if (!attr_set) {
            QSML_TRY_STATUS(check_cuda(ctx,
                                       cudaFuncSetAttribute(k_softmax_wide<T, TH>,
                                                            cudaFuncAttributeMaxDynamicSharedMemorySize,
                                                            static_cast<int>(2 * rowpipe::kWideMaxRowBytes)),
                                       "softmax: shared-memory attribute"));
            attr_set = true;
        }
        if (TH < 512) {
            // several CTAs per SM when their buffers and registers fit (one
            // occupancy query per row width)
            static std::unordered_map<size_t, int> per_sm_by_smem;
            auto it = per_sm_by_smem.find(smem);
            if (it == per_sm_by_smem.end()) {
                cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, k_softmax_wide<T, TH>, TH, smem);
                if (per_sm < 1) per_sm = 1;
                per_sm_by_smem[smem] = per_sm;
            } else {
                per_sm = it->second;
            }
        }
    }
    int64_t grid = static_cast<int64_t>(ctx->num_sms) * per_sm;
    if (grid > rows) grid = rows;
    const int defer = plan_launch(ctx, sm_footprint(x, y, rows, cols));
    const cudaError_t e = launch_pdl(k_softmax_wide<T, TH>, dim3(static_cast<unsigned>(grid)), dim3(TH), smem,
                                     ctx->stream, x, y, rows, cols, ctx->status, defer);
    if (e != cudaSuccess) return check_cuda(ctx, e, "k_softmax_wide");
    return after_launch(ctx, "k_softmax_wide");
}

// 128 threads per row up to 1024 packs, 256 for binary16 rows up to 52 KiB
// (at least two CTAs per SM), 512 beyond.
template <typename T>
qsml_status_t launch_wide(Context* ctx, const T* x, T* y, int64_t rows, int cols) {
    if (cols / Pack<T>::N <= 1024) return launch_wide_as<T, 128>(ctx, x, y, rows, cols);
    if constexpr (sizeof(T) == 2) {
        if (cols / Pack<T>::N <= rowpipe::kWide256MaxPacks) return launch_wide_as<T, 256>(ctx, x, y, rows, cols);
    }
    return launch_wide_as<T, 512>(ctx, x, y, rows, cols);
}

template <typename T>
qsml_status_t run_softmax(Context* ctx, const T* x, T* y, int64_t outer, int64_t k, int64_t inner) {
    constexpr int PV = Pack<T>::N;
    if (inner == 1) {
        const int64_t rows = outer, cols = k;
        const uint64_t row_bytes = static_cast<uint64_t>(cols) * sizeof(T);
        const bool wide_ok = row_bytes % 16 == 0 && row_bytes <= rowpipe::kWideMaxRowBytes && aligned16(x) &&
                             aligned16(y) && ctx->status;
        // binary16 rows from 8 KiB up: a CTA per row (X[16384,4096]: 5.5 TB/s
        // against 4.8 for a warp per row; 4 KiB rows run faster on a warp)
        if (sizeof(T) == 2 && wide_ok && row_bytes >= 8192 && rows >= ctx->num_sms)
            return launch_wide<T>(ctx, x, y, rows, static_cast<int>(cols));
        rowpipe::Plan plan;
        if (rowpipe::use_pipe(cols * sizeof(T), sizeof(T)) && aligned16(x) && aligned16(y) && ctx->status && cols <= INT32_MAX &&
            rows >= ctx->num_sms && rowpipe::plan(ctx, rows, static_cast<uint64_t>(cols) * sizeof(T), 0, &plan))
            return launch_pipe<T>(ctx, x, y, rows, static_cast<int>(cols), plan);
        const bool wide = rowpipe::use_wide(row_bytes, sizeof(T)) && wide_ok;
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
        if (wide) return launch_wide<T>(ctx, x, y, rows, static_cast<int>(cols));
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
