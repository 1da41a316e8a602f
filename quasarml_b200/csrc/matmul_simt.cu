// CUDA-core matmul: C[b] = A[b] * B[b], row-major, fp32 accumulate.
//
// Reference: Ops/LinAlg.cpp:84-158 (matmul_shader_blocked) accumulates
// acc = fma(A[r][k], B[k][c], acc) for k ascending.  This kernel keeps that
// exact order per output (one fma chain from k = 0 to K-1, no split-K, no
// zero padding in k), so fp32 results are bit-identical to the reference's
// arithmetic.  Tiles: 128x128 outputs per CTA, k-slices of 16 staged in
// shared memory (A transposed so both fragments are row reads), 8x8 outputs
// per thread.  The next slice's global loads are in flight while this one is
// computed (16-byte loads for interior tiles of binary32 operands), and each
// thread's fragments for step kk+1 are read from shared memory while the 64
// fmas of step kk issue.  The fmas are issued two at a time as sm_100's packed
// fma.rn.f32x2 (outputs (i, 2j) and (i, 2j+1) in one instruction, A's value in
// both lanes): each lane is one IEEE fma rounded to nearest even, exactly what
// fmaf does, so the per-output chain and its bits are unchanged while the
// kernel, issue-bound with scalar fmas, issues a third fewer instructions.
// Used for QSML_MM_FP32_FFMA and as the fp16-input fallback for shapes the
// tensor-core kernel does not take.
#include "qsml_internal.cuh"

#include "matmul.cuh"

namespace qsml {
namespace {

constexpr int BM = 128, BN = 128, BK = 16, TM = 8, TN = 8;

// Two fp32 values as one 64-bit operand of a packed instruction (lo = first).
__device__ __forceinline__ uint64_t pack2(float lo, float hi) {
    uint64_t r;
    asm("mov.b64 %0, {%1, %2};" : "=l"(r) : "f"(lo), "f"(hi));
    return r;
}
__device__ __forceinline__ void unpack2(uint64_t v, float& lo, float& hi) {
    asm("mov.b64 {%0, %1}, %2;" : "=f"(lo), "=f"(hi) : "l"(v));
}
// d = a * b + d in each of the two lanes, each lane rounded once to nearest
// even (per lane the operation of fmaf).
__device__ __forceinline__ void fma2(uint64_t& d, uint64_t a, uint64_t b) {
    asm("fma.rn.f32x2 %0, %1, %2, %0;" : "+l"(d) : "l"(a), "l"(b));
}

__device__ __forceinline__ float ldf(const float* p) { return *p; }
__device__ __forceinline__ float ldf(const __half* p) { return __half2float(*p); }
__device__ __forceinline__ void stf(float* p, float v) { *p = v; }
__device__ __forceinline__ void stf(__half* p, float v) { *p = __float2half_rn(v); }

template <typename TI, typename TO>
__global__ void __launch_bounds__(256, 2) k_matmul_simt(const TI* __restrict__ A, const TI* __restrict__ B,
                                                        TO* __restrict__ C, int M, int N, int K, int64_t lda,
                                                        int64_t ldb, int64_t sA, int64_t sB, int64_t sC) {
    __shared__ __align__(16) float As[2][BK][BM];
    __shared__ __align__(16) float Bs[2][BK][BN];
    const int tid = threadIdx.x;
    // Threads as a 16 x 16 grid (tx, ty); each warp is a 4 (ty) x 8 (tx) block of
    // it, so a warp's fragment reads below are 64 bytes of A and 128 bytes of B:
    // one shared-memory wavefront each.
    const int tx = 8 * ((tid >> 5) & 1) + (tid & 7), ty = 4 * (tid >> 6) + ((tid >> 3) & 3);
    const int bz = blockIdx.z;
    A += bz * sA;
    B += bz * sB;
    C += bz * sC;
    const int row0 = blockIdx.y * BM, col0 = blockIdx.x * BN;

    // Loads of a k-slice: A (128 x 16) thread -> row tid / 2, k (tid % 2) * 8 + 0..7;
    // B (16 x 128) thread -> k tid / 16, columns (tid % 16) * 8 + 0..7.
    const int ar = tid >> 1, ak = (tid & 1) * 8;
    const int bk = tid >> 4, bc = (tid & 15) * 8;
    // Interior tiles of binary32 operands with 16-byte aligned rows take
    // vector loads; everything else loads element by element with bounds.
    bool vec = false;
    if constexpr (sizeof(TI) == 4)
        vec = row0 + BM <= M && col0 + BN <= N && lda % 4 == 0 && ldb % 4 == 0 &&
              ((reinterpret_cast<uintptr_t>(A) | reinterpret_cast<uintptr_t>(B)) & 15u) == 0;
    float ra[8], rb[8];

    auto load_slice = [&](int k0) {
        if constexpr (sizeof(TI) == 4) {
            if (vec && k0 + BK <= K) {
                const float4* pa = reinterpret_cast<const float4*>(A + static_cast<int64_t>(row0 + ar) * lda + k0 + ak);
                const float4 a0 = pa[0], a1 = pa[1];
                const float4* pb = reinterpret_cast<const float4*>(B + static_cast<int64_t>(k0 + bk) * ldb + col0 + bc);
                const float4 b0 = pb[0], b1 = pb[1];
                ra[0] = a0.x; ra[1] = a0.y; ra[2] = a0.z; ra[3] = a0.w;
                ra[4] = a1.x; ra[5] = a1.y; ra[6] = a1.z; ra[7] = a1.w;
                rb[0] = b0.x; rb[1] = b0.y; rb[2] = b0.z; rb[3] = b0.w;
                rb[4] = b1.x; rb[5] = b1.y; rb[6] = b1.z; rb[7] = b1.w;
                return;
            }
        }
#pragma unroll
        for (int j = 0; j < 8; ++j) {
            const int r = row0 + ar, k = k0 + ak + j;
            ra[j] = (r < M && k < K) ? ldf(A + static_cast<int64_t>(r) * lda + k) : 0.0f;
        }
#pragma unroll
        for (int j = 0; j < 8; ++j) {
            const int k = k0 + bk, c = col0 + bc + j;
            rb[j] = (k < K && c < N) ? ldf(B + static_cast<int64_t>(k) * ldb + c) : 0.0f;
        }
    };
    auto store_slice = [&](int buf) {
#pragma unroll
        for (int j = 0; j < 8; ++j) As[buf][ak + j][ar] = ra[j];
        *reinterpret_cast<float4*>(&Bs[buf][bk][bc]) = make_float4(rb[0], rb[1], rb[2], rb[3]);
        *reinterpret_cast<float4*>(&Bs[buf][bk][bc + 4]) = make_float4(rb[4], rb[5], rb[6], rb[7]);
    };
    // Thread (tx, ty) owns rows ty*4 + {0..3} + {0, 64} and columns tx*4 + {0..3} + {0, 64}.
    auto load_frag = [&](int buf, int kk, float* a, float* b) {
        const float4 a0 = *reinterpret_cast<const float4*>(&As[buf][kk][ty * 4]);
        const float4 a1 = *reinterpret_cast<const float4*>(&As[buf][kk][ty * 4 + 64]);
        const float4 b0 = *reinterpret_cast<const float4*>(&Bs[buf][kk][tx * 4]);
        const float4 b1 = *reinterpret_cast<const float4*>(&Bs[buf][kk][tx * 4 + 64]);
        a[0] = a0.x; a[1] = a0.y; a[2] = a0.z; a[3] = a0.w; a[4] = a1.x; a[5] = a1.y; a[6] = a1.z; a[7] = a1.w;
        b[0] = b0.x; b[1] = b0.y; b[2] = b0.z; b[3] = b0.w; b[4] = b1.x; b[5] = b1.y; b[6] = b1.z; b[7] = b1.w;
    };

    // acc2[i][j] holds outputs (i, 2j) and (i, 2j+1) of the thread's 8 x 8.
    uint64_t acc2[TM][TN / 2];
#pragma unroll
    for (int i = 0; i < TM; ++i)
#pragma unroll
        for (int j = 0; j < TN / 2; ++j) acc2[i][j] = 0;  // both lanes +0.0f
    // One k step: acc(i, c) = fma(a[i], b[c], acc(i, c)) for the 8 x 8 outputs.
    auto step = [&](const float* a, const float* b) {
        uint64_t b2[TN / 2];
#pragma unroll
        for (int j = 0; j < TN / 2; ++j) b2[j] = pack2(b[2 * j], b[2 * j + 1]);
#pragma unroll
        for (int i = 0; i < TM; ++i) {
            const uint64_t a2 = pack2(a[i], a[i]);
#pragma unroll
            for (int j = 0; j < TN / 2; ++j) fma2(acc2[i][j], a2, b2[j]);
        }
    };

    const int nslices = (K + BK - 1) / BK;
    load_slice(0);
    store_slice(0);
    __syncthreads();
    for (int s = 0; s < nslices; ++s) {
        const int buf = s & 1;
        if (s + 1 < nslices) load_slice((s + 1) * BK);
        const int kn = K - s * BK < BK ? K - s * BK : BK;  // valid k in this slice
        if (kn == BK) {
            float fa[2][TM], fb[2][TN];
            load_frag(buf, 0, fa[0], fb[0]);
#pragma unroll
            for (int kk = 0; kk < BK; ++kk) {
                if (kk + 1 < BK) load_frag(buf, kk + 1, fa[(kk + 1) & 1], fb[(kk + 1) & 1]);
                step(fa[kk & 1], fb[kk & 1]);
            }
        } else {
            // the last, partial slice: only the valid k (no fma with padding)
            for (int kk = 0; kk < kn; ++kk) {
                float a[TM], b[TN];
                load_frag(buf, kk, a, b);
                step(a, b);
            }
        }
        if (s + 1 < nslices) store_slice(buf ^ 1);
        __syncthreads();
    }
    float acc[TM][TN];
#pragma unroll
    for (int i = 0; i < TM; ++i)
#pragma unroll
        for (int j = 0; j < TN / 2; ++j) unpack2(acc2[i][j], acc[i][2 * j], acc[i][2 * j + 1]);
#pragma unroll
    for (int i = 0; i < TM; ++i) {
        const int r = row0 + ty * 4 + (i & 3) + (i >> 2) * 64;
        if (r >= M) continue;
#pragma unroll
        for (int j = 0; j < TN; ++j) {
            const int c = col0 + tx * 4 + (j & 3) + (j >> 2) * 64;
            if (c < N) stf(C + static_cast<int64_t>(r) * N + c, acc[i][j]);
        }
    }
}

}  // namespace

template <typename TI, typename TO>
qsml_status_t matmul_simt(Context* ctx, const MatmulArgs& g) {
    dim3 grid(static_cast<unsigned>((g.N + BN - 1) / BN), static_cast<unsigned>((g.M + BM - 1) / BM),
              static_cast<unsigned>(g.batch));
    k_matmul_simt<TI, TO><<<grid, 256, 0, ctx->stream>>>(
        static_cast<const TI*>(g.A), static_cast<const TI*>(g.B), static_cast<TO*>(g.C), static_cast<int>(g.M),
        static_cast<int>(g.N), static_cast<int>(g.K), g.lda, g.ldb, g.sA, g.sB, g.sC);
    return after_launch(ctx, "k_matmul_simt");
}

template qsml_status_t matmul_simt<float, float>(Context*, const MatmulArgs&);
template qsml_status_t matmul_simt<__half, float>(Context*, const MatmulArgs&);
template qsml_status_t matmul_simt<__half, __half>(Context*, const MatmulArgs&);

}  // namespace qsml
