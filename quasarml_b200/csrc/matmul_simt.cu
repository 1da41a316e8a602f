// CUDA-core matmul: C[b] = A[b] * B[b], row-major, fp32 accumulate.
//
// Reference: Ops/LinAlg.cpp:84-158 (matmul_shader_blocked) accumulates
// acc = fma(A[r][k], B[k][c], acc) for k ascending.  This kernel keeps that
// exact order per output (one fma chain from k = 0 to K-1, no split-K, no
// zero padding in k), so fp32 results are bit-identical to the reference's
// arithmetic.  Tiles: 128x128 outputs per CTA, k-slices of 8 staged in
// shared memory (A transposed so both fragments are row reads), 8x8 outputs
// per thread, register prefetch of the next slice while computing this one.
// Used for QSML_MM_FP32_FFMA and as the fp16-input fallback for shapes the
// tensor-core kernel does not take.
#include "qsml_internal.cuh"

#include "matmul.cuh"

namespace qsml {
namespace {

constexpr int BM = 128, BN = 128, BK = 8, TM = 8, TN = 8;

__device__ __forceinline__ float ldf(const float* p) { return *p; }
__device__ __forceinline__ float ldf(const __half* p) { return __half2float(*p); }
__device__ __forceinline__ void stf(float* p, float v) { *p = v; }
__device__ __forceinline__ void stf(__half* p, float v) { *p = __float2half_rn(v); }

template <typename TI, typename TO>
__global__ void __launch_bounds__(256) k_matmul_simt(const TI* __restrict__ A, const TI* __restrict__ B,
                                                     TO* __restrict__ C, int M, int N, int K, int64_t lda,
                                                     int64_t ldb, int64_t sA, int64_t sB, int64_t sC) {
    __shared__ float As[2][BK][BM];
    __shared__ float Bs[2][BK][BN];
    const int tid = threadIdx.x;
    const int tx = tid % 16, ty = tid / 16;
    const int bz = blockIdx.z;
    A += bz * sA;
    B += bz * sB;
    C += bz * sC;
    const int row0 = blockIdx.y * BM, col0 = blockIdx.x * BN;

    // Each thread loads 4 elements of the A slice (128 x 8) and 4 of B (8 x 128).
    // A: thread -> (r = tid / 2, k = (tid % 2) * 4 + j); B: (k = tid / 32, c = (tid % 32) * 4 + j).
    const int ar = tid >> 1, ak = (tid & 1) * 4;
    const int bk = tid >> 5, bc = (tid & 31) * 4;
    float ra[4], rb[4];

    auto load_slice = [&](int k0) {
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            int r = row0 + ar, k = k0 + ak + j;
            ra[j] = (r < M && k < K) ? ldf(A + static_cast<int64_t>(r) * lda + k) : 0.0f;
        }
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            int k = k0 + bk, c = col0 + bc + j;
            rb[j] = (k < K && c < N) ? ldf(B + static_cast<int64_t>(k) * ldb + c) : 0.0f;
        }
    };
    auto store_slice = [&](int buf) {
#pragma unroll
        for (int j = 0; j < 4; ++j) As[buf][ak + j][ar] = ra[j];
#pragma unroll
        for (int j = 0; j < 4; ++j) Bs[buf][bk][bc + j] = rb[j];
    };

    float acc[TM][TN];
#pragma unroll
    for (int i = 0; i < TM; ++i)
#pragma unroll
        for (int j = 0; j < TN; ++j) acc[i][j] = 0.0f;

    const int nslices = (K + BK - 1) / BK;
    load_slice(0);
    store_slice(0);
    __syncthreads();
    for (int s = 0; s < nslices; ++s) {
        const int buf = s & 1;
        if (s + 1 < nslices) load_slice((s + 1) * BK);
        const int kn = K - s * BK < BK ? K - s * BK : BK;  // valid k in this slice
        if (kn == BK) {
#pragma unroll
            for (int kk = 0; kk < BK; ++kk) {
                float a[TM], b[TN];
#pragma unroll
                for (int i = 0; i < TM; i += 4) {
                    float4 v = *reinterpret_cast<const float4*>(&As[buf][kk][ty * 4 + i * 16]);
                    a[i] = v.x; a[i + 1] = v.y; a[i + 2] = v.z; a[i + 3] = v.w;
                }
#pragma unroll
                for (int j = 0; j < TN; j += 4) {
                    float4 v = *reinterpret_cast<const float4*>(&Bs[buf][kk][tx * 4 + j * 16]);
                    b[j] = v.x; b[j + 1] = v.y; b[j + 2] = v.z; b[j + 3] = v.w;
                }
#pragma unroll
                for (int i = 0; i < TM; ++i)
#pragma unroll
                    for (int j = 0; j < TN; ++j) acc[i][j] = __fmaf_rn(a[i], b[j], acc[i][j]);
            }
        } else {
            for (int kk = 0; kk < kn; ++kk) {
                float a[TM], b[TN];
#pragma unroll
                for (int i = 0; i < TM; i += 4) {
                    float4 v = *reinterpret_cast<const float4*>(&As[buf][kk][ty * 4 + i * 16]);
                    a[i] = v.x; a[i + 1] = v.y; a[i + 2] = v.z; a[i + 3] = v.w;
                }
#pragma unroll
                for (int j = 0; j < TN; j += 4) {
                    float4 v = *reinterpret_cast<const float4*>(&Bs[buf][kk][tx * 4 + j * 16]);
                    b[j] = v.x; b[j + 1] = v.y; b[j + 2] = v.z; b[j + 3] = v.w;
                }
#pragma unroll
                for (int i = 0; i < TM; ++i)
#pragma unroll
                    for (int j = 0; j < TN; ++j) acc[i][j] = __fmaf_rn(a[i], b[j], acc[i][j]);
            }
        }
        if (s + 1 < nslices) {
            store_slice(buf ^ 1);
        }
        __syncthreads();
    }
    // Thread (tx, ty) owns rows ty*4 + {0..3} + {0, 64} and cols tx*4 + {0..3} + {0, 64}.
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
