// Tensor-core matmul for fp16 inputs with fp32 accumulation on sm_100a:
// tcgen05.mma with the accumulator in tensor memory (TMEM), operands staged in
// shared memory by TMA (cp.async.bulk.tensor, no multicast).
//
// Reference: Ops::matmul (Ops/LinAlg.cpp:221-271) runs a SIMT shader with
// 16x16 workgroups and 4x4 register blocks; Ops::batch_matmul
// (LinAlg.cpp:273-290) is broken.  Here:
//   * C tile 128 x 256 per CTA, k-blocks of 64; one tcgen05.mma
//     (M=128, N=256, K=16, cta_group::1) per 16-wide k slice;
//   * A [M,K] row-major is K-major in shared memory, B [K,N] row-major is
//     MN-major (N contiguous); both use the 128-byte swizzle TMA writes;
//   * 4-stage ring of shared-memory buffers with full/empty mbarriers:
//     warp 0 (one lane) issues the TMA loads, warp 1 (one lane) issues the
//     MMAs and commits each stage back to the producer;
//   * two 256-column fp32 accumulators in TMEM (512 columns allocated): the
//     4 epilogue warps drain one (tcgen05.ld 32x32b -> registers ->
//     swizzled shared-memory staging -> TMA bulk-tensor store, clipped at the
//     matrix edges by the hardware) while the MMA warp fills the other;
//   * persistent CTAs (one per SM) walk the tiles in groups of 16 M-tiles so
//     concurrently running tiles share A and B panels in L2;
//   * every wait is bounded: on expiry the CTA records QSML_E_TIMEOUT in the
//     context's status word, lets its in-flight copies and MMAs finish
//     (again bounded), frees its TMEM and returns.
#include <cuda.h>
#include <cudaTypedefs.h>

#include "matmul.cuh"

namespace qsml {
namespace {

constexpr int BM = 128, BN = 256, BK = 64, STAGES = 4;
constexpr int A_STAGE_BYTES = BM * BK * 2;        // 16 KiB
constexpr int B_STAGE_BYTES = BK * BN * 2;        // 32 KiB
constexpr int B_BOX_BYTES = BK * 64 * 2;          // one 64-column TMA box: 8 KiB
constexpr int STAGE_BYTES = A_STAGE_BYTES + B_STAGE_BYTES;
constexpr int TMEM_COLS = 512;                    // 2 accumulators x 256 fp32 columns
constexpr int GROUP_M = 16;
constexpr int NUM_THREADS = 192;                  // warp 0 TMA, warp 1 MMA, warps 2-5 epilogue
constexpr long long WAIT_CYCLES = 2000000000LL;   // ~1 s at 2 GHz
constexpr int C_BOX_BYTES = 32 * 128;              // epilogue staging: 32 rows x 128 bytes
constexpr int C_STAGE_BYTES = 4 * 2 * C_BOX_BYTES;  // 4 epilogue warps x 2 buffers = 32 KiB
constexpr size_t SMEM_BYTES =
    size_t(STAGES) * STAGE_BYTES + C_STAGE_BYTES + 1024 /*align*/ + 256 /*barriers*/;

// Instruction descriptor: D f32, A/B f16, A K-major, B MN-major, N=256, M=128.
constexpr uint32_t IDESC = (1u << 4) | (0u << 7) | (0u << 10) | (0u << 15) | (1u << 16) |
                           (uint32_t(BN >> 3) << 17) | (uint32_t(BM >> 4) << 24);

struct TileMap {
    int tiles_m, tiles_n, batch;
    __device__ void decode(int t, int& b, int& mt, int& nt) const {
        const int per = tiles_m * tiles_n;
        b = t / per;
        const int r = t - b * per;
        const int group = r / (GROUP_M * tiles_n);
        const int first_m = group * GROUP_M;
        const int gm = min(GROUP_M, tiles_m - first_m);
        const int within = r - group * GROUP_M * tiles_n;
        mt = first_m + within % gm;
        nt = within / gm;
    }
};

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
    return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ void mbar_init(uint32_t bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(bar), "r"(count) : "memory");
}

__device__ __forceinline__ void mbar_expect_tx(uint32_t bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(bar), "r"(bytes) : "memory");
}

__device__ __forceinline__ void mbar_arrive(uint32_t bar) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(bar) : "memory");
}

__device__ __forceinline__ bool mbar_test(uint32_t bar, uint32_t parity) {
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

// Bounded wait for the phase of `bar` with parity `parity`.  Returns false
// (and raises the CTA's abort flag) if it does not complete in WAIT_CYCLES or
// another role already aborted.
__device__ __forceinline__ bool mbar_wait(uint32_t bar, uint32_t parity, volatile int* abort_flag) {
    if (mbar_test(bar, parity)) return true;
    const long long t0 = clock64();
    for (;;) {
        if (mbar_test(bar, parity)) return true;
        if (*abort_flag) return false;
        if (clock64() - t0 > WAIT_CYCLES) {
            *abort_flag = 1;
            return false;
        }
    }
}

__device__ __forceinline__ void tma_load_3d(uint32_t dst, const CUtensorMap* map, uint32_t bar, int c0, int c1,
                                            int c2) {
    asm volatile(
        "cp.async.bulk.tensor.3d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3, %4}], [%5];"
        ::"r"(dst), "l"(reinterpret_cast<uint64_t>(map)), "r"(c0), "r"(c1), "r"(c2), "r"(bar)
        : "memory");
}

// Shared-memory matrix descriptor, 128-byte swizzle, sm_100 version field.
__device__ __forceinline__ uint64_t smem_desc(uint32_t saddr, uint32_t lbo, uint32_t sbo) {
    uint64_t d = 0;
    d |= static_cast<uint64_t>((saddr & 0x3FFFFu) >> 4);
    d |= static_cast<uint64_t>((lbo >> 4) & 0x3FFFu) << 16;
    d |= static_cast<uint64_t>((sbo >> 4) & 0x3FFFu) << 32;
    d |= static_cast<uint64_t>(1) << 46;  // descriptor version for tcgen05
    d |= static_cast<uint64_t>(2) << 61;  // SWIZZLE_128B
    return d;
}

__device__ __forceinline__ void mma_f16(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc, uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}"
        ::"r"(d_tmem), "l"(adesc), "l"(bdesc), "r"(IDESC), "r"(accumulate)
        : "memory");
}

__device__ __forceinline__ void mma_commit(uint32_t bar) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(bar)
                 : "memory");
}

__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

// 32 consecutive fp32 columns of this thread's TMEM lane.
__device__ __forceinline__ void tmem_ld32(uint32_t taddr, uint32_t (&r)[32]) {
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x32.b32 "
        "{%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15, "
        "%16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31}, [%32];"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
          "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]),
          "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]),
          "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
        : "r"(taddr));
    asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
}

template <bool OUT_F16>
__global__ void __launch_bounds__(NUM_THREADS, 1)
    k_gemm_tc_f16(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                  const __grid_constant__ CUtensorMap tmC, int M, int N, int K, TileMap tm, int a_batched,
                  int b_batched, int* status) {
    extern __shared__ unsigned char smem_raw[];
    const uint32_t raw = smem_u32(smem_raw);
    const uint32_t base = (raw + 1023u) & ~1023u;  // swizzled tiles need 1024-byte alignment
    unsigned char* gbase = smem_raw + (base - raw);
    const uint32_t sA = base;
    const uint32_t sB = base + STAGES * A_STAGE_BYTES;
    const uint32_t sC_stage = base + STAGES * STAGE_BYTES;  // 1024-aligned: the swizzle needs it
    const uint32_t bars = sC_stage + C_STAGE_BYTES;
    // barrier layout: full[STAGES], empty[STAGES], tfull[2], tempty[2], drain
    auto full_bar = [&](int s) { return bars + 8u * s; };
    auto empty_bar = [&](int s) { return bars + 8u * (STAGES + s); };
    auto tfull_bar = [&](int a) { return bars + 8u * (2 * STAGES + a); };
    auto tempty_bar = [&](int a) { return bars + 8u * (2 * STAGES + 2 + a); };
    const uint32_t drain_bar = bars + 8u * (2 * STAGES + 4);
    unsigned char* gmisc = gbase + STAGES * STAGE_BYTES + C_STAGE_BYTES + 8 * (2 * STAGES + 5);
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(gmisc);
    volatile int* abort_flag = reinterpret_cast<volatile int*>(gmisc + 4);

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    if (threadIdx.x == 0) {
        for (int s = 0; s < STAGES; ++s) {
            mbar_init(full_bar(s), 1);
            mbar_init(empty_bar(s), 1);
        }
        for (int a = 0; a < 2; ++a) {
            mbar_init(tfull_bar(a), 1);
            mbar_init(tempty_bar(a), 4);  // one arrival per epilogue warp
        }
        mbar_init(drain_bar, 1);
        *abort_flag = 0;
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
        asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
    }
    if (warp == 1) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_slot)),
                     "r"(TMEM_COLS)
                     : "memory");
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem_base = *tmem_slot;

    const int total = tm.tiles_m * tm.tiles_n * tm.batch;
    const int num_kb = (K + BK - 1) / BK;

    if (warp == 0) {
        if (lane == 0) {
            // ---- TMA producer ----
            int stage = 0;
            uint32_t phase = 0;
            int issued[STAGES];
            for (int s = 0; s < STAGES; ++s) issued[s] = -1;
            bool ok = true;
            for (int t = blockIdx.x; t < total && ok; t += gridDim.x) {
                int b, mt, nt;
                tm.decode(t, b, mt, nt);
                const int ab = a_batched ? b : 0, bb = b_batched ? b : 0;
                for (int kb = 0; kb < num_kb; ++kb) {
                    if (!mbar_wait(empty_bar(stage), phase ^ 1u, abort_flag)) {
                        ok = false;
                        break;
                    }
                    mbar_expect_tx(full_bar(stage), STAGE_BYTES);
                    tma_load_3d(sA + stage * A_STAGE_BYTES, &tmA, full_bar(stage), kb * BK, mt * BM, ab);
#pragma unroll
                    for (int j = 0; j < BN / 64; ++j)
                        tma_load_3d(sB + stage * B_STAGE_BYTES + j * B_BOX_BYTES, &tmB, full_bar(stage),
                                    nt * BN + j * 64, kb * BK, bb);
                    issued[stage] = static_cast<int>(phase);
                    if (++stage == STAGES) {
                        stage = 0;
                        phase ^= 1u;
                    }
                }
            }
            // Let every copy this thread started land before the CTA can exit.
            for (int s = 0; s < STAGES; ++s) {
                if (issued[s] < 0) continue;
                const long long t0 = clock64();
                while (!mbar_test(full_bar(s), static_cast<uint32_t>(issued[s])) && clock64() - t0 < WAIT_CYCLES) {
                }
            }
        }
    } else if (warp == 1) {
        if (lane == 0) {
            // ---- MMA issuer ----
            int stage = 0;
            uint32_t phase = 0;
            int acc = 0;
            uint32_t acc_phase = 0;
            bool ok = true;
            for (int t = blockIdx.x; t < total && ok; t += gridDim.x) {
                if (!mbar_wait(tempty_bar(acc), acc_phase ^ 1u, abort_flag)) break;
                tc_fence_after();
                const uint32_t d_tmem = tmem_base + static_cast<uint32_t>(acc * BN);
                for (int kb = 0; kb < num_kb; ++kb) {
                    if (!mbar_wait(full_bar(stage), phase, abort_flag)) {
                        ok = false;
                        break;
                    }
                    tc_fence_after();
                    const uint32_t a0 = sA + stage * A_STAGE_BYTES;
                    const uint32_t b0 = sB + stage * B_STAGE_BYTES;
#pragma unroll
                    for (int k = 0; k < BK / 16; ++k) {
                        // A: K-major, advance 16 fp16 = 32 bytes inside the 128-byte swizzle row.
                        const uint64_t ad = smem_desc(a0 + k * 32, 16, 1024);
                        // B: MN-major, advance 16 k-rows of 128 bytes; 64-column chunks are 8 KiB apart.
                        const uint64_t bd = smem_desc(b0 + k * 16 * 128, B_BOX_BYTES, 1024);
                        mma_f16(d_tmem, ad, bd, (kb > 0 || k > 0) ? 1u : 0u);
                    }
                    mma_commit(empty_bar(stage));  // stage free once these MMAs have read it
                    if (++stage == STAGES) {
                        stage = 0;
                        phase ^= 1u;
                    }
                }
                if (!ok) break;
                mma_commit(tfull_bar(acc));  // accumulator ready for the epilogue
                if (++acc == 2) {
                    acc = 0;
                    acc_phase ^= 1u;
                }
            }
            // Every MMA issued above completes before TMEM is freed.
            mma_commit(drain_bar);
            const long long t0 = clock64();
            while (!mbar_test(drain_bar, 0) && clock64() - t0 < WAIT_CYCLES) {
            }
        }
    } else {
        // ---- epilogue: warps 2..5 own TMEM lanes 32*(warp%4) .. +31 ----
        const int quarter = warp & 3;
        int acc = 0;
        uint32_t acc_phase = 0;
        for (int t = blockIdx.x; t < total; t += gridDim.x) {
            // one lane waits, the warp follows its verdict (tcgen05.ld needs
            // the whole warp converged)
            int ready = 0;
            if (lane == 0) ready = mbar_wait(tfull_bar(acc), acc_phase, abort_flag) ? 1 : 0;
            ready = __shfl_sync(0xffffffffu, ready, 0);
            if (!ready) break;
            tc_fence_after();
            int b, mt, nt;
            tm.decode(t, b, mt, nt);
            const int row0 = mt * BM + quarter * 32;  // first of this warp's 32 rows
            const uint32_t taddr = tmem_base + (static_cast<uint32_t>(quarter * 32) << 16) + static_cast<uint32_t>(acc * BN);
            // Each chunk is 32 rows x 128 bytes (32 fp32 or 64 fp16 columns):
            // lane = row; the row goes to a staging buffer in the 128-byte
            // swizzle the C tensor map expects, then one TMA store writes the
            // box (clipped at the matrix edges by the hardware).
            constexpr int CHUNK_COLS = OUT_F16 ? 64 : 32;
            for (int c0 = 0; c0 < BN; c0 += CHUNK_COLS) {
                // Past the last column nothing is stored; stopping here also
                // keeps "one bulk group per buffer use" true, which the
                // wait_group.read accounting below relies on.
                if (nt * BN + c0 >= N) break;
                uint32_t words[32];  // the row's 128 bytes
                if (OUT_F16) {
                    uint32_t r0[32], r1[32];
                    tmem_ld32(taddr + c0, r0);
                    tmem_ld32(taddr + c0 + 32, r1);
#pragma unroll
                    for (int i = 0; i < 16; ++i) {
                        __half2 h = __floats2half2_rn(__uint_as_float(r0[2 * i]), __uint_as_float(r0[2 * i + 1]));
                        words[i] = *reinterpret_cast<uint32_t*>(&h);
                        __half2 g = __floats2half2_rn(__uint_as_float(r1[2 * i]), __uint_as_float(r1[2 * i + 1]));
                        words[16 + i] = *reinterpret_cast<uint32_t*>(&g);
                    }
                } else {
                    tmem_ld32(taddr + c0, words);
                }
                const int buf = (c0 / CHUNK_COLS) & 1;
                const uint32_t stage = sC_stage + static_cast<uint32_t>((quarter * 2 + buf) * C_BOX_BYTES);
                // the store issued from this buffer two chunks ago has read it
                if (lane == 0) asm volatile("cp.async.bulk.wait_group.read 1;" ::: "memory");
                __syncwarp();
#pragma unroll
                for (int j = 0; j < 8; ++j) {
                    const uint32_t a = stage + lane * 128 + ((j ^ (lane & 7)) << 4);
                    asm volatile("st.shared.v4.b32 [%0], {%1, %2, %3, %4};" ::"r"(a), "r"(words[4 * j]),
                                 "r"(words[4 * j + 1]), "r"(words[4 * j + 2]), "r"(words[4 * j + 3])
                                 : "memory");
                }
                asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
                __syncwarp();
                const int col = nt * BN + c0;
                if (lane == 0 && row0 < M && col < N) {
                    asm volatile(
                        "cp.async.bulk.tensor.3d.global.shared::cta.bulk_group [%0, {%1, %2, %3}], [%4];"
                        ::"l"(reinterpret_cast<uint64_t>(&tmC)), "r"(col), "r"(row0), "r"(b), "r"(stage)
                        : "memory");
                    asm volatile("cp.async.bulk.commit_group;" ::: "memory");
                }
            }
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(tempty_bar(acc));
            if (++acc == 2) {
                acc = 0;
                acc_phase ^= 1u;
            }
        }
        // every TMA store has finished before the CTA can exit
        if (lane == 0) asm volatile("cp.async.bulk.wait_group 0;" ::: "memory");
        __syncwarp();
    }
    tc_fence_before();
    __syncthreads();
    if (*abort_flag && threadIdx.x == 0) atomicExch(status, QSML_E_TIMEOUT);
    if (warp == 1) {
        tc_fence_after();
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem_base), "r"(TMEM_COLS)
                     : "memory");
    }
}

// ---------------------------------------------------------------------------
// Host side
// ---------------------------------------------------------------------------
PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
    static PFN_cuTensorMapEncodeTiled_v12000 fn = [] {
        void* p = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) != cudaSuccess ||
            q != cudaDriverEntryPointSuccess) {
            cudaGetLastError();
            return static_cast<PFN_cuTensorMapEncodeTiled_v12000>(nullptr);
        }
        return reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
    }();
    return fn;
}

// 3-D fp16 tensor map: dims {inner, outer, batch}, 128-byte swizzle.
bool make_map(CUtensorMap* map, const void* ptr, uint64_t inner, uint64_t outer, uint64_t batch, uint64_t row_bytes,
              uint64_t batch_bytes, uint32_t box_inner, uint32_t box_outer,
              CUtensorMapDataType dt = CU_TENSOR_MAP_DATA_TYPE_FLOAT16) {
    auto fn = encode_fn();
    if (!fn) return false;
    cuuint64_t dims[3] = {inner, outer, batch};
    cuuint64_t strides[2] = {row_bytes, batch_bytes};
    cuuint32_t box[3] = {box_inner, box_outer, 1};
    cuuint32_t estr[3] = {1, 1, 1};
    CUresult r = fn(map, dt, 3, const_cast<void*>(ptr), dims, strides, box, estr,
                    CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                    CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    return r == CUDA_SUCCESS;
}

}  // namespace

qsml_status_t matmul_tc_f16(Context* ctx, const MatmulArgs& g, bool out_f16) {
    // What the kernel takes: 16-byte aligned operands and row strides (TMA),
    // N a multiple of 8 (vector stores), and a status word for timeouts.
    const bool shapes_ok = g.K % 8 == 0 && g.N % 8 == 0 && g.lda % 8 == 0 && g.ldb % 8 == 0 && g.sA % 8 == 0 &&
                           g.sB % 8 == 0 && aligned16(g.A) && aligned16(g.B) && aligned16(g.C) && g.M > 0 &&
                           g.N > 0 && g.K > 0;
    if (!shapes_ok) return QSML_E_UNSUPPORTED;
    if (!ctx->status) return QSML_E_UNSUPPORTED;
    const uint64_t a_batch = g.sA ? static_cast<uint64_t>(g.batch) : 1;
    const uint64_t b_batch = g.sB ? static_cast<uint64_t>(g.batch) : 1;
    CUtensorMap tmA, tmB, tmC;
    // C: 128-byte wide boxes of 32 rows (32 fp32 or 64 fp16 columns), written
    // by the epilogue from swizzled shared-memory staging.
    const uint64_t c_es = out_f16 ? 2 : 4;
    if (!make_map(&tmA, g.A, g.K, g.M, a_batch, g.lda * 2, (g.sA ? g.sA : g.lda * g.M) * 2, BK, BM) ||
        !make_map(&tmB, g.B, g.N, g.K, b_batch, g.ldb * 2, (g.sB ? g.sB : g.ldb * g.K) * 2, 64, BK) ||
        !make_map(&tmC, g.C, g.N, g.M, g.batch, g.N * c_es, g.M * g.N * c_es, static_cast<uint32_t>(128 / c_es), 32,
                  out_f16 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT32))
        return QSML_E_UNSUPPORTED;
    // The dynamic shared-memory opt-in is per device; set it once each.
    static std::mutex attr_mu;
    static uint64_t attr_done[2] = {0, 0};
    {
        std::lock_guard<std::mutex> lk(attr_mu);
        const uint64_t bit = uint64_t(1) << (ctx->device & 63);
        if (!(attr_done[out_f16] & bit)) {
            cudaError_t e = out_f16 ? cudaFuncSetAttribute(k_gemm_tc_f16<true>,
                                                           cudaFuncAttributeMaxDynamicSharedMemorySize,
                                                           static_cast<int>(SMEM_BYTES))
                                    : cudaFuncSetAttribute(k_gemm_tc_f16<false>,
                                                           cudaFuncAttributeMaxDynamicSharedMemorySize,
                                                           static_cast<int>(SMEM_BYTES));
            if (e != cudaSuccess) return check_cuda(ctx, e, "matmul: shared-memory attribute");
            attr_done[out_f16] |= bit;
        }
    }
    TileMap tm;
    tm.tiles_m = static_cast<int>((g.M + BM - 1) / BM);
    tm.tiles_n = static_cast<int>((g.N + BN - 1) / BN);
    tm.batch = static_cast<int>(g.batch);
    const int64_t total = static_cast<int64_t>(tm.tiles_m) * tm.tiles_n * tm.batch;
    int grid = static_cast<int>(total < ctx->num_sms ? total : ctx->num_sms);
    if (out_f16)
        k_gemm_tc_f16<true><<<grid, NUM_THREADS, SMEM_BYTES, ctx->stream>>>(
            tmA, tmB, tmC, static_cast<int>(g.M), static_cast<int>(g.N), static_cast<int>(g.K), tm,
            g.sA ? 1 : 0, g.sB ? 1 : 0, ctx->status);
    else
        k_gemm_tc_f16<false><<<grid, NUM_THREADS, SMEM_BYTES, ctx->stream>>>(
            tmA, tmB, tmC, static_cast<int>(g.M), static_cast<int>(g.N), static_cast<int>(g.K), tm,
            g.sA ? 1 : 0, g.sB ? 1 : 0, ctx->status);
    return after_launch(ctx, "k_gemm_tc_f16");
}

}  // namespace qsml
