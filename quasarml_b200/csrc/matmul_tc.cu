// Tensor-core matmul on sm_100a: tcgen05.mma with the accumulator in tensor
// memory (TMEM), operands staged in shared memory by TMA (cp.async.bulk.tensor,
// every CTA loading its own tiles), results written by TMA bulk-tensor stores.
//
// Reference: Ops::matmul (Ops/LinAlg.cpp:221-271) runs a SIMT shader with
// 16x16 workgroups and 4x4 register blocks; Ops::batch_matmul
// (LinAlg.cpp:273-290) is broken.  Two configurations share one kernel:
//   * CfgF16  -- fp16 A/B, fp32 accumulate: C tile 128 x 256, k-blocks of 64,
//                one tcgen05.mma (kind::f16, M=128, N=256, K=16) per 16-wide
//                k slice, 4-stage ring;
//   * Cfg3xTF32 -- fp32 A/B as three tf32 products (A = Ahi + Alo,
//                B = Bhi + Blo; Ahi*Bhi + Ahi*Blo + Alo*Bhi, the Alo*Blo term
//                is below fp32 resolution), C tile 128 x 128, k-blocks of 32,
//                three kind::tf32 MMAs (K=8) per 8-wide k slice, 3-stage ring.
// A third kernel, k_gemm_tc2, runs fp16 on pairs of SMs (tcgen05 cta_group::2,
// C tile 256 x 256); it is described where it is defined.
// Common structure:
//   * A [M,K] row-major is K-major in shared memory, B [K,N] row-major is
//     MN-major (N contiguous); both use a 128-byte swizzle written by TMA
//     (16-byte units, except MN-major tf32 B, which needs 32-byte units);
//   * full/empty mbarriers per stage: warp 0 (one lane) issues the TMA loads,
//     warp 1 (one lane) issues the MMAs and commits each stage back;
//   * two fp32 accumulators in TMEM: the 4 epilogue warps drain one
//     (tcgen05.ld 32x32b -> registers -> swizzled shared-memory staging ->
//     TMA bulk-tensor store, clipped at the matrix edges by the hardware)
//     while the MMA warp fills the other;
//   * persistent CTAs (one per SM) walk the tiles in groups of 16 M-tiles so
//     concurrently running tiles share A and B panels in L2;
//   * every wait is bounded: on expiry the CTA records QSML_E_TIMEOUT in the
//     context's status word, lets its in-flight copies and MMAs finish
//     (again bounded), frees its TMEM and returns.
#include <cuda.h>
#include <cudaTypedefs.h>

#include <cstdlib>

#include "matmul.cuh"

namespace qsml {
namespace {

constexpr int BM = 128;
constexpr int GROUP_M = 16;
constexpr int NUM_THREADS = 192;                    // warp 0 TMA, warp 1 MMA, warps 2-5 epilogue
constexpr long long WAIT_CYCLES = kDefaultWaitCycles;  // ~1 s at 2 GHz
constexpr int C_BOX_BYTES = 32 * 128;               // epilogue staging: 32 rows x 128 bytes
constexpr int C_STAGE_BYTES = 4 * 2 * C_BOX_BYTES;  // 4 epilogue warps x 2 buffers = 32 KiB

// Instruction descriptor: D f32, A/B format, A K-major, B MN-major, N, M=128.
constexpr uint32_t make_idesc(uint32_t ab_format, int n) {
    return (1u << 4) | (ab_format << 7) | (ab_format << 10) | (0u << 15) | (1u << 16) |
           (uint32_t(n >> 3) << 17) | (uint32_t(BM >> 4) << 24);
}

// Shared-memory descriptor layout types (bits 61-63 of the descriptor).
constexpr uint32_t DESC_SW128 = 2;         // 16-byte units swizzled across 8 rows of 128 bytes
constexpr uint32_t DESC_SW128_BASE32 = 1;  // 32-byte units swizzled across 4 rows of 128 bytes

// B is MN-major.  For 16-bit types it uses the ordinary 128-byte swizzle
// (8-row atoms, k groups 1024 bytes apart); MN-major 32-bit (tf32) operands
// only accept the 128-byte swizzle with 32-byte units, whose atoms are 4
// rows, so k groups of 4 rows are 512 bytes apart.  TMA writes the matching
// pattern with CU_TENSOR_MAP_SWIZZLE_128B_ATOM_32B.
struct CfgF16 {
    static constexpr bool TF32 = false;
    static constexpr int BN = 256, BK = 64, STAGES = 4, ESIZE = 2;
    static constexpr int NA = 1, NB = 1;            // A and B tiles per stage
    static constexpr int MMA_K = 16;
    static constexpr uint32_t IDESC = make_idesc(0 /*f16*/, BN);
    static constexpr uint32_t B_DESC_LAYOUT = DESC_SW128, B_SBO = 1024;
    static constexpr CUtensorMapSwizzle B_SWIZZLE = CU_TENSOR_MAP_SWIZZLE_128B;
};

struct Cfg3xTF32 {
    static constexpr bool TF32 = true;
    static constexpr int BN = 128, BK = 32, STAGES = 3, ESIZE = 4;
    static constexpr int NA = 2, NB = 2;            // hi and lo parts of A and of B
    static constexpr int MMA_K = 8;
    static constexpr uint32_t IDESC = make_idesc(2 /*tf32*/, BN);
    static constexpr uint32_t B_DESC_LAYOUT = DESC_SW128_BASE32, B_SBO = 512;
    static constexpr CUtensorMapSwizzle B_SWIZZLE = CU_TENSOR_MAP_SWIZZLE_128B_ATOM_32B;
};

template <class Cfg> struct Layout {
    static constexpr int ROW_ELEMS = 128 / Cfg::ESIZE;             // one 128-byte swizzle row
    static constexpr int A_TILE = BM * Cfg::BK * Cfg::ESIZE;       // K-major: BM rows of 128 B
    static constexpr int B_BOX = Cfg::BK * 128;                    // MN-major: BK rows of 128 B
    static constexpr int B_BOXES = Cfg::BN / ROW_ELEMS;
    static constexpr int B_TILE = B_BOXES * B_BOX;
    static constexpr int STAGE = Cfg::NA * A_TILE + Cfg::NB * B_TILE;
    static constexpr int TMEM_COLS = 2 * Cfg::BN;                  // double-buffered accumulator
    static constexpr size_t SMEM = size_t(Cfg::STAGES) * STAGE + C_STAGE_BYTES + 1024 /*align*/ + 256 /*bars*/;
    static_assert(Cfg::BK * Cfg::ESIZE == 128, "one k-block is one 128-byte swizzle row of A");
    static_assert(SMEM <= 232448, "shared memory budget");
};

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

__device__ __forceinline__ bool mbar_probe(uint32_t bar, uint32_t parity) {  // never suspends
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

// Bounded wait for the phase of `bar` with parity `parity`.  Returns false
// (and raises the CTA's abort flag) if it does not complete in `limit` cycles
// or another role already aborted.
__device__ __forceinline__ bool mbar_wait(uint32_t bar, uint32_t parity, volatile int* abort_flag,
                                          long long limit) {
    // A lowered limit decides alone: poll with test_wait, which never
    // suspends (try_wait may suspend the thread for a hardware-chosen time).
    const bool short_limit = limit < WAIT_CYCLES;
    if (!short_limit && mbar_test(bar, parity)) return true;
    const long long t0 = clock64();
    for (;;) {
        if (short_limit ? mbar_probe(bar, parity) : mbar_test(bar, parity)) return true;
        if (*abort_flag) return false;
        if (clock64() - t0 > limit) {
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

// Shared-memory matrix descriptor (sm_100 version field) for a swizzled layout.
__device__ __forceinline__ uint64_t smem_desc(uint32_t saddr, uint32_t lbo, uint32_t sbo,
                                              uint32_t layout = DESC_SW128) {
    uint64_t d = 0;
    d |= static_cast<uint64_t>((saddr & 0x3FFFFu) >> 4);
    d |= static_cast<uint64_t>((lbo >> 4) & 0x3FFFu) << 16;
    d |= static_cast<uint64_t>((sbo >> 4) & 0x3FFFu) << 32;
    d |= static_cast<uint64_t>(1) << 46;  // descriptor version for tcgen05
    d |= static_cast<uint64_t>(layout) << 61;
    return d;
}

template <class Cfg>
__device__ __forceinline__ void mma(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc, uint32_t accumulate) {
    if constexpr (Cfg::TF32) {
        asm volatile(
            "{\n\t.reg .pred p;\n\t"
            "setp.ne.b32 p, %4, 0;\n\t"
            "tcgen05.mma.cta_group::1.kind::tf32 [%0], %1, %2, %3, p;\n\t}"
            ::"r"(d_tmem), "l"(adesc), "l"(bdesc), "r"(Cfg::IDESC), "r"(accumulate)
            : "memory");
    } else {
        asm volatile(
            "{\n\t.reg .pred p;\n\t"
            "setp.ne.b32 p, %4, 0;\n\t"
            "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}"
            ::"r"(d_tmem), "l"(adesc), "l"(bdesc), "r"(Cfg::IDESC), "r"(accumulate)
            : "memory");
    }
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

// One 32-row x 128-byte box of C (32 fp32 or 64 fp16 columns; lane = row):
// the row goes to a staging buffer in the 128-byte swizzle the C tensor map
// expects, then lane 0 issues one TMA store of the box (clipped at the matrix
// edges by the hardware) as its own bulk group.  Each epilogue warp alternates
// between two buffers by the count of stores it has issued, so the store that
// last read this buffer is the second newest group: wait_group.read 1 leaves
// only the newest (the other buffer) reading.
__device__ __forceinline__ void stage_and_store(uint32_t stage, const uint32_t (&words)[32], int lane,
                                                const CUtensorMap* tmC, int col, int row0, int b) {
    if (lane == 0) asm volatile("cp.async.bulk.wait_group.read 1;" ::: "memory");
    __syncwarp();
#pragma unroll
    for (int j = 0; j < 8; ++j) {
        const uint32_t a = stage + lane * 128 + ((j ^ (lane & 7)) << 4);
        asm volatile("st.shared.v4.b32 [%0], {%1, %2, %3, %4};" ::"r"(a), "r"(words[4 * j]), "r"(words[4 * j + 1]),
                     "r"(words[4 * j + 2]), "r"(words[4 * j + 3])
                     : "memory");
    }
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
    __syncwarp();
    if (lane == 0) {
        asm volatile("cp.async.bulk.tensor.3d.global.shared::cta.bulk_group [%0, {%1, %2, %3}], [%4];"
                     ::"l"(reinterpret_cast<uint64_t>(tmC)), "r"(col), "r"(row0), "r"(b), "r"(stage)
                     : "memory");
        asm volatile("cp.async.bulk.commit_group;" ::: "memory");
    }
}

// Operand maps: tmA[0..NA), tmB[0..NB) (hi then lo for 3xTF32).
struct OperandMaps {
    CUtensorMap a[2];
    CUtensorMap b[2];
};

template <class Cfg, bool OUT_F16>
__global__ void __launch_bounds__(NUM_THREADS, 1)
    k_gemm_tc(const __grid_constant__ OperandMaps ops, const __grid_constant__ CUtensorMap tmC, int M, int N, int K,
              TileMap tm, int a_batched, int b_batched, int* status) {
    using L = Layout<Cfg>;
    constexpr int BN = Cfg::BN, BK = Cfg::BK, STAGES = Cfg::STAGES;
    extern __shared__ unsigned char smem_raw[];
    const uint32_t raw = smem_u32(smem_raw);
    const uint32_t base = (raw + 1023u) & ~1023u;  // swizzled tiles need 1024-byte alignment
    unsigned char* gbase = smem_raw + (base - raw);
    // stage s: A tiles [NA], then B tiles [NB]
    auto a_tile = [&](int s, int i) { return base + s * L::STAGE + i * L::A_TILE; };
    auto b_tile = [&](int s, int i) { return base + s * L::STAGE + Cfg::NA * L::A_TILE + i * L::B_TILE; };
    const uint32_t sC_stage = base + STAGES * L::STAGE;  // 1024-aligned: the swizzle needs it
    const uint32_t bars = sC_stage + C_STAGE_BYTES;
    // barrier layout: full[STAGES], empty[STAGES], tfull[2], tempty[2], drain
    auto full_bar = [&](int s) { return bars + 8u * s; };
    auto empty_bar = [&](int s) { return bars + 8u * (STAGES + s); };
    auto tfull_bar = [&](int a) { return bars + 8u * (2 * STAGES + a); };
    auto tempty_bar = [&](int a) { return bars + 8u * (2 * STAGES + 2 + a); };
    const uint32_t drain_bar = bars + 8u * (2 * STAGES + 4);
    unsigned char* gmisc = gbase + STAGES * L::STAGE + C_STAGE_BYTES + 8 * (2 * STAGES + 5);
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(gmisc);
    volatile int* abort_flag = reinterpret_cast<volatile int*>(gmisc + 4);
    // Waits for data give up after the context's limit; the drain waits
    // before exit keep the full WAIT_CYCLES.
    const long long limit = wait_limit(status);

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
                     "r"(L::TMEM_COLS)
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
                    if (!mbar_wait(empty_bar(stage), phase ^ 1u, abort_flag, limit)) {
                        ok = false;
                        break;
                    }
                    mbar_expect_tx(full_bar(stage), L::STAGE);
#pragma unroll
                    for (int i = 0; i < Cfg::NA; ++i)
                        tma_load_3d(a_tile(stage, i), &ops.a[i], full_bar(stage), kb * BK, mt * BM, ab);
#pragma unroll
                    for (int i = 0; i < Cfg::NB; ++i)
#pragma unroll
                        for (int j = 0; j < L::B_BOXES; ++j)
                            tma_load_3d(b_tile(stage, i) + j * L::B_BOX, &ops.b[i], full_bar(stage),
                                        nt * BN + j * L::ROW_ELEMS, kb * BK, bb);
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
                if (!mbar_wait(tempty_bar(acc), acc_phase ^ 1u, abort_flag, limit)) break;
                tc_fence_after();
                const uint32_t d_tmem = tmem_base + static_cast<uint32_t>(acc * BN);
                for (int kb = 0; kb < num_kb; ++kb) {
                    if (!mbar_wait(full_bar(stage), phase, abort_flag, limit)) {
                        ok = false;
                        break;
                    }
                    tc_fence_after();
#pragma unroll
                    for (int k = 0; k < BK / Cfg::MMA_K; ++k) {
                        // A: K-major, a k slice is 32 bytes inside the 128-byte swizzle row.
                        // B: MN-major, a k slice is MMA_K rows of 128 bytes; the
                        //    128-byte column chunks are one TMA box (B_BOX bytes) apart.
                        const uint32_t ak = static_cast<uint32_t>(k * 32);
                        const uint32_t bk = static_cast<uint32_t>(k * Cfg::MMA_K * 128);
                        const uint32_t acc_in = (kb > 0 || k > 0) ? 1u : 0u;
                        auto bdesc = [&](int part) {
                            return smem_desc(b_tile(stage, part) + bk, L::B_BOX, Cfg::B_SBO, Cfg::B_DESC_LAYOUT);
                        };
                        if constexpr (Cfg::TF32) {
                            // hi*hi + hi*lo + lo*hi
                            mma<Cfg>(d_tmem, smem_desc(a_tile(stage, 0) + ak, 16, 1024), bdesc(0), acc_in);
                            mma<Cfg>(d_tmem, smem_desc(a_tile(stage, 0) + ak, 16, 1024), bdesc(1), 1u);
                            mma<Cfg>(d_tmem, smem_desc(a_tile(stage, 1) + ak, 16, 1024), bdesc(0), 1u);
                        } else {
                            mma<Cfg>(d_tmem, smem_desc(a_tile(stage, 0) + ak, 16, 1024), bdesc(0), acc_in);
                        }
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
        uint32_t stores = 0;  // bulk stores this warp has issued: picks the staging buffer
        for (int t = blockIdx.x; t < total; t += gridDim.x) {
            // one lane waits, the warp follows its result (tcgen05.ld needs
            // the whole warp converged)
            int ready = 0;
            if (lane == 0) ready = mbar_wait(tfull_bar(acc), acc_phase, abort_flag, limit) ? 1 : 0;
            ready = __shfl_sync(0xffffffffu, ready, 0);
            if (!ready) break;
            tc_fence_after();
            int b, mt, nt;
            tm.decode(t, b, mt, nt);
            const int row0 = mt * BM + quarter * 32;  // first of this warp's 32 rows
            const uint32_t taddr =
                tmem_base + (static_cast<uint32_t>(quarter * 32) << 16) + static_cast<uint32_t>(acc * BN);
            // Chunks of 32 rows x 128 bytes, up to the last column of the matrix.
            constexpr int CHUNK_COLS = OUT_F16 ? 64 : 32;
            const int cend = min(BN, N - nt * BN);
            for (int c0 = 0; c0 < cend; c0 += CHUNK_COLS) {
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
                if (c0 + CHUNK_COLS >= cend) {
                    // the warp's last columns of this accumulator are in
                    // registers: release it before storing them
                    tc_fence_before();
                    __syncwarp();
                    if (lane == 0) mbar_arrive(tempty_bar(acc));
                }
                if (row0 >= M) continue;  // rows past the matrix: nothing to store
                stage_and_store(sC_stage + static_cast<uint32_t>((quarter * 2 + (stores & 1u)) * C_BOX_BYTES), words,
                                lane, &tmC, nt * BN + c0, row0, b);
                ++stores;
            }
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
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem_base), "r"(L::TMEM_COLS)
                     : "memory");
    }
}

// ---------------------------------------------------------------------------
// Two-SM variant (fp16 inputs): a cluster of two CTAs computes a 256 x 256
// tile with tcgen05.mma.cta_group::2.  Each CTA holds 128 rows of A and 128
// of the 256 columns of B per k-block (32 KiB per stage instead of 48 KiB for
// the same work per SM), so six stages fit and the operand feed, which bounds
// short-K problems, needs two thirds of the bytes per flop.
//   * both CTAs' producers load their halves with cta_group::2 TMA loads that
//     complete on the leader's (rank 0) full barrier; only the leader's
//     producer arms it (expect_tx of both halves);
//   * the leader's MMA warp issues the MMAs (D rows 0-127 land in its TMEM,
//     rows 128-255 in the peer's) and commits each stage to both CTAs' empty
//     barriers and each finished tile to both CTAs' tfull barriers;
//   * each CTA drains its own TMEM rows; its epilogue warps release the
//     accumulator with remote arrivals on the leader's tempty barrier;
//   * cluster barriers order barrier initialisation and the final TMEM free.
// Every load writes only its own CTA's shared memory.  Every wait is bounded
// as in k_gemm_tc; after an abort each CTA waits a bounded time before tearing
// down so that copies in flight (they complete on the leader's barrier) have
// landed.
// ---------------------------------------------------------------------------
constexpr int P_BK = 64;
constexpr int P_STAGES = 6;
constexpr int P_A_TILE = 128 * P_BK * 2;              // this CTA's 128 rows of A
constexpr int P_B_BOX = P_BK * 128;                   // 64 columns x 64 k of B
constexpr int P_B_TILE = 2 * P_B_BOX;                 // this CTA's 128 columns of B
constexpr int P_STAGE = P_A_TILE + P_B_TILE;          // 32 KiB
constexpr int P_BN = 256;                             // tile columns (both CTAs)
constexpr int P_TMEM_COLS = 2 * P_BN;
constexpr size_t P_SMEM = size_t(P_STAGES) * P_STAGE + C_STAGE_BYTES + 1024 + 256;
static_assert(P_SMEM <= 232448, "shared memory budget of the two-SM kernel");
constexpr uint32_t P_IDESC = (1u << 4) | (0u << 7) | (0u << 10) | (1u << 16) | (uint32_t(P_BN >> 3) << 17) |
                             (uint32_t(256 >> 4) << 24);  // f16 x f16 -> f32, B MN-major, N=256, M=256

__device__ __forceinline__ uint32_t cluster_rank() {
    uint32_t r;
    asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
    return r;
}

__device__ __forceinline__ uint32_t map_to_rank(uint32_t saddr, uint32_t rank) {
    uint32_t out;
    asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(out) : "r"(saddr), "r"(rank));
    return out;
}

__device__ __forceinline__ void cluster_sync() {
    asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}

__device__ __forceinline__ void tma_load_3d_pair(uint32_t dst, const CUtensorMap* map, uint32_t cluster_bar, int c0,
                                                 int c1, int c2) {
    asm volatile(
        "cp.async.bulk.tensor.3d.cta_group::2.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3, "
        "%4}], [%5];" ::"r"(dst),
        "l"(reinterpret_cast<uint64_t>(map)), "r"(c0), "r"(c1), "r"(c2), "r"(cluster_bar)
        : "memory");
}

__device__ __forceinline__ void mma_pair(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc, uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::2.kind::f16 [%0], %1, %2, %3, p;\n\t}"
        ::"r"(d_tmem), "l"(adesc), "l"(bdesc), "r"(P_IDESC), "r"(accumulate)
        : "memory");
}

// Arrive on the barrier at this shared-memory offset in both CTAs of the pair
// once the MMAs issued so far have completed.
__device__ __forceinline__ void mma_commit_pair(uint32_t bar) {
    asm volatile(
        "tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.multicast::cluster.b64 [%0], %1;" ::"r"(bar),
        "h"(static_cast<uint16_t>(0x3))
        : "memory");
}

__device__ __forceinline__ void mma_commit_pair_local(uint32_t bar) {
    asm volatile("tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(bar)
                 : "memory");
}

__device__ __forceinline__ void mbar_arrive_remote(uint32_t cluster_bar) {
    asm volatile("mbarrier.arrive.release.cluster.shared::cluster.b64 _, [%0];" ::"r"(cluster_bar) : "memory");
}

template <bool OUT_F16>
__global__ void __launch_bounds__(NUM_THREADS, 1)
    k_gemm_tc2(const __grid_constant__ OperandMaps ops, const __grid_constant__ CUtensorMap tmC, int M, int N, int K,
               TileMap tm, int a_batched, int b_batched, int* status) {
    extern __shared__ unsigned char smem_raw[];
    const uint32_t raw = smem_u32(smem_raw);
    const uint32_t base = (raw + 1023u) & ~1023u;
    unsigned char* gbase = smem_raw + (base - raw);
    auto a_tile = [&](int s) { return base + s * P_STAGE; };
    auto b_tile = [&](int s) { return base + s * P_STAGE + P_A_TILE; };
    const uint32_t sC_stage = base + P_STAGES * P_STAGE;
    const uint32_t bars = sC_stage + C_STAGE_BYTES;
    auto full_bar = [&](int s) { return bars + 8u * s; };
    auto empty_bar = [&](int s) { return bars + 8u * (P_STAGES + s); };
    auto tfull_bar = [&](int a) { return bars + 8u * (2 * P_STAGES + a); };
    auto tempty_bar = [&](int a) { return bars + 8u * (2 * P_STAGES + 2 + a); };
    const uint32_t drain_bar = bars + 8u * (2 * P_STAGES + 4);
    unsigned char* gmisc = gbase + P_STAGES * P_STAGE + C_STAGE_BYTES + 8 * (2 * P_STAGES + 5);
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(gmisc);
    volatile int* abort_flag = reinterpret_cast<volatile int*>(gmisc + 4);

    const uint32_t rank = cluster_rank();
    const bool leader = rank == 0;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    if (threadIdx.x == 0) {
        for (int s = 0; s < P_STAGES; ++s) {
            mbar_init(full_bar(s), 1);   // the leader's producer arms it
            mbar_init(empty_bar(s), 1);  // one commit per consumed stage
        }
        for (int a = 0; a < 2; ++a) {
            mbar_init(tfull_bar(a), 1);
            mbar_init(tempty_bar(a), 8);  // 4 epilogue warps in each CTA
        }
        mbar_init(drain_bar, 1);
        *abort_flag = 0;
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
        asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
    }
    if (warp == 1) {
        asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_slot)),
                     "r"(P_TMEM_COLS)
                     : "memory");
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;" ::: "memory");
    }
    tc_fence_before();
    cluster_sync();  // barriers of both CTAs initialised, TMEM allocated
    tc_fence_after();
    const uint32_t tmem_base = *tmem_slot;

    const int total = tm.tiles_m * tm.tiles_n * tm.batch;
    const int nclusters = static_cast<int>(gridDim.x >> 1);
    const int cid = static_cast<int>(blockIdx.x >> 1);
    const int num_kb = (K + P_BK - 1) / P_BK;

    if (warp == 0) {
        if (lane == 0) {
            // ---- producer (both CTAs): this CTA's halves of A and B ----
            int stage = 0;
            uint32_t phase = 0;
            bool ok = true;
            for (int t = cid; t < total && ok; t += nclusters) {
                int b, mt, nt;
                tm.decode(t, b, mt, nt);
                const int ab = a_batched ? b : 0, bb = b_batched ? b : 0;
                for (int kb = 0; kb < num_kb; ++kb) {
                    if (!mbar_wait(empty_bar(stage), phase ^ 1u, abort_flag, WAIT_CYCLES)) {
                        ok = false;
                        break;
                    }
                    if (leader) mbar_expect_tx(full_bar(stage), 2 * P_STAGE);
                    const uint32_t lbar = map_to_rank(full_bar(stage), 0);
                    tma_load_3d_pair(a_tile(stage), &ops.a[0], lbar, kb * P_BK, mt * 256 + static_cast<int>(rank) * 128,
                                     ab);
#pragma unroll
                    for (int j = 0; j < 2; ++j)
                        tma_load_3d_pair(b_tile(stage) + j * P_B_BOX, &ops.b[0], lbar,
                                         nt * P_BN + static_cast<int>(rank) * 128 + j * 64, kb * P_BK, bb);
                    if (++stage == P_STAGES) {
                        stage = 0;
                        phase ^= 1u;
                    }
                }
            }
        }
    } else if (warp == 1) {
        if (lane == 0 && leader) {
            // ---- MMA issuer (leader only) ----
            int stage = 0;
            uint32_t phase = 0;
            int acc = 0;
            uint32_t acc_phase = 0;
            bool ok = true;
            for (int t = cid; t < total && ok; t += nclusters) {
                if (!mbar_wait(tempty_bar(acc), acc_phase ^ 1u, abort_flag, WAIT_CYCLES)) break;
                tc_fence_after();
                const uint32_t d_tmem = tmem_base + static_cast<uint32_t>(acc * P_BN);
                for (int kb = 0; kb < num_kb; ++kb) {
                    if (!mbar_wait(full_bar(stage), phase, abort_flag, WAIT_CYCLES)) {
                        ok = false;
                        break;
                    }
                    tc_fence_after();
#pragma unroll
                    for (int k = 0; k < P_BK / 16; ++k) {
                        const uint32_t acc_in = (kb > 0 || k > 0) ? 1u : 0u;
                        mma_pair(d_tmem, smem_desc(a_tile(stage) + k * 32, 16, 1024),
                                 smem_desc(b_tile(stage) + k * 16 * 128, P_B_BOX, 1024), acc_in);
                    }
                    mma_commit_pair(empty_bar(stage));  // the stage is free in both CTAs
                    if (++stage == P_STAGES) {
                        stage = 0;
                        phase ^= 1u;
                    }
                }
                if (!ok) break;
                mma_commit_pair(tfull_bar(acc));  // both halves of the accumulator are ready
                if (++acc == 2) {
                    acc = 0;
                    acc_phase ^= 1u;
                }
            }
            mma_commit_pair_local(drain_bar);
            const long long t0 = clock64();
            while (!mbar_test(drain_bar, 0) && clock64() - t0 < WAIT_CYCLES) {
            }
        }
    } else {
        // ---- epilogue (both CTAs): this CTA's 128 rows of the tile ----
        const int quarter = warp & 3;
        int acc = 0;
        uint32_t acc_phase = 0;
        uint32_t stores = 0;  // bulk stores this warp has issued: picks the staging buffer
        const uint32_t tempty_leader0 = map_to_rank(tempty_bar(0), 0);
        const uint32_t tempty_leader1 = map_to_rank(tempty_bar(1), 0);
        for (int t = cid; t < total; t += nclusters) {
            int ready = 0;
            if (lane == 0) ready = mbar_wait(tfull_bar(acc), acc_phase, abort_flag, WAIT_CYCLES) ? 1 : 0;
            ready = __shfl_sync(0xffffffffu, ready, 0);
            if (!ready) break;
            tc_fence_after();
            int b, mt, nt;
            tm.decode(t, b, mt, nt);
            const int row0 = mt * 256 + static_cast<int>(rank) * 128 + quarter * 32;
            const uint32_t taddr =
                tmem_base + (static_cast<uint32_t>(quarter * 32) << 16) + static_cast<uint32_t>(acc * P_BN);
            constexpr int CHUNK_COLS = OUT_F16 ? 64 : 32;
            const int cend = min(P_BN, N - nt * P_BN);  // the tile's columns inside the matrix
            const uint32_t tempty_leader = acc == 0 ? tempty_leader0 : tempty_leader1;
            for (int c0 = 0; c0 < cend; c0 += CHUNK_COLS) {
                uint32_t words[32];
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
                if (c0 + CHUNK_COLS >= cend) {
                    // the warp's last columns of this accumulator are in
                    // registers: release it before storing them
                    tc_fence_before();
                    __syncwarp();
                    if (lane == 0) mbar_arrive_remote(tempty_leader);
                }
                if (row0 >= M) continue;  // rows past the matrix: nothing to store
                stage_and_store(sC_stage + static_cast<uint32_t>((quarter * 2 + (stores & 1u)) * C_BOX_BYTES), words,
                                lane, &tmC, nt * P_BN + c0, row0, b);
                ++stores;
            }
            if (++acc == 2) {
                acc = 0;
                acc_phase ^= 1u;
            }
        }
        if (lane == 0) asm volatile("cp.async.bulk.wait_group 0;" ::: "memory");
        __syncwarp();
    }
    tc_fence_before();
    __syncthreads();
    if (*abort_flag) {
        if (threadIdx.x == 0) atomicExch(status, QSML_E_TIMEOUT);
        // copies still in flight complete on the leader's barrier: give them
        // time to land before the CTA pair's shared memory is released
        const long long t0 = clock64();
        while (clock64() - t0 < 20000000LL) {
        }
    }
    cluster_sync();  // the leader's MMAs are drained and both epilogues are done
    if (warp == 1) {
        tc_fence_after();
        asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" ::"r"(tmem_base), "r"(P_TMEM_COLS)
                     : "memory");
    }
}

// fp32 -> (hi, lo) for 3xTF32: hi is x rounded to tf32 (cvt.rna, low 13 bits
// zero), lo = x - hi exactly, itself rounded to tf32 (its own error is below
// 2^-22 |x|).
__global__ void __launch_bounds__(256) k_split_tf32(const float4* __restrict__ x, float4* __restrict__ hi,
                                                    float4* __restrict__ lo, int64_t n4) {
    for (int64_t i = static_cast<int64_t>(blockIdx.x) * 256 + threadIdx.x; i < n4;
         i += static_cast<int64_t>(gridDim.x) * 256) {
        float4 v = x[i], h, l;
        float* pv = &v.x;
        float* ph = &h.x;
        float* pl = &l.x;
#pragma unroll
        for (int e = 0; e < 4; ++e) {
            uint32_t hb, lb;
            asm("cvt.rna.tf32.f32 %0, %1;" : "=r"(hb) : "f"(pv[e]));
            ph[e] = __uint_as_float(hb);
            const float r = __fsub_rn(pv[e], ph[e]);
            asm("cvt.rna.tf32.f32 %0, %1;" : "=r"(lb) : "f"(r));
            pl[e] = __uint_as_float(lb);
        }
        hi[i] = h;
        lo[i] = l;
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

// 3-D tensor map: dims {inner, outer, batch}, 128-byte swizzle (16- or 32-byte units).
bool make_map(CUtensorMap* map, const void* ptr, uint64_t inner, uint64_t outer, uint64_t batch, uint64_t row_bytes,
              uint64_t batch_bytes, uint32_t box_inner, uint32_t box_outer, CUtensorMapDataType dt,
              CUtensorMapSwizzle swizzle = CU_TENSOR_MAP_SWIZZLE_128B) {
    auto fn = encode_fn();
    if (!fn) return false;
    cuuint64_t dims[3] = {inner, outer, batch};
    cuuint64_t strides[2] = {row_bytes, batch_bytes};
    cuuint32_t box[3] = {box_inner, box_outer, 1};
    cuuint32_t estr[3] = {1, 1, 1};
    CUresult r = fn(map, dt, 3, const_cast<void*>(ptr), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                    swizzle, CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    return r == CUDA_SUCCESS;
}

// Opt in to the kernel's dynamic shared memory once per device.
template <class Cfg, bool OUT_F16>
qsml_status_t set_smem_attr(Context* ctx) {
    static std::mutex mu;
    static uint64_t done = 0;
    std::lock_guard<std::mutex> lk(mu);
    const uint64_t bit = uint64_t(1) << (ctx->device & 63);
    if (done & bit) return QSML_OK;
    cudaError_t e = cudaFuncSetAttribute(k_gemm_tc<Cfg, OUT_F16>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         static_cast<int>(Layout<Cfg>::SMEM));
    if (e != cudaSuccess) return check_cuda(ctx, e, "matmul: shared-memory attribute");
    done |= bit;
    return QSML_OK;
}

// Operand pointers per part (hi/lo for 3xTF32) with their batch strides.
struct Operands {
    const void* a[2];
    const void* b[2];
    int64_t lda, ldb, sA, sB;
};

template <class Cfg, bool OUT_F16>
qsml_status_t launch_tc(Context* ctx, const MatmulArgs& g, const Operands& o) {
    constexpr CUtensorMapDataType in_t =
        Cfg::TF32 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT32 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16;
    constexpr uint64_t es = Cfg::ESIZE;
    const uint64_t a_batch = o.sA ? static_cast<uint64_t>(g.batch) : 1;
    const uint64_t b_batch = o.sB ? static_cast<uint64_t>(g.batch) : 1;
    OperandMaps maps;
    for (int i = 0; i < Cfg::NA; ++i)
        if (!make_map(&maps.a[i], o.a[i], g.K, g.M, a_batch, o.lda * es, (o.sA ? o.sA : o.lda * g.M) * es,
                      Layout<Cfg>::ROW_ELEMS, BM, in_t))
            return QSML_E_UNSUPPORTED;
    for (int i = 0; i < Cfg::NB; ++i)
        if (!make_map(&maps.b[i], o.b[i], g.N, g.K, b_batch, o.ldb * es, (o.sB ? o.sB : o.ldb * g.K) * es,
                      Layout<Cfg>::ROW_ELEMS, Cfg::BK, in_t, Cfg::B_SWIZZLE))
            return QSML_E_UNSUPPORTED;
    for (int i = Cfg::NA; i < 2; ++i) maps.a[i] = maps.a[0];
    for (int i = Cfg::NB; i < 2; ++i) maps.b[i] = maps.b[0];
    // C: 128-byte wide boxes of 32 rows (32 fp32 or 64 fp16 columns).
    CUtensorMap tmC;
    const uint64_t c_es = OUT_F16 ? 2 : 4;
    if (!make_map(&tmC, g.C, g.N, g.M, g.batch, g.N * c_es, g.M * g.N * c_es, static_cast<uint32_t>(128 / c_es), 32,
                  OUT_F16 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT32))
        return QSML_E_UNSUPPORTED;
    QSML_TRY_STATUS((set_smem_attr<Cfg, OUT_F16>(ctx)));
    TileMap tm;
    tm.tiles_m = static_cast<int>((g.M + BM - 1) / BM);
    tm.tiles_n = static_cast<int>((g.N + Cfg::BN - 1) / Cfg::BN);
    tm.batch = static_cast<int>(g.batch);
    const int64_t total = static_cast<int64_t>(tm.tiles_m) * tm.tiles_n * tm.batch;
    const int grid = static_cast<int>(total < ctx->num_sms ? total : ctx->num_sms);
    k_gemm_tc<Cfg, OUT_F16><<<grid, NUM_THREADS, Layout<Cfg>::SMEM, ctx->stream>>>(
        maps, tmC, static_cast<int>(g.M), static_cast<int>(g.N), static_cast<int>(g.K), tm, o.sA ? 1 : 0,
        o.sB ? 1 : 0, ctx->status);
    return after_launch(ctx, Cfg::TF32 ? "k_gemm_tc<3xtf32>" : "k_gemm_tc<f16>");
}

// The two-SM kernel: same operand and output maps as CfgF16 (A boxes of 128
// rows x 64 k, B boxes of 64 columns x 64 k), 256 x 256 tiles, one cluster of
// two CTAs per SM pair.
template <bool OUT_F16>
qsml_status_t launch_tc2(Context* ctx, const MatmulArgs& g, const Operands& o) {
    const uint64_t a_batch = o.sA ? static_cast<uint64_t>(g.batch) : 1;
    const uint64_t b_batch = o.sB ? static_cast<uint64_t>(g.batch) : 1;
    OperandMaps maps;
    if (!make_map(&maps.a[0], o.a[0], g.K, g.M, a_batch, o.lda * 2, (o.sA ? o.sA : o.lda * g.M) * 2, 64, 128,
                  CU_TENSOR_MAP_DATA_TYPE_FLOAT16) ||
        !make_map(&maps.b[0], o.b[0], g.N, g.K, b_batch, o.ldb * 2, (o.sB ? o.sB : o.ldb * g.K) * 2, 64, P_BK,
                  CU_TENSOR_MAP_DATA_TYPE_FLOAT16))
        return QSML_E_UNSUPPORTED;
    maps.a[1] = maps.a[0];
    maps.b[1] = maps.b[0];
    CUtensorMap tmC;
    const uint64_t c_es = OUT_F16 ? 2 : 4;
    if (!make_map(&tmC, g.C, g.N, g.M, g.batch, g.N * c_es, g.M * g.N * c_es, static_cast<uint32_t>(128 / c_es), 32,
                  OUT_F16 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT32))
        return QSML_E_UNSUPPORTED;

    cudaLaunchConfig_t cfg = {};
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = 2;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    cfg.blockDim = dim3(NUM_THREADS);
    cfg.dynamicSmemBytes = P_SMEM;
    cfg.stream = ctx->stream;
    cfg.attrs = attr;
    cfg.numAttrs = 1;

    // Shared-memory opt-in and the number of co-resident clusters, once per device.
    static std::mutex mu;
    static int max_clusters[64] = {};
    int clusters = 0;
    {
        std::lock_guard<std::mutex> lk(mu);
        int& mc = max_clusters[ctx->device & 63];
        if (mc == 0) {
            cudaError_t e = cudaFuncSetAttribute(k_gemm_tc2<OUT_F16>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                                 static_cast<int>(P_SMEM));
            if (e != cudaSuccess) return check_cuda(ctx, e, "matmul: shared-memory attribute");
            cfg.gridDim = dim3(2 * (ctx->num_sms / 2));
            e = cudaOccupancyMaxActiveClusters(&mc, k_gemm_tc2<OUT_F16>, &cfg);
            if (e != cudaSuccess || mc <= 0) {
                cudaGetLastError();
                mc = -1;  // no cluster of two fits: the one-SM kernel serves this device
            }
        }
        clusters = mc;
    }
    if (clusters < 0) return QSML_E_UNSUPPORTED;
    TileMap tm;
    tm.tiles_m = static_cast<int>((g.M + 255) / 256);
    tm.tiles_n = static_cast<int>((g.N + P_BN - 1) / P_BN);
    tm.batch = static_cast<int>(g.batch);
    const int64_t total = static_cast<int64_t>(tm.tiles_m) * tm.tiles_n * tm.batch;
    if (total < clusters) clusters = static_cast<int>(total);
    cfg.gridDim = dim3(2 * clusters);
    cudaError_t e = cudaLaunchKernelEx(&cfg, k_gemm_tc2<OUT_F16>, maps, tmC, static_cast<int>(g.M),
                                       static_cast<int>(g.N), static_cast<int>(g.K), tm, o.sA ? 1 : 0, o.sB ? 1 : 0,
                                       ctx->status);
    if (e != cudaSuccess) return check_cuda(ctx, e, "k_gemm_tc2<f16>");
    return after_launch(ctx, "k_gemm_tc2<f16>");
}

// Which fp16 kernel: QSML_GEMM_2SM=1 forces the two-SM kernel, =0 the one-SM
// kernel; otherwise the two-SM kernel runs when the 256 x 256 tiles fill the
// SM pairs at least once.
bool use_two_sm(const Context* ctx, const MatmulArgs& g) {
    const char* env = std::getenv("QSML_GEMM_2SM");
    if (env && env[0] == '0') return false;
    if (env && env[0] == '1') return true;
    const int64_t tiles = ((g.M + 255) / 256) * ((g.N + 255) / 256) * g.batch;
    return tiles >= ctx->num_sms / 2;
}

// What the kernels take: 16-byte aligned operands and row strides (TMA), N a
// multiple of 8 (128-byte output boxes stay inside rows of whole 16-byte units).
bool tc_shape_ok(const MatmulArgs& g, int es) {
    const int64_t q = 16 / es;
    return g.K % q == 0 && g.N % 8 == 0 && g.lda % q == 0 && g.ldb % q == 0 && g.sA % q == 0 && g.sB % q == 0 &&
           aligned16(g.A) && aligned16(g.B) && aligned16(g.C) && g.M > 0 && g.N > 0 && g.K > 0;
}

}  // namespace

qsml_status_t matmul_tc_f16(Context* ctx, const MatmulArgs& g, bool out_f16) {
    if (!tc_shape_ok(g, 2) || !ctx->status) return QSML_E_UNSUPPORTED;
    Operands o{{g.A, g.A}, {g.B, g.B}, g.lda, g.ldb, g.sA, g.sB};
    if (use_two_sm(ctx, g)) {
        const qsml_status_t st = out_f16 ? launch_tc2<true>(ctx, g, o) : launch_tc2<false>(ctx, g, o);
        if (st != QSML_E_UNSUPPORTED) return st;
    }
    return out_f16 ? launch_tc<CfgF16, true>(ctx, g, o) : launch_tc<CfgF16, false>(ctx, g, o);
}

qsml_status_t matmul_tc_3xtf32(Context* ctx, const MatmulArgs& g) {
    if (!tc_shape_ok(g, 4) || !ctx->status) return QSML_E_UNSUPPORTED;
    // Split A and B into contiguous hi/lo copies (scratch from the caching
    // allocator, returned to it after the launch: reuse is stream-ordered).
    const int64_t a_elems = (g.sA ? g.batch : 1) * g.M * g.K;
    const int64_t b_elems = (g.sB ? g.batch : 1) * g.K * g.N;
    const bool a_dense = g.lda == g.K && (!g.sA || g.sA == g.M * g.K);
    const bool b_dense = g.ldb == g.N && (!g.sB || g.sB == g.K * g.N);
    if (!a_dense || !b_dense) return QSML_E_UNSUPPORTED;
    void* buf[4] = {nullptr, nullptr, nullptr, nullptr};
    std::string err;
    const size_t sizes[4] = {static_cast<size_t>(a_elems) * 4, static_cast<size_t>(a_elems) * 4,
                             static_cast<size_t>(b_elems) * 4, static_cast<size_t>(b_elems) * 4};
    for (int i = 0; i < 4; ++i) {
        qsml_status_t st = ctx->allocator->alloc(sizes[i], &buf[i], &err);
        if (st != QSML_OK) {
            for (int j = 0; j < i; ++j) ctx->allocator->free(buf[j], &err);
            return set_error(ctx, st, err);
        }
    }
    auto split = [&](const void* src, void* hi, void* lo, int64_t n) {
        const int64_t n4 = n / 4;  // K % 4 == 0 and N % 8 == 0, so n is a multiple of 4
        int64_t blocks = (n4 + 255) / 256;
        if (blocks > int64_t(ctx->num_sms) * 16) blocks = int64_t(ctx->num_sms) * 16;
        k_split_tf32<<<static_cast<unsigned>(blocks), 256, 0, ctx->stream>>>(
            static_cast<const float4*>(src), static_cast<float4*>(hi), static_cast<float4*>(lo), n4);
        return after_launch(ctx, "k_split_tf32");
    };
    qsml_status_t st = split(g.A, buf[0], buf[1], a_elems);
    if (st == QSML_OK) st = split(g.B, buf[2], buf[3], b_elems);
    if (st == QSML_OK) {
        Operands o{{buf[0], buf[1]}, {buf[2], buf[3]}, g.K, g.N, g.sA ? g.M * g.K : 0, g.sB ? g.K * g.N : 0};
        st = launch_tc<Cfg3xTF32, false>(ctx, g, o);
        if (st == QSML_E_UNSUPPORTED) st = set_error(ctx, QSML_E_CUDA, "matmul 3xTF32: tensor map creation failed");
    }
    for (int i = 0; i < 4; ++i) ctx->allocator->free(buf[i], &err);
    return st;
}

}  // namespace qsml
