// Matmul internals shared by the CUDA-core and tensor-core kernels.
#pragma once

#include "qsml_internal.cuh"

namespace qsml {

struct MatmulArgs {
    const void* A;
    const void* B;
    void* C;
    int64_t batch, M, N, K;
    int64_t lda, ldb;      // row strides of A and B (elements); unit column stride
    int64_t sA, sB, sC;    // batch strides (elements), 0 = shared operand
};

template <typename TI, typename TO>
qsml_status_t matmul_simt(Context* ctx, const MatmulArgs& g);

// Tensor-core fp16 x fp16 -> fp32 (tcgen05 + TMEM, TMA-fed).  Returns
// QSML_E_UNSUPPORTED (without recording an error) when the shape or layout
// is outside what the kernel takes, so the caller can pick another path.
qsml_status_t matmul_tc_f16(Context* ctx, const MatmulArgs& g, bool out_f16);

// fp32 inputs as three tf32 tensor-core products (Ahi*Bhi + Ahi*Blo +
// Alo*Bhi) with fp32 accumulation; A and B must be dense.  Same
// QSML_E_UNSUPPORTED convention as matmul_tc_f16.
qsml_status_t matmul_tc_3xtf32(Context* ctx, const MatmulArgs& g);

}  // namespace qsml
