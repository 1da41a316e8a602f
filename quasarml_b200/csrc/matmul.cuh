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

}  // namespace qsml
