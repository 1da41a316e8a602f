// qsml_matmul entry point: validates descriptors and picks the kernel.
//
// Reference: Ops::matmul (Ops/LinAlg.cpp:221-271) asserts rank 2, equal
// inner dims and equal dtypes, then dispatches a SIMT shader in row bands
// of at most 4096 workgroups with a host synchronize after each band;
// Ops::batch_matmul (LinAlg.cpp:273-290) multiplies slice 0 N times and
// returns an unwritten tensor.  Here one launch covers every batch entry.
#include "matmul.cuh"

using namespace qsml;

namespace {

qsml_status_t fill_args(Context* ctx, const qsml_tdesc* a, const qsml_tdesc* b, const qsml_tdesc* c, MatmulArgs* g) {
    if (a->ndim != b->ndim || (a->ndim != 2 && a->ndim != 3))
        return set_error(ctx, QSML_E_SHAPE, "qsml_matmul: A and B must both be rank 2 or both rank 3");
    const int o = a->ndim - 2;
    g->batch = a->ndim == 3 ? a->shape[0] : 1;
    if (a->ndim == 3 && b->shape[0] != a->shape[0])
        return set_error(ctx, QSML_E_SHAPE, "qsml_matmul: batch sizes differ");
    g->M = a->shape[o];
    g->K = a->shape[o + 1];
    g->N = b->shape[o + 1];
    if (b->shape[o] != g->K) return set_error(ctx, QSML_E_SHAPE, "qsml_matmul: inner dimensions differ");
    if (c->ndim != a->ndim || c->shape[o] != g->M || c->shape[o + 1] != g->N ||
        (a->ndim == 3 && c->shape[0] != g->batch))
        return set_error(ctx, QSML_E_SHAPE, "qsml_matmul: C has the wrong shape");
    if (!is_contiguous(c)) return set_error(ctx, QSML_E_SHAPE, "qsml_matmul: C must be contiguous");
    if ((g->K > 1 && a->stride[o + 1] != 1) || (g->N > 1 && b->stride[o + 1] != 1))
        return set_error(ctx, QSML_E_UNSUPPORTED,
                         "qsml_matmul: A and B need unit stride in their last dim (materialise with qsml_gather)");
    if (g->M > INT32_MAX || g->N > INT32_MAX || g->K > INT32_MAX || g->batch > 65535)
        return set_error(ctx, QSML_E_UNSUPPORTED, "qsml_matmul: dimensions too large");
    g->lda = a->stride[o];
    g->ldb = b->stride[o];
    g->sA = a->ndim == 3 ? (a->shape[0] > 1 ? a->stride[0] : 0) : 0;
    g->sB = b->ndim == 3 ? (b->shape[0] > 1 ? b->stride[0] : 0) : 0;
    g->sC = g->M * g->N;
    g->A = a->data;
    g->B = b->data;
    g->C = c->data;
    return QSML_OK;
}

}  // namespace

extern "C" qsml_status_t qsml_matmul(qsml_ctx* handle, const qsml_tdesc* a, const qsml_tdesc* b,
                                     const qsml_tdesc* c, int32_t precision) {
    QSML_CTX(handle);
    QSML_TRY_STATUS(check_desc(C_, a, "a"));
    QSML_TRY_STATUS(check_desc(C_, b, "b"));
    QSML_TRY_STATUS(check_desc(C_, c, "c"));
    if (a->dtype != b->dtype) return set_error(C_, QSML_E_DTYPE, "qsml_matmul: A and B dtypes differ");
    MatmulArgs g;
    QSML_TRY_STATUS(fill_args(C_, a, b, c, &g));
    if (g.batch == 0 || g.M == 0 || g.N == 0) return QSML_OK;
    if (g.K == 0) {
        const int es = dtype_size(c->dtype);
        return check_cuda(C_, cudaMemsetAsync(c->data, 0, static_cast<size_t>(g.batch * g.M * g.N) * es, C_->stream),
                          "qsml_matmul zero");
    }
    if (a->dtype == QSML_F32) {
        if (c->dtype != QSML_F32) return set_error(C_, QSML_E_DTYPE, "qsml_matmul: F32 inputs need an F32 C");
        if (precision == QSML_MM_AUTO || precision == QSML_MM_FP32_FFMA) return matmul_simt<float, float>(C_, g);
        if (precision == QSML_MM_FP32_3XTF32) {
            qsml_status_t st = matmul_tc_3xtf32(C_, g);
            if (st == QSML_E_UNSUPPORTED)
                return set_error(C_, st, "qsml_matmul: 3xTF32 needs dense A and B, K % 4 == 0, N % 8 == 0 and "
                                         "16-byte aligned operands");
            return st;
        }
        return set_error(C_, QSML_E_INVALID, "qsml_matmul: precision does not apply to F32 inputs");
    }
    if (a->dtype == QSML_F16) {
        if (c->dtype != QSML_F32 && c->dtype != QSML_F16)
            return set_error(C_, QSML_E_DTYPE, "qsml_matmul: F16 inputs need an F32 or F16 C");
        if (precision != QSML_MM_AUTO && precision != QSML_MM_FP16_F32ACC)
            return set_error(C_, QSML_E_INVALID, "qsml_matmul: precision does not apply to F16 inputs");
        const bool out_f16 = c->dtype == QSML_F16;
        qsml_status_t st = matmul_tc_f16(C_, g, out_f16);
        if (st != QSML_E_UNSUPPORTED) return st;
        return out_f16 ? matmul_simt<__half, __half>(C_, g) : matmul_simt<__half, float>(C_, g);
    }
    return set_error(C_, QSML_E_DTYPE, "qsml_matmul: dtype must be F32 or F16");
}
