// Elementwise building blocks shared by the per-op kernels (elementwise.cu)
// and the fused-expression kernel (ew_fused.cu): element types, the
// operators with their exact rounding, and the NumPy-broadcast planner.
#pragma once

#include <type_traits>

#include "qsml_internal.cuh"
#include "ew_ops.cuh"

namespace qsml {
namespace ew {

// ---------------------------------------------------------------------------
// Element types: storage type T, compute type C.
// ---------------------------------------------------------------------------
template <typename T> struct Elem;
template <> struct Elem<float> {
    using C = float;
    static __device__ __forceinline__ float ld(float v) { return v; }
    static __device__ __forceinline__ float st(float v) { return v; }
};
template <> struct Elem<__half> {
    using C = float;
    static __device__ __forceinline__ float ld(__half v) { return __half2float(v); }
    static __device__ __forceinline__ __half st(float v) { return __float2half_rn(v); }
};
template <> struct Elem<int32_t> {
    using C = int32_t;
    static __device__ __forceinline__ int32_t ld(int32_t v) { return v; }
    static __device__ __forceinline__ int32_t st(int32_t v) { return v; }
};

template <typename T> struct alignas(16) Pack {
    static constexpr int N = 16 / sizeof(T);
    T v[N];
};

// Operators: ew_ops.cuh.  Scalar right operand held by value:
template <int OP> struct ScalarOp {
    float s;
    __device__ __forceinline__ float operator()(float a) const { return BinOp<OP>()(a, s); }
    __device__ __forceinline__ int32_t operator()(int32_t a) const {
        return BinOp<OP>()(a, static_cast<int32_t>(s));
    }
};

// relu on binary16 keeps NaN payloads and maps every non-positive to +0,
// exactly like the binary32 rule (conversion is exact both ways).

// ---------------------------------------------------------------------------
// Plan: collapsed output shape and per-operand element strides.
// ---------------------------------------------------------------------------
template <int NI> struct EwPlanT {
    int nd;
    int64_t shape[kMaxDims];
    int64_t st[NI][kMaxDims];  // input strides (0 = broadcast)
};
using EwPlan = EwPlanT<2>;

// Offset of the first element of collapsed row `row` for input j.
template <typename IDX, typename Plan>
__device__ __forceinline__ int64_t row_offset(const Plan& p, int j, IDX row) {
    int64_t off = 0;
    for (int d = p.nd - 2; d >= 1; --d) {
        IDX e = static_cast<IDX>(p.shape[d]);
        IDX c = row % e;
        row /= e;
        off += static_cast<int64_t>(c) * p.st[j][d];
    }
    if (p.nd >= 2) off += static_cast<int64_t>(row) * p.st[j][0];
    return off;
}

// ---------------------------------------------------------------------------
// Host planning
// ---------------------------------------------------------------------------

// Aligns each input's shape/strides to out's dims (NumPy broadcasting) and
// collapses.  Returns QSML_OK or a shape error.
template <int NI>
qsml_status_t make_plan(Context* ctx, const qsml_tdesc* out, const qsml_tdesc* const* ins, int nin, EwPlanT<NI>* p) {
    const int nd = out->ndim;
    int64_t shape[kMaxDims];
    int64_t st[NI][kMaxDims];
    for (int d = 0; d < nd; ++d) shape[d] = out->shape[d];
    for (int j = 0; j < nin; ++j) {
        const qsml_tdesc* a = ins[j];
        if (a->ndim > nd) return set_error(ctx, QSML_E_SHAPE, "input has more dims than the output");
        for (int d = 0; d < nd; ++d) {
            int ad = a->ndim - nd + d;
            if (ad < 0) { st[j][d] = 0; continue; }
            if (a->shape[ad] == out->shape[d]) st[j][d] = out->shape[d] == 1 ? 0 : a->stride[ad];
            else if (a->shape[ad] == 1) st[j][d] = 0;
            else return set_error(ctx, QSML_E_SHAPE, "operand shape does not broadcast to the output shape");
        }
    }
    // Output shape must be exactly the broadcast of the inputs: every out
    // extent > 1 must come from some input.
    for (int d = 0; d < nd; ++d) {
        if (out->shape[d] == 1) continue;
        bool from_input = false;
        for (int j = 0; j < nin; ++j) {
            int ad = ins[j]->ndim - nd + d;
            if (ad >= 0 && ins[j]->shape[ad] == out->shape[d]) from_input = true;
        }
        if (!from_input) return set_error(ctx, QSML_E_SHAPE, "output shape is not the broadcast shape of the inputs");
    }
    // Drop size-1 dims, then merge dims contiguous for every operand
    // (out is contiguous, so only the inputs decide).
    int n = 0;
    for (int d = 0; d < nd; ++d) {
        if (shape[d] == 1) continue;
        if (n > 0) {
            bool merge = true;
            for (int j = 0; j < nin; ++j)
                if (p->st[j][n - 1] != st[j][d] * shape[d]) merge = false;
            if (merge) {
                p->shape[n - 1] *= shape[d];
                for (int j = 0; j < nin; ++j) p->st[j][n - 1] = st[j][d];
                continue;
            }
        }
        p->shape[n] = shape[d];
        for (int j = 0; j < nin; ++j) p->st[j][n] = st[j][d];
        ++n;
    }
    if (n == 0) {
        p->shape[0] = 1;
        for (int j = 0; j < NI; ++j) p->st[j][0] = 0;
        n = 1;
    }
    for (int j = nin; j < NI; ++j)
        for (int d = 0; d < n; ++d) p->st[j][d] = 0;
    p->nd = n;
    return QSML_OK;
}

}  // namespace ew
}  // namespace qsml
