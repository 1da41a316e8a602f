// Elementwise kernels: broadcast binary ops, scalar-operand ops, unary ops
// and fill.
//
// Reference: Ops/Elementwise.cpp:139-417 builds one GLSL shader per op with
// one element per invocation (`result[idx] = a[idx] op b[idx]`,
// Ops/ShaderGen.cpp:40-53) and requires equal shapes.  Here every op shares
// one host planner and three kernels:
//   * the planner applies NumPy broadcasting (stride 0 on broadcast dims) and
//     collapses dims that are contiguous for every operand, so
//     A[4096,4096] + B[1,4096] becomes a [4096 rows x 4096 cols] problem;
//   * k_ew_rows: 16-byte vector loads/stores along the collapsed inner dim,
//     per-row broadcast offsets computed once per vector (the inner stride of
//     each operand is 0 or 1), several independent vectors per thread;
//   * k_ew_flat: the 1-D contiguous case with a scalar tail;
//   * k_ew_generic: any strides (one element per thread), always correct.
// Arithmetic is IEEE binary32 with explicit round-to-nearest intrinsics, so
// no multiply-add contraction can happen (bit-exact with the oracle).
#include "ew_common.cuh"

namespace qsml {
namespace {

using namespace ew;

constexpr int kThreads = 256;
constexpr int kUnroll = 4;

// ---------------------------------------------------------------------------
// Plan: collapsed output shape and per-operand element strides (ew_common.cuh).
// ---------------------------------------------------------------------------
template <typename T, int NIN> struct Ptrs {
    const T* in[2];
    T* out;
};

template <typename C, int NIN, typename Op>
__device__ __forceinline__ C apply(const Op& op, C a, C b) {
    if constexpr (NIN == 2) return op(a, b);
    else return op(a);
}

// Row kernel: out is [R, Cn] with Cn % VEC == 0; each input's inner stride is
// 0 (one value per row, splatted) or 1 (16-byte vectors).
template <typename T, int NIN, typename Op, typename IDX>
__global__ void __launch_bounds__(kThreads) k_ew_rows(Ptrs<T, NIN> P, EwPlan plan, IDX items, IDX cpr, Op op,
                                                      int defer) {
    pdl_start(defer);
    using E = Elem<T>;
    using CT = typename E::C;
    constexpr int V = Pack<T>::N;
    const IDX base = static_cast<IDX>(blockIdx.x) * (kThreads * kUnroll) + threadIdx.x;
    Pack<T> r[2][kUnroll];
    IDX outoff[kUnroll];
    bool ok[kUnroll];
#pragma unroll
    for (int u = 0; u < kUnroll; ++u) {
        IDX it = base + static_cast<IDX>(u) * kThreads;
        ok[u] = it < items;
        if (!ok[u]) continue;
        IDX row = it / cpr;
        IDX cv = it - row * cpr;
        outoff[u] = it;
#pragma unroll
        for (int j = 0; j < NIN; ++j) {
            int64_t off = row_offset<IDX>(plan, j, row);
            if (plan.st[j][plan.nd - 1] != 0) {
                r[j][u] = *reinterpret_cast<const Pack<T>*>(P.in[j] + off + static_cast<int64_t>(cv) * V);
            } else {
                T s = P.in[j][off];
#pragma unroll
                for (int e = 0; e < V; ++e) r[j][u].v[e] = s;
            }
        }
    }
#pragma unroll
    for (int u = 0; u < kUnroll; ++u) {
        if (!ok[u]) continue;
        Pack<T> o;
#pragma unroll
        for (int e = 0; e < V; ++e) {
            CT a = E::ld(r[0][u].v[e]);
            CT b = NIN == 2 ? E::ld(r[NIN - 1][u].v[e]) : a;
            o.v[e] = E::st(apply<CT, NIN>(op, a, b));
        }
        reinterpret_cast<Pack<T>*>(P.out)[outoff[u]] = o;
    }
    pdl_end(defer);
}

// 1-D contiguous (or scalar-broadcast) operands: vector body + scalar tail.
template <typename T, int NIN, typename Op, bool VEC>
__global__ void __launch_bounds__(kThreads) k_ew_flat(Ptrs<T, NIN> P, EwPlan plan, int64_t n, Op op, int defer) {
    pdl_start(defer);
    using E = Elem<T>;
    using CT = typename E::C;
    constexpr int V = VEC ? Pack<T>::N : 1;
    const int64_t npk = n / V;
    const int64_t base = static_cast<int64_t>(blockIdx.x) * (kThreads * kUnroll) + threadIdx.x;
    bool bc[2];
    T sv[2];
#pragma unroll
    for (int j = 0; j < NIN; ++j) {
        bc[j] = plan.st[j][0] == 0;
        sv[j] = bc[j] ? P.in[j][0] : T();
    }
    if constexpr (VEC) {
        Pack<T> r[2][kUnroll];
#pragma unroll
        for (int u = 0; u < kUnroll; ++u) {
            int64_t pk = base + static_cast<int64_t>(u) * kThreads;
            if (pk >= npk) continue;
#pragma unroll
            for (int j = 0; j < NIN; ++j) {
                if (!bc[j]) {
                    r[j][u] = reinterpret_cast<const Pack<T>*>(P.in[j])[pk];
                } else {
#pragma unroll
                    for (int e = 0; e < Pack<T>::N; ++e) r[j][u].v[e] = sv[j];
                }
            }
        }
#pragma unroll
        for (int u = 0; u < kUnroll; ++u) {
            int64_t pk = base + static_cast<int64_t>(u) * kThreads;
            if (pk >= npk) continue;
            Pack<T> o;
#pragma unroll
            for (int e = 0; e < Pack<T>::N; ++e) {
                CT a = E::ld(r[0][u].v[e]);
                CT b = NIN == 2 ? E::ld(r[NIN - 1][u].v[e]) : a;
                o.v[e] = E::st(apply<CT, NIN>(op, a, b));
            }
            reinterpret_cast<Pack<T>*>(P.out)[pk] = o;
        }
        // tail: the last n % V elements, handled by the first threads of block 0
        if (blockIdx.x == 0) {
            int64_t i = npk * V + threadIdx.x;
            if (i < n) {
                CT a = E::ld(bc[0] ? sv[0] : P.in[0][i]);
                CT b = a;
                if (NIN == 2) b = E::ld(bc[NIN - 1] ? sv[NIN - 1] : P.in[NIN - 1][i]);
                P.out[i] = E::st(apply<CT, NIN>(op, a, b));
            }
        }
    } else {
#pragma unroll
        for (int u = 0; u < kUnroll; ++u) {
            int64_t i = base + static_cast<int64_t>(u) * kThreads;
            if (i >= n) continue;
            CT a = E::ld(bc[0] ? sv[0] : P.in[0][i]);
            CT b = a;
            if (NIN == 2) b = E::ld(bc[NIN - 1] ? sv[NIN - 1] : P.in[NIN - 1][i]);
            P.out[i] = E::st(apply<CT, NIN>(op, a, b));
        }
    }
    pdl_end(defer);
}

// Any strides, one element per thread (grid-stride).
template <typename T, int NIN, typename Op>
__global__ void __launch_bounds__(kThreads) k_ew_generic(Ptrs<T, NIN> P, EwPlan plan, int64_t n, Op op) {
    using E = Elem<T>;
    using CT = typename E::C;
    for (int64_t i = static_cast<int64_t>(blockIdx.x) * kThreads + threadIdx.x; i < n;
         i += static_cast<int64_t>(gridDim.x) * kThreads) {
        int64_t rem = i, off[2] = {0, 0};
        for (int d = plan.nd - 1; d >= 0; --d) {
            int64_t c = rem % plan.shape[d];
            rem /= plan.shape[d];
#pragma unroll
            for (int j = 0; j < NIN; ++j) off[j] += c * plan.st[j][d];
        }
        CT a = E::ld(P.in[0][off[0]]);
        CT b = NIN == 2 ? E::ld(P.in[NIN - 1][off[NIN - 1]]) : a;
        P.out[i] = E::st(apply<CT, NIN>(op, a, b));
    }
}

// ---------------------------------------------------------------------------
// Host planning
// ---------------------------------------------------------------------------

// What an elementwise launch reads (its inputs' spans) and writes, for overlap.
inline Footprint ew_footprint(const qsml_tdesc* const* ins, int nin, const qsml_tdesc* out) {
    Footprint f;
    for (int j = 0; j < nin; ++j) f.read(view_span(ins[j]));
    f.write(view_span(out));
    return f;
}

template <typename T, int NIN, typename Op>
qsml_status_t launch_ew(Context* ctx, const EwPlan& p, const qsml_tdesc* const* ins, const qsml_tdesc* out, Op op) {
    constexpr int V = Pack<T>::N;
    Ptrs<T, NIN> P;
    for (int j = 0; j < 2; ++j) P.in[j] = static_cast<const T*>(ins[j < NIN ? j : 0]->data);
    P.out = static_cast<T*>(out->data);
    int64_t n = 1;
    for (int d = 0; d < p.nd; ++d) n *= p.shape[d];
    if (n == 0) return QSML_OK;

    const int last = p.nd - 1;
    bool inner_ok = true;  // every inner stride is 0 or 1
    for (int j = 0; j < NIN; ++j)
        if (p.st[j][last] != 0 && p.st[j][last] != 1) inner_ok = false;

    if (inner_ok && p.nd == 1) {
        bool vec = aligned16(P.out);
        for (int j = 0; j < NIN; ++j)
            if (p.st[j][0] == 1 && !aligned16(P.in[j])) vec = false;
        if (vec) {
            int64_t npk = n / V;
            int64_t blocks = (npk + kThreads * kUnroll - 1) / (kThreads * kUnroll);
            if (blocks < 1) blocks = 1;
            {
                const int defer = plan_launch(ctx, ew_footprint(ins, NIN, out));
                const cudaError_t e = launch_pdl(k_ew_flat<T, NIN, Op, true>, dim3(static_cast<unsigned>(blocks)),
                                                 dim3(kThreads), 0, ctx->stream, P, p, n, op, defer);
                if (e != cudaSuccess) return check_cuda(ctx, e, "k_ew_flat");
            }
        } else {
            int64_t blocks = (n + kThreads * kUnroll - 1) / (kThreads * kUnroll);
            {
                const int defer = plan_launch(ctx, ew_footprint(ins, NIN, out));
                const cudaError_t e = launch_pdl(k_ew_flat<T, NIN, Op, false>, dim3(static_cast<unsigned>(blocks)),
                                                 dim3(kThreads), 0, ctx->stream, P, p, n, op, defer);
                if (e != cudaSuccess) return check_cuda(ctx, e, "k_ew_flat");
            }
        }
        return after_launch(ctx, "k_ew_flat");
    }

    if (inner_ok && p.shape[last] % V == 0 && aligned16(P.out)) {
        bool vec = true;
        for (int j = 0; j < NIN; ++j) {
            if (p.st[j][last] != 1) continue;
            if (!aligned16(P.in[j])) vec = false;
            for (int d = 0; d < last; ++d)
                if (p.st[j][d] % V != 0) vec = false;
        }
        if (vec) {
            int64_t cpr = p.shape[last] / V;
            int64_t items = n / V;
            int64_t blocks = (items + kThreads * kUnroll - 1) / (kThreads * kUnroll);
            bool small = items < (int64_t(1) << 31);
            for (int d = 0; d < p.nd; ++d)
                if (p.shape[d] >= (int64_t(1) << 31)) small = false;
            if (small) {
                {
                    const int defer = plan_launch(ctx, ew_footprint(ins, NIN, out));
                    const cudaError_t e = launch_pdl(k_ew_rows<T, NIN, Op, uint32_t>,
                                                     dim3(static_cast<unsigned>(blocks)), dim3(kThreads), 0,
                                                     ctx->stream, P, p, static_cast<uint32_t>(items),
                                                     static_cast<uint32_t>(cpr), op, defer);
                    if (e != cudaSuccess) return check_cuda(ctx, e, "k_ew_rows");
                }
            } else {
                {
                    const int defer = plan_launch(ctx, ew_footprint(ins, NIN, out));
                    const cudaError_t e = launch_pdl(k_ew_rows<T, NIN, Op, int64_t>,
                                                     dim3(static_cast<unsigned>(blocks)), dim3(kThreads), 0,
                                                     ctx->stream, P, p, items, cpr, op, defer);
                    if (e != cudaSuccess) return check_cuda(ctx, e, "k_ew_rows");
                }
            }
            return after_launch(ctx, "k_ew_rows");
        }
    }

    int64_t blocks = (n + kThreads - 1) / kThreads;
    int64_t cap = static_cast<int64_t>(ctx->num_sms) * 16;
    if (blocks > cap) blocks = cap;
    k_ew_generic<T, NIN, Op><<<static_cast<unsigned>(blocks), kThreads, 0, ctx->stream>>>(P, p, n, op);
    return after_launch(ctx, "k_ew_generic");
}

template <typename T, int NIN, template <int> class OpT, int... OPS>
struct OpDispatch;

template <typename T, int NIN, typename Op>
qsml_status_t run_typed(Context* ctx, const EwPlan& p, const qsml_tdesc* const* ins, const qsml_tdesc* out, Op op) {
    return launch_ew<T, NIN, Op>(ctx, p, ins, out, op);
}

template <typename T>
qsml_status_t binary_typed(Context* ctx, int op, const EwPlan& p, const qsml_tdesc* const* ins, const qsml_tdesc* out) {
    switch (op) {
        case QSML_OP_ADD: return run_typed<T, 2>(ctx, p, ins, out, BinOp<QSML_OP_ADD>());
        case QSML_OP_SUB: return run_typed<T, 2>(ctx, p, ins, out, BinOp<QSML_OP_SUB>());
        case QSML_OP_MUL: return run_typed<T, 2>(ctx, p, ins, out, BinOp<QSML_OP_MUL>());
        case QSML_OP_DIV: return run_typed<T, 2>(ctx, p, ins, out, BinOp<QSML_OP_DIV>());
        case QSML_OP_POW:
            if constexpr (std::is_same<T, int32_t>::value) return set_error(ctx, QSML_E_DTYPE, "pow needs a float dtype");
            else return run_typed<T, 2>(ctx, p, ins, out, BinOp<QSML_OP_POW>());
    }
    return set_error(ctx, QSML_E_INVALID, "unknown binary op");
}

template <typename T>
qsml_status_t scalar_typed(Context* ctx, int op, float s, const EwPlan& p, const qsml_tdesc* const* ins, const qsml_tdesc* out) {
    switch (op) {
        case QSML_OP_ADD: return run_typed<T, 1>(ctx, p, ins, out, ScalarOp<QSML_OP_ADD>{s});
        case QSML_OP_SUB: return run_typed<T, 1>(ctx, p, ins, out, ScalarOp<QSML_OP_SUB>{s});
        case QSML_OP_MUL: return run_typed<T, 1>(ctx, p, ins, out, ScalarOp<QSML_OP_MUL>{s});
        case QSML_OP_DIV: return run_typed<T, 1>(ctx, p, ins, out, ScalarOp<QSML_OP_DIV>{s});
        case QSML_OP_POW:
            if constexpr (std::is_same<T, int32_t>::value) return set_error(ctx, QSML_E_DTYPE, "pow needs a float dtype");
            else return run_typed<T, 1>(ctx, p, ins, out, ScalarOp<QSML_OP_POW>{s});
    }
    return set_error(ctx, QSML_E_INVALID, "unknown scalar op");
}

template <typename T>
qsml_status_t unary_typed(Context* ctx, int op, const EwPlan& p, const qsml_tdesc* const* ins, const qsml_tdesc* out) {
    if constexpr (std::is_same<T, int32_t>::value) {
        switch (op) {
            case QSML_UN_RELU: return run_typed<T, 1>(ctx, p, ins, out, UnOp<QSML_UN_RELU>());
            case QSML_UN_NEG: return run_typed<T, 1>(ctx, p, ins, out, UnOp<QSML_UN_NEG>());
            case QSML_UN_ABS: return run_typed<T, 1>(ctx, p, ins, out, UnOp<QSML_UN_ABS>());
        }
        return set_error(ctx, QSML_E_DTYPE, "this unary op needs a float dtype");
    } else {
        switch (op) {
            case QSML_UN_RELU: return run_typed<T, 1>(ctx, p, ins, out, UnOp<QSML_UN_RELU>());
            case QSML_UN_NEG: return run_typed<T, 1>(ctx, p, ins, out, UnOp<QSML_UN_NEG>());
            case QSML_UN_ABS: return run_typed<T, 1>(ctx, p, ins, out, UnOp<QSML_UN_ABS>());
            case QSML_UN_SQRT: return run_typed<T, 1>(ctx, p, ins, out, UnOp<QSML_UN_SQRT>());
            case QSML_UN_EXP: return run_typed<T, 1>(ctx, p, ins, out, UnOp<QSML_UN_EXP>());
            case QSML_UN_LOG: return run_typed<T, 1>(ctx, p, ins, out, UnOp<QSML_UN_LOG>());
            case QSML_UN_SIN: return run_typed<T, 1>(ctx, p, ins, out, UnOp<QSML_UN_SIN>());
            case QSML_UN_COS: return run_typed<T, 1>(ctx, p, ins, out, UnOp<QSML_UN_COS>());
            case QSML_UN_TANH: return run_typed<T, 1>(ctx, p, ins, out, UnOp<QSML_UN_TANH>());
            case QSML_UN_SIGMOID: return run_typed<T, 1>(ctx, p, ins, out, UnOp<QSML_UN_SIGMOID>());
            case QSML_UN_GELU: return run_typed<T, 1>(ctx, p, ins, out, UnOp<QSML_UN_GELU>());
        }
        return set_error(ctx, QSML_E_INVALID, "unknown unary op");
    }
}

qsml_status_t check_out(Context* ctx, const qsml_tdesc* out) {
    QSML_TRY_STATUS(check_desc(ctx, out, "out"));
    if (!is_contiguous(out)) return set_error(ctx, QSML_E_SHAPE, "out must be contiguous");
    return QSML_OK;
}

template <typename T>
__global__ void k_fill(T* p, T v, int64_t n) {
    for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < n;
         i += static_cast<int64_t>(gridDim.x) * blockDim.x)
        p[i] = v;
}

}  // namespace
}  // namespace qsml

using namespace qsml;

extern "C" {

qsml_status_t qsml_binary(qsml_ctx* handle, int32_t op, const qsml_tdesc* a, const qsml_tdesc* b,
                          const qsml_tdesc* out) {
    QSML_CTX(handle);
    QSML_TRY_STATUS(check_desc(C_, a, "a"));
    QSML_TRY_STATUS(check_desc(C_, b, "b"));
    QSML_TRY_STATUS(check_out(C_, out));
    if (a->dtype != b->dtype || a->dtype != out->dtype)
        return set_error(C_, QSML_E_DTYPE, "qsml_binary: dtypes of a, b and out must match");
    if (op < QSML_OP_ADD || op > QSML_OP_POW) return set_error(C_, QSML_E_INVALID, "qsml_binary: unknown op");
    const qsml_tdesc* ins[2] = {a, b};
    EwPlan p;
    QSML_TRY_STATUS(make_plan(C_, out, ins, 2, &p));
    switch (a->dtype) {
        case QSML_F32: return binary_typed<float>(C_, op, p, ins, out);
        case QSML_F16: return binary_typed<__half>(C_, op, p, ins, out);
        case QSML_I32: return binary_typed<int32_t>(C_, op, p, ins, out);
    }
    return set_error(C_, QSML_E_DTYPE, "qsml_binary: dtype must be F32, F16 or I32");
}

qsml_status_t qsml_binary_scalar(qsml_ctx* handle, int32_t op, const qsml_tdesc* a, float s,
                                 const qsml_tdesc* out) {
    QSML_CTX(handle);
    QSML_TRY_STATUS(check_desc(C_, a, "a"));
    QSML_TRY_STATUS(check_out(C_, out));
    if (a->dtype != out->dtype) return set_error(C_, QSML_E_DTYPE, "qsml_binary_scalar: dtype mismatch");
    if (op < QSML_OP_ADD || op > QSML_OP_POW) return set_error(C_, QSML_E_INVALID, "qsml_binary_scalar: unknown op");
    const qsml_tdesc* ins[1] = {a};
    EwPlan p;
    QSML_TRY_STATUS(make_plan(C_, out, ins, 1, &p));
    switch (a->dtype) {
        case QSML_F32: return scalar_typed<float>(C_, op, s, p, ins, out);
        case QSML_F16: return scalar_typed<__half>(C_, op, s, p, ins, out);
        case QSML_I32: return scalar_typed<int32_t>(C_, op, s, p, ins, out);
    }
    return set_error(C_, QSML_E_DTYPE, "qsml_binary_scalar: dtype must be F32, F16 or I32");
}

qsml_status_t qsml_unary(qsml_ctx* handle, int32_t op, const qsml_tdesc* a, const qsml_tdesc* out) {
    QSML_CTX(handle);
    QSML_TRY_STATUS(check_desc(C_, a, "a"));
    QSML_TRY_STATUS(check_out(C_, out));
    if (a->dtype != out->dtype) return set_error(C_, QSML_E_DTYPE, "qsml_unary: dtype mismatch");
    const qsml_tdesc* ins[1] = {a};
    EwPlan p;
    QSML_TRY_STATUS(make_plan(C_, out, ins, 1, &p));
    switch (a->dtype) {
        case QSML_F32: return unary_typed<float>(C_, op, p, ins, out);
        case QSML_F16: return unary_typed<__half>(C_, op, p, ins, out);
        case QSML_I32: return unary_typed<int32_t>(C_, op, p, ins, out);
    }
    return set_error(C_, QSML_E_DTYPE, "qsml_unary: dtype must be F32, F16 or I32");
}

qsml_status_t qsml_fill(qsml_ctx* handle, void* dst, const void* value, int32_t elem_size, int64_t count) {
    QSML_CTX(handle);
    if (count <= 0) return QSML_OK;
    if (!dst || !value) return set_error(C_, QSML_E_INVALID, "qsml_fill: null pointer");
    int64_t blocks = (count + 255) / 256;
    int64_t cap = static_cast<int64_t>(C_->num_sms) * 16;
    if (blocks > cap) blocks = cap;
    switch (elem_size) {
        case 1:
            return check_cuda(C_, cudaMemsetAsync(dst, *static_cast<const uint8_t*>(value), count, C_->stream),
                              "qsml_fill");
        case 2: {
            uint16_t v;
            std::memcpy(&v, value, 2);
            if ((reinterpret_cast<uintptr_t>(dst) & 1) != 0) return set_error(C_, QSML_E_INVALID, "qsml_fill: misaligned");
            k_fill<uint16_t><<<static_cast<unsigned>(blocks), 256, 0, C_->stream>>>(static_cast<uint16_t*>(dst), v, count);
            return after_launch(C_, "k_fill");
        }
        case 4: {
            uint32_t v;
            std::memcpy(&v, value, 4);
            if ((reinterpret_cast<uintptr_t>(dst) & 3) != 0) return set_error(C_, QSML_E_INVALID, "qsml_fill: misaligned");
            k_fill<uint32_t><<<static_cast<unsigned>(blocks), 256, 0, C_->stream>>>(static_cast<uint32_t*>(dst), v, count);
            return after_launch(C_, "k_fill");
        }
        case 8: {
            uint64_t v;
            std::memcpy(&v, value, 8);
            if ((reinterpret_cast<uintptr_t>(dst) & 7) != 0) return set_error(C_, QSML_E_INVALID, "qsml_fill: misaligned");
            k_fill<uint64_t><<<static_cast<unsigned>(blocks), 256, 0, C_->stream>>>(static_cast<uint64_t*>(dst), v, count);
            return after_launch(C_, "k_fill");
        }
    }
    return set_error(C_, QSML_E_INVALID, "qsml_fill: elem_size must be 1, 2, 4 or 8");
}

}  // extern "C"
