// Fused elementwise expressions: one kernel evaluates a whole DAG of
// elementwise ops (binary, scalar-operand, unary) over broadcast inputs,
// reading each input once and writing only the final result.
//
// Reference: every op in Ops/Elementwise.cpp:139-417 is its own dispatch
// writing a full-size intermediate, with a full barrier between dispatches;
// kernel fusion is listed as not done (README.md:78).  A chain such as
// relu(pow((A + B) * B - A, 2) / D) on [4096, 4096] moves 872 MB that way and
// ~134 MB fused.
//
// Two kernels run an expression.  Where the collapsed layout is at most 2-D
// with every input contiguous or broadcast along the inner dim, a kernel
// generated for the expression and compiled at run time (ew_jit.cu) runs it.
// Everything else, or every call when runtime compilation is unavailable or
// switched off (qsml_set_fuse_mode), runs the precompiled interpreter below:
//   * the host linearises the DAG into code for an accumulator machine: one
//     accumulator, the loaded inputs, up to three temporaries and per-
//     instruction constants.  Subtrees are ordered by their temporary need
//     (Sethi-Ullman), so most expressions need none;
//   * each instruction is one dense opcode that already names its operand
//     ("acc = acc - input 2", "acc = 0.5 * acc", "save to temp 1", ...), so
//     the kernel dispatches it with a single warp-uniform switch into an
//     unrolled loop whose registers are fixed at compile time: no data moves
//     between registers and no nested dispatch;
//   * the kernel is specialised on the number of inputs and on whether the
//     program uses temporaries, so the register file holds only what the
//     expression can touch; transcendental ops and general powers run out of
//     line (one call per element) to keep the dispatch loop small in the
//     instruction cache;
//   * each thread loads kW elements of every input (16-byte vectors on the
//     collapsed inner dim where the layout allows) before running the code;
//   * every op is the same functor the per-op kernels use and its result is
//     rounded to the storage dtype, so a fused expression is bit-identical to
//     the chain of qsml_binary / qsml_binary_scalar / qsml_unary calls.
#include "ew_common.cuh"
#include "ew_jit.cuh"

#include <vector>

namespace qsml {
namespace {

using namespace ew;

constexpr int kFThreads = 128;
constexpr int kFIn = QSML_FUSE_MAX_INPUTS;  // 6
constexpr int kFTmp = 3;
constexpr int kFInsn = 48;
constexpr int kW = 8;  // elements per thread

// Operand slots: inputs 0..5, temporaries 6..8, the instruction's constant 9.
constexpr int kSlots = kFIn + kFTmp + 1;
constexpr int kSlotTmp0 = kFIn;
constexpr int kSlotConst = kFIn + kFTmp;

// Dense opcodes.
//   [0, 80)  acc = acc OP x  or  x OP acc for OP in add/sub/mul/div:
//            code = ((reversed * 4 + OP) * kSlots + slot)
constexpr int OC_POW = 80;    // acc = pow(acc, slot `arg`)
constexpr int OC_RPOW = 81;   // acc = pow(slot `arg`, acc)
constexpr int OC_SQR = 82;    // acc = acc * acc (pow with the constant exponent 2)
constexpr int OC_RELU = 83;
constexpr int OC_NEG = 84;
constexpr int OC_ABS = 85;
constexpr int OC_SQRT = 86;
constexpr int OC_SLOW = 87;   // acc = UN_`arg`(acc): exp, log, sin, cos, tanh, sigmoid, gelu
constexpr int OC_LOAD = 88;   // + slot: acc = slot
constexpr int OC_SAVE = 98;   // + temporary: temp = acc
constexpr int OC_COUNT = 101;
static_assert(kSlots == 10 && OC_LOAD + kSlots == OC_SAVE && OC_SAVE + kFTmp == OC_COUNT, "opcode layout");

struct FuseProg {
    int n;
    uint8_t code[kFInsn];
    uint8_t arg[kFInsn];
    float cval[kFInsn];
};

template <int NIN, int NTMP> struct Regs {
    float in[NIN][kW];
    float tmp[NTMP > 0 ? NTMP : 1][kW];
    float acc[kW];
};

template <bool HALF> __device__ __forceinline__ float rnd(float x) {
    if constexpr (HALF) return __half2float(__float2half_rn(x));
    else return x;
}

// Out-of-line element ops: one copy of each transcendental in the binary.
static __device__ __noinline__ float un_slow(int op, float x) {
    switch (op) {
        case QSML_UN_EXP: return UnOp<QSML_UN_EXP>()(x);
        case QSML_UN_LOG: return UnOp<QSML_UN_LOG>()(x);
        case QSML_UN_SIN: return UnOp<QSML_UN_SIN>()(x);
        case QSML_UN_COS: return UnOp<QSML_UN_COS>()(x);
        case QSML_UN_TANH: return UnOp<QSML_UN_TANH>()(x);
        case QSML_UN_SIGMOID: return UnOp<QSML_UN_SIGMOID>()(x);
        default: return UnOp<QSML_UN_GELU>()(x);
    }
}

static __device__ __noinline__ float pow_slow(float x, float y) { return pow_f32(x, y); }

template <int OP, bool HALF, bool REV>
__device__ __forceinline__ void bin_row(float (&acc)[kW], const float (&o)[kW]) {
#pragma unroll
    for (int e = 0; e < kW; ++e) acc[e] = rnd<HALF>(REV ? BinOp<OP>()(o[e], acc[e]) : BinOp<OP>()(acc[e], o[e]));
}

template <int OP, bool HALF, bool REV>
__device__ __forceinline__ void bin_const(float (&acc)[kW], float c) {
#pragma unroll
    for (int e = 0; e < kW; ++e) acc[e] = rnd<HALF>(REV ? BinOp<OP>()(c, acc[e]) : BinOp<OP>()(acc[e], c));
}

template <int UOP, bool HALF>
__device__ __forceinline__ void un_row(float (&acc)[kW]) {
#pragma unroll
    for (int e = 0; e < kW; ++e) acc[e] = rnd<HALF>(UnOp<UOP>()(acc[e]));
}

__device__ __forceinline__ void copy_row(float (&d)[kW], const float (&s)[kW]) {
#pragma unroll
    for (int e = 0; e < kW; ++e) d[e] = s[e];
}

// Value of operand slot `slot` (runtime) into o: only the two pow opcodes
// take their operand this way.
template <int NIN, int NTMP>
__device__ __forceinline__ void fetch(const Regs<NIN, NTMP>& r, int slot, float c, float (&o)[kW]) {
#pragma unroll
    for (int e = 0; e < kW; ++e) o[e] = c;
#pragma unroll
    for (int j = 0; j < NIN; ++j)
        if (slot == j) copy_row(o, r.in[j]);
#pragma unroll
    for (int t = 0; t < NTMP; ++t)
        if (slot == kSlotTmp0 + t) copy_row(o, r.tmp[t]);
}

template <int CODE, bool HALF, int NIN, int NTMP>
__device__ __forceinline__ void exec(Regs<NIN, NTMP>& r, float c, int arg) {
    if constexpr (CODE < OC_POW) {
        constexpr int slot = CODE % kSlots;
        constexpr int op = (CODE / kSlots) % 4;
        constexpr bool rev = CODE / kSlots >= 4;
        if constexpr (slot < NIN) bin_row<op, HALF, rev>(r.acc, r.in[slot]);
        else if constexpr (slot >= kSlotTmp0 && slot < kSlotTmp0 + NTMP)
            bin_row<op, HALF, rev>(r.acc, r.tmp[slot - kSlotTmp0]);
        else if constexpr (slot == kSlotConst) bin_const<op, HALF, rev>(r.acc, c);
        // other slots are never emitted for this specialisation
    } else if constexpr (CODE == OC_POW || CODE == OC_RPOW) {
        float o[kW];
        fetch(r, arg, c, o);
#pragma unroll
        for (int e = 0; e < kW; ++e)
            r.acc[e] = rnd<HALF>(CODE == OC_POW ? pow_slow(r.acc[e], o[e]) : pow_slow(o[e], r.acc[e]));
    } else if constexpr (CODE == OC_SQR) {
#pragma unroll
        for (int e = 0; e < kW; ++e) r.acc[e] = rnd<HALF>(__fmul_rn(r.acc[e], r.acc[e]));
    } else if constexpr (CODE == OC_RELU) {
        un_row<QSML_UN_RELU, HALF>(r.acc);
    } else if constexpr (CODE == OC_NEG) {
        un_row<QSML_UN_NEG, HALF>(r.acc);
    } else if constexpr (CODE == OC_ABS) {
        un_row<QSML_UN_ABS, HALF>(r.acc);
    } else if constexpr (CODE == OC_SQRT) {
        un_row<QSML_UN_SQRT, HALF>(r.acc);
    } else if constexpr (CODE == OC_SLOW) {
#pragma unroll
        for (int e = 0; e < kW; ++e) r.acc[e] = rnd<HALF>(un_slow(arg, r.acc[e]));
    } else if constexpr (CODE < OC_SAVE) {
        constexpr int slot = CODE - OC_LOAD;
        if constexpr (slot < NIN) copy_row(r.acc, r.in[slot]);
        else if constexpr (slot >= kSlotTmp0 && slot < kSlotTmp0 + NTMP) copy_row(r.acc, r.tmp[slot - kSlotTmp0]);
        else if constexpr (slot == kSlotConst) {
#pragma unroll
            for (int e = 0; e < kW; ++e) r.acc[e] = c;
        }
    } else {
        constexpr int t = CODE - OC_SAVE;
        if constexpr (t < NTMP) copy_row(r.tmp[t], r.acc);
    }
}

// The program comes from kernel parameter space (__grid_constant__), read
// with uniform indices: every thread of the grid runs the same sequence.
template <bool HALF, int NIN, int NTMP>
__device__ __forceinline__ void run_prog(Regs<NIN, NTMP>& r, const FuseProg& p) {
    for (int i = 0; i < p.n; ++i) {
        const float c = p.cval[i];
        const int a = p.arg[i];
        switch (p.code[i]) {
#define QSML_X(n) \
    case n: exec<n, HALF, NIN, NTMP>(r, c, a); break;
#define QSML_X10(d) QSML_X(d##0) QSML_X(d##1) QSML_X(d##2) QSML_X(d##3) QSML_X(d##4) \
    QSML_X(d##5) QSML_X(d##6) QSML_X(d##7) QSML_X(d##8) QSML_X(d##9)
            QSML_X(0) QSML_X(1) QSML_X(2) QSML_X(3) QSML_X(4) QSML_X(5) QSML_X(6) QSML_X(7) QSML_X(8) QSML_X(9)
            QSML_X10(1) QSML_X10(2) QSML_X10(3) QSML_X10(4) QSML_X10(5) QSML_X10(6) QSML_X10(7) QSML_X10(8)
            QSML_X10(9) QSML_X(100)
#undef QSML_X10
#undef QSML_X
            default: break;
        }
    }
}
static_assert(OC_COUNT == 101, "the dispatch switch lists opcodes 0..100");

using FPlan = EwPlanT<kFIn>;

template <typename T> struct FPtrs {
    const T* in[kFIn];
    T* out;
};

// Registers a specialisation may use: leaves room for ~4-8 CTAs per SM.
template <int NIN, int NTMP> constexpr int min_blocks() {
    constexpr int regs = NIN * kW + NTMP * kW + kW + 40;
    constexpr int b = 65536 / (kFThreads * regs);
    return b < 2 ? 2 : (b > 8 ? 8 : b);
}

// Vector path: out is [rows, cols] (collapsed) with cols % V == 0, every
// input's inner stride 0 or 1, all extents below 2^31.  A thread takes
// U = kW / V vectors, kFThreads apart.
template <typename T, int NIN, int NTMP>
__global__ void __launch_bounds__(kFThreads, (min_blocks<NIN, NTMP>()))
    k_ew_fused_rows(FPtrs<T> P, const __grid_constant__ FPlan plan, uint32_t items, uint32_t cpr,
                    const __grid_constant__ FuseProg prog) {
    constexpr int V = Pack<T>::N;
    constexpr int U = kW / V;
    constexpr bool HALF = std::is_same<T, __half>::value;
    static_assert(kW % V == 0, "whole vectors per thread");
    Regs<NIN, NTMP> r;
    const uint32_t base = blockIdx.x * (kFThreads * U) + threadIdx.x;
#pragma unroll
    for (int u = 0; u < U; ++u) {
        const uint32_t it = base + static_cast<uint32_t>(u) * kFThreads;
        const bool ok = it < items;
        const uint32_t row = ok ? it / cpr : 0;
        const uint32_t cv = ok ? it - row * cpr : 0;
#pragma unroll
        for (int j = 0; j < NIN; ++j) {
            Pack<T> v;
            if (ok) {
                const int64_t off = row_offset<uint32_t>(plan, j, row);
                if (plan.st[j][plan.nd - 1] != 0) {
                    v = *reinterpret_cast<const Pack<T>*>(P.in[j] + off + static_cast<int64_t>(cv) * V);
                } else {
                    const T s = P.in[j][off];
#pragma unroll
                    for (int e = 0; e < V; ++e) v.v[e] = s;
                }
            } else {
#pragma unroll
                for (int e = 0; e < V; ++e) v.v[e] = T();
            }
#pragma unroll
            for (int e = 0; e < V; ++e) r.in[j][u * V + e] = Elem<T>::ld(v.v[e]);
        }
    }
    run_prog<HALF>(r, prog);
#pragma unroll
    for (int u = 0; u < U; ++u) {
        const uint32_t it = base + static_cast<uint32_t>(u) * kFThreads;
        if (it >= items) continue;
        Pack<T> o;
#pragma unroll
        for (int e = 0; e < V; ++e) o.v[e] = Elem<T>::st(r.acc[u * V + e]);
        reinterpret_cast<Pack<T>*>(P.out)[it] = o;
    }
}

// Any layout: kW elements per thread, kFThreads apart, full index
// decomposition per element and input.
template <typename T>
__global__ void __launch_bounds__(kFThreads) k_ew_fused_generic(FPtrs<T> P, const __grid_constant__ FPlan plan,
                                                                int nin, int64_t n,
                                                                const __grid_constant__ FuseProg prog) {
    constexpr bool HALF = std::is_same<T, __half>::value;
    Regs<kFIn, kFTmp> r;
    const int64_t base = static_cast<int64_t>(blockIdx.x) * (kFThreads * kW) + threadIdx.x;
#pragma unroll
    for (int e = 0; e < kW; ++e) {
        const int64_t i = base + static_cast<int64_t>(e) * kFThreads;
        int64_t off[kFIn];
#pragma unroll
        for (int j = 0; j < kFIn; ++j) off[j] = 0;
        if (i < n) {
            int64_t rem = i;
            for (int d = plan.nd - 1; d >= 0; --d) {
                const int64_t c = rem % plan.shape[d];
                rem /= plan.shape[d];
#pragma unroll
                for (int j = 0; j < kFIn; ++j) off[j] += c * plan.st[j][d];
            }
        }
#pragma unroll
        for (int j = 0; j < kFIn; ++j) r.in[j][e] = (i < n && j < nin) ? Elem<T>::ld(P.in[j][off[j]]) : 0.0f;
    }
    run_prog<HALF>(r, prog);
#pragma unroll
    for (int e = 0; e < kW; ++e) {
        const int64_t i = base + static_cast<int64_t>(e) * kFThreads;
        if (i < n) P.out[i] = Elem<T>::st(r.acc[e]);
    }
}

// ---------------------------------------------------------------------------
// Host: DAG -> accumulator code
// ---------------------------------------------------------------------------
class FuseCompiler {
public:
    FuseCompiler(Context* ctx, const qsml_fuse_node* nodes, int n, int nin)
        : ctx_(ctx), nodes_(nodes), n_(n), nin_(nin), need_(n, 0) {
        prog_.n = 0;
    }

    // Checks every node (kinds, codes, operand order, input indices).
    qsml_status_t validate() {
        for (int i = 0; i < n_; ++i) QSML_TRY_STATUS(check_node(i));
        return QSML_OK;
    }

    // Returns the interpreter program and the number of temporaries it uses
    // (after validate()).
    qsml_status_t compile(FuseProg* out, int* temps) {
        for (int i = 0; i < n_; ++i) need_[i] = need_of(i);
        if (need_[n_ - 1] > kFTmp)
            return set_error(ctx_, QSML_E_UNSUPPORTED,
                             "qsml_elementwise_fused: expression needs more than 3 temporaries");
        QSML_TRY_STATUS(gen(n_ - 1));
        *out = prog_;
        *temps = need_[n_ - 1];
        return QSML_OK;
    }

private:
    bool leaf(int i) const { return nodes_[i].kind == QSML_FUSE_INPUT || nodes_[i].kind == QSML_FUSE_CONST; }

    qsml_status_t check_node(int i) {
        const qsml_fuse_node& d = nodes_[i];
        auto bad = [&](const char* why) {
            return set_error(ctx_, QSML_E_INVALID,
                             "qsml_elementwise_fused: node " + std::to_string(i) + ": " + why);
        };
        switch (d.kind) {
            case QSML_FUSE_INPUT:
                if (d.code < 0 || d.code >= nin_) return bad("input index out of range");
                return QSML_OK;
            case QSML_FUSE_CONST: return QSML_OK;
            case QSML_FUSE_BINARY:
                if (d.code < QSML_OP_ADD || d.code > QSML_OP_POW) return bad("unknown binary op");
                if (d.a < 0 || d.a >= i || d.b < 0 || d.b >= i) return bad("operands must be earlier nodes");
                return QSML_OK;
            case QSML_FUSE_UNARY:
                if (d.code < QSML_UN_RELU || d.code > QSML_UN_GELU) return bad("unknown unary op");
                if (d.a < 0 || d.a >= i) return bad("operand must be an earlier node");
                return QSML_OK;
        }
        return bad("unknown node kind");
    }

    // Temporaries needed to evaluate node i into the accumulator.
    int need_of(int i) const {
        const qsml_fuse_node& d = nodes_[i];
        if (leaf(i)) return 0;
        if (d.kind == QSML_FUSE_UNARY) return need_[d.a];
        if (leaf(d.b)) return need_[d.a];
        if (leaf(d.a)) return need_[d.b];
        const int l = need_[d.a], r = need_[d.b];
        return l == r ? l + 1 : (l > r ? l : r);
    }

    qsml_status_t emit(int code, int arg, float cval) {
        if (prog_.n >= kFInsn)
            return set_error(ctx_, QSML_E_UNSUPPORTED, "qsml_elementwise_fused: expression too long");
        prog_.code[prog_.n] = static_cast<uint8_t>(code);
        prog_.arg[prog_.n] = static_cast<uint8_t>(arg);
        prog_.cval[prog_.n] = cval;
        ++prog_.n;
        return QSML_OK;
    }

    // Operand slot (and constant value) of a leaf.
    int leaf_slot(int i, float* c) const {
        *c = 0.0f;
        if (nodes_[i].kind == QSML_FUSE_INPUT) return nodes_[i].code;
        *c = nodes_[i].value;
        return kSlotConst;
    }

    // acc = acc OP slot (rev = false) or slot OP acc (rev = true).
    qsml_status_t emit_bin(int op, bool rev, int slot, float c) {
        if (op == QSML_OP_POW) {
            // pow(x, 2) is the single product x*x in every kernel
            if (!rev && slot == kSlotConst && c == 2.0f) return emit(OC_SQR, 0, 0.0f);
            return emit(rev ? OC_RPOW : OC_POW, slot, c);
        }
        return emit(((rev ? 4 : 0) + op) * kSlots + slot, 0, c);
    }

    qsml_status_t gen(int i) {
        const qsml_fuse_node& d = nodes_[i];
        float c;
        if (leaf(i)) {
            const int s = leaf_slot(i, &c);
            return emit(OC_LOAD + s, 0, c);
        }
        if (d.kind == QSML_FUSE_UNARY) {
            QSML_TRY_STATUS(gen(d.a));
            switch (d.code) {
                case QSML_UN_RELU: return emit(OC_RELU, 0, 0.0f);
                case QSML_UN_NEG: return emit(OC_NEG, 0, 0.0f);
                case QSML_UN_ABS: return emit(OC_ABS, 0, 0.0f);
                case QSML_UN_SQRT: return emit(OC_SQRT, 0, 0.0f);
            }
            return emit(OC_SLOW, d.code, 0.0f);
        }
        if (leaf(d.b)) {
            QSML_TRY_STATUS(gen(d.a));
            const int s = leaf_slot(d.b, &c);
            return emit_bin(d.code, false, s, c);
        }
        if (leaf(d.a)) {
            QSML_TRY_STATUS(gen(d.b));
            const int s = leaf_slot(d.a, &c);
            return emit_bin(d.code, true, s, c);
        }
        // Both operands are expressions: evaluate the hungrier one first (it
        // may use every free temporary), park it in the next temporary,
        // evaluate the other with one fewer, combine.
        const bool a_first = need_[d.a] >= need_[d.b];
        QSML_TRY_STATUS(gen(a_first ? d.a : d.b));
        const int t = tmp_used_++;
        if (t >= kFTmp) return set_error(ctx_, QSML_E_UNSUPPORTED, "qsml_elementwise_fused: out of temporaries");
        qsml_status_t st = emit(OC_SAVE + t, 0, 0.0f);
        if (st == QSML_OK) st = gen(a_first ? d.b : d.a);
        // a first: acc = tmp(a) OP acc(b); b first: acc = acc(a) OP tmp(b)
        if (st == QSML_OK) st = emit_bin(d.code, a_first, kSlotTmp0 + t, 0.0f);
        --tmp_used_;
        return st;
    }

    Context* ctx_;
    const qsml_fuse_node* nodes_;
    int n_, nin_;
    std::vector<int> need_;
    FuseProg prog_;
    int tmp_used_ = 0;
};

template <typename T, int NIN, int NTMP>
void launch_rows(Context* ctx, const FPtrs<T>& P, const FPlan& p, int64_t blocks, uint32_t items, uint32_t cpr,
                 const FuseProg& prog) {
    k_ew_fused_rows<T, NIN, NTMP><<<static_cast<unsigned>(blocks), kFThreads, 0, ctx->stream>>>(P, p, items, cpr,
                                                                                                  prog);
}

template <typename T, int NTMP>
void launch_rows_nin(Context* ctx, int nin, const FPtrs<T>& P, const FPlan& p, int64_t blocks, uint32_t items,
                     uint32_t cpr, const FuseProg& prog) {
    switch (nin) {
        case 1: launch_rows<T, 1, NTMP>(ctx, P, p, blocks, items, cpr, prog); break;
        case 2: launch_rows<T, 2, NTMP>(ctx, P, p, blocks, items, cpr, prog); break;
        case 3: launch_rows<T, 3, NTMP>(ctx, P, p, blocks, items, cpr, prog); break;
        case 4: launch_rows<T, 4, NTMP>(ctx, P, p, blocks, items, cpr, prog); break;
        default: launch_rows<T, kFIn, NTMP>(ctx, P, p, blocks, items, cpr, prog); break;
    }
}

// Every input is contiguous (stride 1, 16-byte aligned vectors) or
// broadcast (stride 0) along the collapsed inner dim, the inner extent is a
// whole number of 16-byte vectors V, and out is 16-byte aligned.
bool vector_layout(const FPlan& p, const qsml_tdesc* const* ins, int nin, const qsml_tdesc* out, int V) {
    const int last = p.nd - 1;
    bool vec = nin >= 1 && p.shape[last] % V == 0 && aligned16(out->data);
    for (int j = 0; j < nin && vec; ++j) {
        const int64_t si = p.st[j][last];
        if (si != 0 && si != 1) vec = false;
        if (si == 1) {
            if (!aligned16(ins[j]->data)) vec = false;
            for (int d = 0; d < last; ++d)
                if (p.st[j][d] % V != 0) vec = false;
        }
    }
    return vec;
}

template <typename T>
qsml_status_t launch_fused(Context* ctx, const FPlan& p, const qsml_tdesc* const* ins, int nin, const qsml_tdesc* out,
                           const FuseProg& prog, int temps) {
    constexpr int V = Pack<T>::N;
    FPtrs<T> P;
    for (int j = 0; j < kFIn; ++j) P.in[j] = static_cast<const T*>(ins[j < nin ? j : 0]->data);
    P.out = static_cast<T*>(out->data);
    int64_t n = 1;
    for (int d = 0; d < p.nd; ++d) n *= p.shape[d];
    if (n == 0) return QSML_OK;
    const int last = p.nd - 1;
    const bool vec = vector_layout(p, ins, nin, out, V);
    constexpr int U = kW / V;
    if (vec && n + int64_t(kFThreads) * kW < (int64_t(1) << 31)) {
        const int64_t items = n / V;
        const int64_t cpr = p.shape[last] / V;
        const int64_t blocks = (items + kFThreads * U - 1) / (kFThreads * U);
        if (temps == 0)
            launch_rows_nin<T, 0>(ctx, nin, P, p, blocks, static_cast<uint32_t>(items), static_cast<uint32_t>(cpr), prog);
        else
            launch_rows_nin<T, kFTmp>(ctx, nin, P, p, blocks, static_cast<uint32_t>(items), static_cast<uint32_t>(cpr),
                                      prog);
        return after_launch(ctx, "k_ew_fused_rows");
    }
    const int64_t blocks = (n + kFThreads * kW - 1) / (kFThreads * kW);
    if (blocks > INT32_MAX) return set_error(ctx, QSML_E_UNSUPPORTED, "qsml_elementwise_fused: too large");
    k_ew_fused_generic<T><<<static_cast<unsigned>(blocks), kFThreads, 0, ctx->stream>>>(P, p, nin, n, prog);
    return after_launch(ctx, "k_ew_fused_generic");
}

}  // namespace
}  // namespace qsml

using namespace qsml;

extern "C" qsml_status_t qsml_elementwise_fused(qsml_ctx* handle, const qsml_fuse_node* nodes, int32_t n_nodes,
                                                const qsml_tdesc* inputs, int32_t n_inputs, const qsml_tdesc* out) {
    QSML_CTX(handle);
    if (!nodes || n_nodes < 1 || n_nodes > QSML_FUSE_MAX_NODES)
        return set_error(C_, QSML_E_INVALID, "qsml_elementwise_fused: need 1 to 64 nodes");
    if (n_inputs < 0 || n_inputs > QSML_FUSE_MAX_INPUTS || (n_inputs > 0 && !inputs))
        return set_error(C_, QSML_E_INVALID, "qsml_elementwise_fused: need 0 to 6 inputs");
    QSML_TRY_STATUS(check_desc(C_, out, "out"));
    if (!is_contiguous(out)) return set_error(C_, QSML_E_SHAPE, "qsml_elementwise_fused: out must be contiguous");
    if (out->dtype != QSML_F32 && out->dtype != QSML_F16)
        return set_error(C_, QSML_E_DTYPE, "qsml_elementwise_fused: dtype must be F32 or F16");
    const qsml_tdesc* ins[kFIn];
    for (int j = 0; j < n_inputs; ++j) {
        QSML_TRY_STATUS(check_desc(C_, &inputs[j], "input"));
        if (inputs[j].dtype != out->dtype)
            return set_error(C_, QSML_E_DTYPE, "qsml_elementwise_fused: inputs and out must share one dtype");
        ins[j] = &inputs[j];
    }
    FuseCompiler comp(C_, nodes, n_nodes, n_inputs);
    QSML_TRY_STATUS(comp.validate());
    FPlan p;
    QSML_TRY_STATUS(make_plan(C_, out, ins, n_inputs, &p));
    if (numel(out) == 0) return QSML_OK;
    const bool half = out->dtype == QSML_F16;
    if (C_->fuse_mode != QSML_FUSE_MODE_INTERP) {
        const int V = half ? 8 : 4;
        bool ran = false;
        if (p.nd <= 2 && vector_layout(p, ins, n_inputs, out, V)) {
            JitInput jin[kFIn];
            for (int j = 0; j < n_inputs; ++j)
                jin[j] = JitInput{ins[j]->data, p.nd == 2 ? p.st[j][0] : 0, p.st[j][p.nd - 1] == 1};
            QSML_TRY_STATUS(fused_jit(C_, nodes, n_nodes, jin, n_inputs, half, out->data, numel(out) / V,
                                      p.shape[p.nd - 1] / V, &ran));
        }
        if (ran) {
            C_->fuse_jit_launches++;
            return QSML_OK;
        }
        if (C_->fuse_mode == QSML_FUSE_MODE_JIT)
            return set_error(C_, QSML_E_UNSUPPORTED,
                             "qsml_elementwise_fused: no runtime-compiled kernel for this layout or no NVRTC");
    }
    FuseProg prog;
    int temps = 0;
    QSML_TRY_STATUS(comp.compile(&prog, &temps));
    if (n_inputs == 0) ins[0] = out;  // pointer placeholder; no input is read
    C_->fuse_interp_launches++;
    if (!half) return launch_fused<float>(C_, p, ins, n_inputs, out, prog, temps);
    return launch_fused<__half>(C_, p, ins, n_inputs, out, prog, temps);
}

extern "C" qsml_status_t qsml_set_fuse_mode(qsml_ctx* handle, int32_t mode) {
    QSML_CTX(handle);
    if (mode < QSML_FUSE_MODE_AUTO || mode > QSML_FUSE_MODE_JIT)
        return set_error(C_, QSML_E_INVALID, "qsml_set_fuse_mode: unknown mode");
    C_->fuse_mode = mode;
    return QSML_OK;
}

extern "C" qsml_status_t qsml_fuse_stats(qsml_ctx* handle, uint64_t* jit_launches, uint64_t* interp_launches,
                                         uint64_t* jit_kernels) {
    QSML_CTX(handle);
    if (jit_launches) *jit_launches = C_->fuse_jit_launches;
    if (interp_launches) *interp_launches = C_->fuse_interp_launches;
    if (jit_kernels) *jit_kernels = fused_jit_kernels();
    return QSML_OK;
}
