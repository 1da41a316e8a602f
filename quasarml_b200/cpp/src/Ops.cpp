// QuasarML::Ops over libqsml_cuda.so.  Each op allocates its result (the
// reference's convention, e.g. Ops/Elementwise.cpp:143), builds descriptors
// and makes one C ABI call; a nonzero status becomes std::runtime_error.
// View ops (reshape, transpose, slice, squeeze, unsqueeze) return zero-copy
// strided tensors sharing the input's storage.
#include <algorithm>
#include <numeric>

#include "Common/Assert.h"
#include "Core/Device.h"
#include "Core/Tensor.h"
#include "Ops/Elementwise.h"
#include "Ops/LinAlg.h"
#include "Ops/Manipulation.h"
#include "Ops/Reduction.h"

namespace QuasarML {
namespace Ops {

namespace {

using TP = std::shared_ptr<Tensor>;

// NumPy broadcasting of two shapes (the reference only has the one-sided
// Tensor::is_broadcastable test, Core/Tensor.cpp:142-151).
std::vector<u32> broadcast_shape(const std::vector<u32>& a, const std::vector<u32>& b) {
    const size_t n = std::max(a.size(), b.size());
    std::vector<u32> out(n);
    for (size_t i = 0; i < n; ++i) {
        const long ia = static_cast<long>(a.size() + i) - static_cast<long>(n);
        const long ib = static_cast<long>(b.size() + i) - static_cast<long>(n);
        const u32 da = ia >= 0 ? a[ia] : 1, db = ib >= 0 ? b[ib] : 1;
        QS_ASSERT(da == db || da == 1 || db == 1, "Shapes " + shape_to_string(a) + " and " + shape_to_string(b) +
                                                      " do not broadcast");
        out[i] = da == 1 ? db : da;
    }
    return out;
}

// ---- deferred (fused) elementwise ops ---------------------------------------
// An operand is spliced into the new expression: a deferred tensor brings its
// nodes (its inputs merged into the new input list), a materialised one
// becomes an input node.  An expression that would exceed the fused entry
// point's limits evaluates its largest deferred operand first.
class ExprBuilder {
public:
    ExprBuilder() : e_(std::make_shared<LazyExpr>()) {}

    int operand(const TP& t) {
        if (!t->is_lazy()) return add({QSML_FUSE_INPUT, input_index(t), 0, 0, 0.0f});
        const LazyExpr& src = *t->lazy_expr();
        std::vector<int> remap(src.inputs.size());
        for (size_t j = 0; j < src.inputs.size(); ++j) remap[j] = input_index(src.inputs[j]);
        const int base = static_cast<int>(e_->nodes.size());
        for (qsml_fuse_node n : src.nodes) {
            if (n.kind == QSML_FUSE_INPUT) n.code = remap[n.code];
            if (n.kind == QSML_FUSE_BINARY || n.kind == QSML_FUSE_UNARY) n.a += base;
            if (n.kind == QSML_FUSE_BINARY) n.b += base;
            e_->nodes.push_back(n);
        }
        return static_cast<int>(e_->nodes.size()) - 1;
    }
    int constant(f32 v) { return add({QSML_FUSE_CONST, 0, 0, 0, v}); }
    int binary(int op, int a, int b) { return add({QSML_FUSE_BINARY, op, a, b, 0.0f}); }
    int unary(int op, int a) { return add({QSML_FUSE_UNARY, op, a, 0, 0.0f}); }

    bool fits() const {
        return e_->nodes.size() <= QSML_FUSE_MAX_NODES && e_->inputs.size() <= QSML_FUSE_MAX_INPUTS;
    }
    std::shared_ptr<LazyExpr> expr() const { return e_; }

private:
    int add(qsml_fuse_node n) {
        e_->nodes.push_back(n);
        return static_cast<int>(e_->nodes.size()) - 1;
    }
    int input_index(const TP& t) {
        for (size_t j = 0; j < e_->inputs.size(); ++j)
            if (e_->inputs[j] == t) return static_cast<int>(j);
        e_->inputs.push_back(t);
        return static_cast<int>(e_->inputs.size()) - 1;
    }
    std::shared_ptr<LazyExpr> e_;
};

bool deferrable(const Device& device, const TP& t) {
    return device.defer_elementwise() && (t->dtype() == DataType::F32 || t->dtype() == DataType::F16);
}

TP make_deferred(Device& device, const std::vector<u32>& shape, DataType dtype, const std::shared_ptr<LazyExpr>& e) {
    auto out = std::make_shared<Tensor>(&device, shape, dtype, e);
    out->register_reads();
    return out;
}

// Builds `build(builder, operand node indices...)`; if the result does not
// fit, evaluates the deferred operands (largest first) and retries.
template <typename Build>
std::shared_ptr<LazyExpr> build_expr(std::vector<TP> ops, Build build) {
    for (;;) {
        ExprBuilder b;
        std::vector<int> idx;
        for (const auto& t : ops) idx.push_back(b.operand(t));
        build(b, idx);
        if (b.fits()) return b.expr();
        size_t big = 0, best = 0;
        for (size_t i = 0; i < ops.size(); ++i)
            if (ops[i]->is_lazy() && ops[i]->lazy_expr()->nodes.size() >= best) {
                best = ops[i]->lazy_expr()->nodes.size();
                big = i;
            }
        QS_ASSERT(ops[big]->is_lazy(), "fused expression limits exceeded");
        ops[big]->materialize();
    }
}

TP binary(Device& device, int op, const TP& a, const TP& b) {
    QS_ASSERT(a && b, "null tensor");
    QS_ASSERT(a->dtype() == b->dtype(), "Type mismatch");
    if (deferrable(device, a)) {
        auto shape = broadcast_shape(a->shape(), b->shape());
        auto e = build_expr({a, b}, [op](ExprBuilder& bl, const std::vector<int>& i) { bl.binary(op, i[0], i[1]); });
        return make_deferred(device, shape, a->dtype(), e);
    }
    auto out = device.create_tensor(broadcast_shape(a->shape(), b->shape()), a->dtype());
    qsml_tdesc da = a->desc(), db = b->desc(), dout = out->desc();
    device.check(qsml_binary(device.ctx(), op, &da, &db, &dout));
    return out;
}

TP scalar_op(Device& device, int op, const TP& a, f32 s) {
    QS_ASSERT(a, "null tensor");
    if (deferrable(device, a)) {
        auto e = build_expr({a}, [op, s](ExprBuilder& bl, const std::vector<int>& i) {
            bl.binary(op, i[0], bl.constant(s));
        });
        return make_deferred(device, a->shape(), a->dtype(), e);
    }
    auto out = device.create_tensor(a->shape(), a->dtype());
    qsml_tdesc da = a->desc(), dout = out->desc();
    device.check(qsml_binary_scalar(device.ctx(), op, &da, s, &dout));
    return out;
}

TP unary(Device& device, int op, const TP& a) {
    QS_ASSERT(a, "null tensor");
    if (deferrable(device, a)) {
        auto e = build_expr({a}, [op](ExprBuilder& bl, const std::vector<int>& i) { bl.unary(op, i[0]); });
        return make_deferred(device, a->shape(), a->dtype(), e);
    }
    auto out = device.create_tensor(a->shape(), a->dtype());
    qsml_tdesc da = a->desc(), dout = out->desc();
    device.check(qsml_unary(device.ctx(), op, &da, &dout));
    return out;
}

i32 norm_axis(i32 axis, u32 rank) {
    if (axis < 0) axis += static_cast<i32>(rank);
    QS_ASSERT(axis >= 0 && axis < static_cast<i32>(rank), "Invalid axis");
    return axis;
}

// Ops/Reduction.cpp:297-305: the axis is dropped (kept as 1 with keepdims);
// reducing the only axis gives shape [1].
std::vector<u32> reduced_shape(const std::vector<u32>& s, i32 axis, bool keepdims) {
    std::vector<u32> out;
    for (i32 i = 0; i < static_cast<i32>(s.size()); ++i) {
        if (i == axis) {
            if (keepdims) out.push_back(1);
        } else {
            out.push_back(s[i]);
        }
    }
    if (out.empty()) out.push_back(1);
    return out;
}

// Views (slices with a step, transposes) are reduced in place; only a view
// whose dims the library cannot collapse (QSML_E_UNSUPPORTED) is gathered
// into a contiguous copy first.
void reduce_into(Device& device, int op, const TP& a, int32_t axis, bool keepdims, const TP& out) {
    a->materialize();
    qsml_tdesc dx = a->desc(), dout = out->desc();
    int st = qsml_reduce(device.ctx(), op, &dx, axis, keepdims ? 1 : 0, &dout);
    if (st == QSML_E_UNSUPPORTED && !a->is_contiguous()) {
        auto x = a->contiguous();
        dx = x->desc();
        st = qsml_reduce(device.ctx(), op, &dx, axis, keepdims ? 1 : 0, &dout);
    }
    device.check(st);
}

TP reduce_all(Device& device, int op, const TP& a) {
    QS_ASSERT(a, "null tensor");
    auto out = device.create_tensor({1}, a->dtype());
    reduce_into(device, op, a, QSML_AXIS_ALL, false, out);
    return out;
}

TP reduce_axis(Device& device, int op, const TP& a, i32 axis, bool keepdims) {
    QS_ASSERT(a, "null tensor");
    axis = norm_axis(axis, a->rank());
    auto out = device.create_tensor(reduced_shape(a->shape(), axis, keepdims), a->dtype());
    reduce_into(device, op, a, axis, keepdims, out);
    return out;
}

// Unit last-dim stride for matmul operands (other strides are passed through).
TP unit_inner(const TP& t) {
    const auto st = t->strides();
    if (t->shape().back() == 1 || st.back() == 1) return t;
    return t->contiguous();
}

}  // namespace

// ---- elementwise ------------------------------------------------------------
TP add(Device& d, TP a, TP b) { return binary(d, QSML_OP_ADD, a, b); }
TP subtract(Device& d, TP a, TP b) { return binary(d, QSML_OP_SUB, a, b); }
TP multiply(Device& d, TP a, TP b) { return binary(d, QSML_OP_MUL, a, b); }
TP divide(Device& d, TP a, TP b) { return binary(d, QSML_OP_DIV, a, b); }
TP pow(Device& d, TP a, TP e) { return binary(d, QSML_OP_POW, a, e); }
TP pow(Device& d, TP a, f32 e) { return scalar_op(d, QSML_OP_POW, a, e); }
TP add_scalar(Device& d, TP a, f32 s) { return scalar_op(d, QSML_OP_ADD, a, s); }
TP multiply_scalar(Device& d, TP a, f32 s) { return scalar_op(d, QSML_OP_MUL, a, s); }
TP neg(Device& d, TP a) { return unary(d, QSML_UN_NEG, a); }
TP abs(Device& d, TP a) { return unary(d, QSML_UN_ABS, a); }
TP sqrt(Device& d, TP a) { return unary(d, QSML_UN_SQRT, a); }
TP exp(Device& d, TP a) { return unary(d, QSML_UN_EXP, a); }
TP log(Device& d, TP a) { return unary(d, QSML_UN_LOG, a); }
TP sin(Device& d, TP a) { return unary(d, QSML_UN_SIN, a); }
TP cos(Device& d, TP a) { return unary(d, QSML_UN_COS, a); }
TP tanh(Device& d, TP a) { return unary(d, QSML_UN_TANH, a); }
TP relu(Device& d, TP a) { return unary(d, QSML_UN_RELU, a); }
TP sigmoid(Device& d, TP a) { return unary(d, QSML_UN_SIGMOID, a); }
TP gelu(Device& d, TP a) { return unary(d, QSML_UN_GELU, a); }

// Ops/Elementwise.cpp:395-417: exp(x - max) / sum(exp(x - max)) over `axis`
// (any axis here), one kernel.
TP softmax(Device& d, TP a, i32 axis) {
    QS_ASSERT(a, "null tensor");
    axis = norm_axis(axis, a->rank());
    auto x = a->contiguous();
    auto out = d.create_tensor(a->shape(), a->dtype());
    qsml_tdesc dx = x->desc(), dout = out->desc();
    d.check(qsml_softmax(d.ctx(), &dx, axis, &dout));
    return out;
}

// ---- reductions -------------------------------------------------------------
TP sum(Device& d, TP a) { return reduce_all(d, QSML_RED_SUM, a); }
TP sum(Device& d, TP a, i32 axis, bool keepdims) { return reduce_axis(d, QSML_RED_SUM, a, axis, keepdims); }
TP mean(Device& d, TP a) { return reduce_all(d, QSML_RED_MEAN, a); }
TP mean(Device& d, TP a, i32 axis, bool keepdims) { return reduce_axis(d, QSML_RED_MEAN, a, axis, keepdims); }
TP max(Device& d, TP a) { return reduce_all(d, QSML_RED_MAX, a); }
TP max(Device& d, TP a, i32 axis, bool keepdims) { return reduce_axis(d, QSML_RED_MAX, a, axis, keepdims); }
TP min(Device& d, TP a) { return reduce_all(d, QSML_RED_MIN, a); }
TP min(Device& d, TP a, i32 axis, bool keepdims) { return reduce_axis(d, QSML_RED_MIN, a, axis, keepdims); }
TP prod(Device& d, TP a) { return reduce_all(d, QSML_RED_PROD, a); }

// The reference's argmax/argmin (Ops/Reduction.cpp:388-396) ignore the axis
// and return max/min values.  These return I32 indices over `axis` (the axis
// is dropped from the shape): the first index of the largest (smallest)
// value, a NaN counting as beyond every number.
TP arg_reduce(Device& device, int op, const TP& a, i32 axis) {
    QS_ASSERT(a, "null tensor");
    axis = norm_axis(axis, a->rank());
    QS_ASSERT(a->dim(axis) > 0, "argmax/argmin of an empty axis");
    auto out = device.create_tensor(reduced_shape(a->shape(), axis, false), DataType::I32);
    // a transpose is read in place; other views are gathered first
    a->materialize();
    qsml_tdesc dx = a->desc(), dout = out->desc();
    int st = qsml_arg_reduce(device.ctx(), op, &dx, axis, 0, &dout);
    if (st == QSML_E_UNSUPPORTED && !a->is_contiguous()) {
        auto x = a->contiguous();
        dx = x->desc();
        st = qsml_arg_reduce(device.ctx(), op, &dx, axis, 0, &dout);
    }
    device.check(st);
    return out;
}
TP argmax(Device& d, TP a, i32 axis) { return arg_reduce(d, QSML_ARG_MAX, a, axis); }
TP argmin(Device& d, TP a, i32 axis) { return arg_reduce(d, QSML_ARG_MIN, a, axis); }

// ---- linear algebra ---------------------------------------------------------
TP matmul(Device& d, TP a, TP b) { return matmul(d, a, b, a->dtype()); }

TP matmul(Device& d, TP a, TP b, DataType out_dtype) {
    QS_ASSERT(a->rank() == 2 && b->rank() == 2, "matmul requires 2D tensors");
    QS_ASSERT(a->dim(1) == b->dim(0), "Inner dimensions must match");
    QS_ASSERT(a->dtype() == b->dtype(), "Type mismatch");
    auto A = unit_inner(a), B = unit_inner(b);
    auto C = d.create_tensor({a->dim(0), b->dim(1)}, out_dtype);
    qsml_tdesc da = A->desc(), db = B->desc(), dc = C->desc();
    d.check(qsml_matmul(d.ctx(), &da, &db, &dc, QSML_MM_AUTO));
    return C;
}

TP batch_matmul(Device& d, TP a, TP b) {
    QS_ASSERT(a->rank() == 3 && b->rank() == 3, "batch_matmul requires 3D tensors");
    QS_ASSERT(a->dim(0) == b->dim(0), "Batch size must match");
    QS_ASSERT(a->dim(2) == b->dim(1), "Inner dimensions must match");
    QS_ASSERT(a->dtype() == b->dtype(), "Type mismatch");
    auto A = unit_inner(a), B = unit_inner(b);
    auto C = d.create_tensor({a->dim(0), a->dim(1), b->dim(2)}, a->dtype());
    qsml_tdesc da = A->desc(), db = B->desc(), dc = C->desc();
    d.check(qsml_matmul(d.ctx(), &da, &db, &dc, QSML_MM_AUTO));
    return C;
}

TP dot(Device& d, TP a, TP b) {
    QS_ASSERT(a->numel() == b->numel(), "Tensors must have same number of elements");
    QS_ASSERT(a->dtype() == b->dtype(), "Type mismatch");
    return sum(d, multiply(d, a->contiguous()->flatten(), b->contiguous()->flatten()));
}

TP transpose(Device& d, TP a) {
    QS_ASSERT(a->rank() == 2, "transpose requires 2D tensor");
    return transpose(d, a, 0, 1);
}

// A view with two dims exchanged (the reference ignores dim0/dim1,
// Ops/LinAlg.cpp:348-351).
TP transpose(Device&, TP a, i32 dim0, i32 dim1) {
    dim0 = norm_axis(dim0, a->rank());
    dim1 = norm_axis(dim1, a->rank());
    auto shape = a->shape();
    auto st = a->strides();
    std::swap(shape[dim0], shape[dim1]);
    std::swap(st[dim0], st[dim1]);
    return a->strided_view(shape, st, a->element_offset());
}

TP outer(Device& d, TP a, TP b) {
    QS_ASSERT(a->rank() == 1 && b->rank() == 1, "outer requires 1D tensors");
    QS_ASSERT(a->dtype() == b->dtype(), "Type mismatch");
    auto col = a->strided_view({a->dim(0), 1}, {a->strides()[0], 1}, a->element_offset());
    auto row = b->strided_view({1, b->dim(0)}, {1, b->strides()[0]}, b->element_offset());
    return multiply(d, col, row);
}

TP layer_norm(Device& d, TP x, TP gamma, TP beta, f32 eps) {
    auto X = x->contiguous(), G = gamma->contiguous(), B = beta->contiguous();
    auto Y = d.create_tensor(x->shape(), x->dtype());
    qsml_tdesc dx = X->desc(), dg = G->desc(), db = B->desc(), dy = Y->desc();
    d.check(qsml_layer_norm(d.ctx(), &dx, &dg, &db, eps, &dy));
    return Y;
}

// ---- manipulation -----------------------------------------------------------
TP reshape(Device&, TP a, const std::vector<u32>& new_shape) {
    QS_ASSERT(compute_numel(new_shape) == a->numel(), "Element count mismatch");
    return a->contiguous()->view(new_shape);
}

TP flatten(Device&, TP a) { return a->contiguous()->flatten(); }

TP squeeze(Device&, TP a) {
    std::vector<u32> shape;
    std::vector<u64> st;
    for (u32 i = 0; i < a->rank(); ++i) {
        if (a->dim(i) == 1) continue;
        shape.push_back(a->dim(i));
        st.push_back(a->strides()[i]);
    }
    if (shape.empty()) {
        shape.push_back(1);
        st.push_back(1);
    }
    return a->strided_view(shape, st, a->element_offset());
}

TP squeeze(Device&, TP a, i32 dim) {
    dim = norm_axis(dim, a->rank());
    QS_ASSERT(a->dim(dim) == 1, "Dimension is not 1");
    auto shape = a->shape();
    auto st = a->strides();
    shape.erase(shape.begin() + dim);
    st.erase(st.begin() + dim);
    if (shape.empty()) {
        shape.push_back(1);
        st.push_back(1);
    }
    return a->strided_view(shape, st, a->element_offset());
}

TP unsqueeze(Device&, TP a, i32 dim) {
    if (dim < 0) dim = static_cast<i32>(a->rank()) + dim + 1;
    QS_ASSERT(dim >= 0 && dim <= static_cast<i32>(a->rank()), "Invalid dim");
    auto shape = a->shape();
    auto st = a->strides();
    const u64 s = dim < static_cast<i32>(st.size()) ? st[dim] * shape[dim] : 1;
    shape.insert(shape.begin() + dim, 1);
    st.insert(st.begin() + dim, s);
    return a->strided_view(shape, st, a->element_offset());
}

TP concat(Device& d, const std::vector<TP>& tensors, i32 axis) {
    QS_ASSERT(!tensors.empty(), "Empty tensor list");
    const auto& first = tensors[0];
    axis = norm_axis(axis, first->rank());
    u32 total = 0;
    for (const auto& t : tensors) {
        QS_ASSERT(t->rank() == first->rank(), "Rank mismatch");
        QS_ASSERT(t->dtype() == first->dtype(), "Type mismatch");
        for (u32 i = 0; i < t->rank(); ++i)
            if (static_cast<i32>(i) != axis) QS_ASSERT(t->dim(i) == first->dim(i), "Shape mismatch off the concat axis");
        total += t->dim(axis);
    }
    auto shape = first->shape();
    shape[axis] = total;
    auto out = d.create_tensor(shape, first->dtype());
    const auto ost = out->strides();
    u64 off = 0;
    for (const auto& t : tensors) {
        auto part_shape = shape;
        part_shape[axis] = t->dim(axis);
        auto part = out->strided_view(part_shape, ost, off * ost[axis]);
        qsml_tdesc ds = t->desc(), dp = part->desc();
        d.check(qsml_gather(d.ctx(), &ds, &dp));
        off += t->dim(axis);
    }
    return out;
}

TP stack(Device& d, const std::vector<TP>& tensors, i32 axis) {
    QS_ASSERT(!tensors.empty(), "Empty tensor list");
    const auto& first = tensors[0];
    for (const auto& t : tensors) {
        QS_ASSERT(t->shape() == first->shape(), "Shape mismatch");
        QS_ASSERT(t->dtype() == first->dtype(), "Type mismatch");
    }
    if (axis < 0) axis += static_cast<i32>(first->rank()) + 1;
    QS_ASSERT(axis >= 0 && axis <= static_cast<i32>(first->rank()), "Invalid axis");
    auto shape = first->shape();
    shape.insert(shape.begin() + axis, static_cast<u32>(tensors.size()));
    auto out = d.create_tensor(shape, first->dtype());
    auto st = out->strides();
    const u64 step = st[axis];
    st.erase(st.begin() + axis);
    for (size_t i = 0; i < tensors.size(); ++i) {
        auto part = out->strided_view(first->shape(), st, i * step);
        qsml_tdesc ds = tensors[i]->desc(), dp = part->desc();
        d.check(qsml_gather(d.ctx(), &ds, &dp));
    }
    return out;
}

TP slice(Device& d, TP a, i32 axis, u64 start, u64 end) { return slice(d, a, axis, start, end, 1); }

// A strided view of elements start, start+step, ... < end along `axis`
// (the reference copies one byte range through the host and ignores the
// axis, Ops/Manipulation.cpp:146-161).
TP slice(Device&, TP a, i32 axis, u64 start, u64 end, u64 step) {
    axis = norm_axis(axis, a->rank());
    QS_ASSERT(step >= 1, "slice step must be positive");
    QS_ASSERT(start < end && end <= a->dim(axis), "Invalid slice range");
    auto shape = a->shape();
    auto st = a->strides();
    shape[axis] = static_cast<u32>((end - start + step - 1) / step);
    const u64 offset = a->element_offset() + start * st[axis];
    st[axis] *= step;
    return a->strided_view(shape, st, offset);
}

TP broadcast_to(Device& d, TP a, const std::vector<u32>& shape) {
    QS_ASSERT(a->is_broadcastable(shape), "Cannot broadcast to shape");
    std::vector<u64> st(shape.size(), 0);
    const size_t diff = shape.size() - a->rank();
    for (size_t i = 0; i < a->rank(); ++i)
        st[diff + i] = (a->dim(static_cast<u32>(i)) == 1 && shape[diff + i] != 1) ? 0 : a->strides()[i];
    auto src = a->strided_view(shape, st, a->element_offset());
    auto out = d.create_tensor(shape, a->dtype());
    qsml_tdesc ds = src->desc(), dout = out->desc();
    d.check(qsml_gather(d.ctx(), &ds, &dout));
    return out;
}

TP copy(Device& d, TP a) {
    auto out = d.create_tensor(a->shape(), a->dtype());
    qsml_tdesc ds = a->desc(), dout = out->desc();
    d.check(qsml_gather(d.ctx(), &ds, &dout));
    return out;
}

TP contiguous(Device&, TP a) { return a->contiguous(); }

TP cast(Device& d, TP a, DataType dtype) {
    QS_ASSERT(a, "null tensor");
    auto x = a->contiguous();
    auto out = d.create_tensor(a->shape(), dtype);
    qsml_tdesc dx = x->desc(), dout = out->desc();
    d.check(qsml_cast(d.ctx(), &dx, &dout));
    return out;
}

}  // namespace Ops
}  // namespace QuasarML
