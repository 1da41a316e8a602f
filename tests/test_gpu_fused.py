"""Fused elementwise expressions (qsml_elementwise_fused).

1. relu(pow((A+B)*B - A, 2) / D) at 4096x4096, B[1,4096], D[4096,1] in one
   launch: bit-identical to the oracle's op-by-op chain.
2. Random expression DAGs (1-4 broadcast inputs, binary, scalar and unary
   nodes, shared subexpressions) in F32 and F16: bit-identical to the same
   sequence of unfused qsml_binary / qsml_binary_scalar / qsml_unary calls,
   which is the contract of the fused entry point.
3. Layouts that leave the vector path (strided views, odd inner extents,
   1-D), expressions that need temporaries, and the error statuses.
"""
import numpy as np
import pytest

from helpers import assert_bits_equal, d, dev, empty, host
from quasarml_b200 import abi, datagen

pytestmark = pytest.mark.gpu


@pytest.fixture
def mode(ctx, request):
    """Runs the test with the fuse mode given by the parameter, then restores AUTO."""
    ctx.set_fuse_mode(request.param)
    yield request.param
    ctx.set_fuse_mode(abi.FUSE_MODE_AUTO)


@pytest.mark.parametrize("mode", [abi.FUSE_MODE_AUTO, abi.FUSE_MODE_INTERP], indirect=True)
def test_chain_4096_one_launch_bitexact(ctx, orc, mode):
    A = datagen.uniform(datagen.SEEDS["ew_A"], (4096, 4096), -1.0, 1.0)
    B = datagen.uniform(datagen.SEEDS["ew_B"], (1, 4096), -1.0, 1.0)
    D = datagen.uniform(datagen.SEEDS["ew_D"], (4096, 1), 0.5, 2.0)
    tA, tB, tD = dev(A), dev(B), dev(D)
    out = empty((4096, 4096), np.float32)
    e = abi.Expr()
    a, b, dd = e.input(0), e.input(1), e.input(2)
    t = e.binary(abi.OP_SUB, e.binary(abi.OP_MUL, e.binary(abi.OP_ADD, a, b), b), a)
    e.unary(abi.UN_RELU, e.binary(abi.OP_DIV, e.binary(abi.OP_POW, t, e.const(2.0)), dd))
    n0 = ctx.launch_count()
    j0, i0, _ = ctx.fuse_stats()
    ctx.elementwise_fused(e.nodes, [d(tA), d(tB), d(tD)], d(out))
    assert ctx.launch_count() - n0 == 1
    j1, i1, _ = ctx.fuse_stats()
    # AUTO runs the runtime-compiled kernel for this 2-D layout
    assert (j1 - j0, i1 - i0) == ((1, 0) if mode == abi.FUSE_MODE_AUTO else (0, 1))
    r = orc.relu(orc.binary(orc.DIV, orc.pow_scalar(orc.binary(orc.SUB, orc.binary(orc.MUL, orc.binary(
        orc.ADD, A, B), B), A), 2.0), D))
    assert_bits_equal(host(out), r, "fused chain")


# ---------------------------------------------------------------------------
# Random DAGs against the unfused calls
# ---------------------------------------------------------------------------
BIN = [abi.OP_ADD, abi.OP_SUB, abi.OP_MUL, abi.OP_DIV, abi.OP_POW]
UN = [abi.UN_RELU, abi.UN_NEG, abi.UN_ABS, abi.UN_SQRT, abi.UN_EXP, abi.UN_LOG, abi.UN_SIN, abi.UN_COS,
      abi.UN_TANH, abi.UN_SIGMOID, abi.UN_GELU]


def random_expr(rng, n_inputs, n_ops):
    """Node list whose operands are earlier nodes; constants only as the
    right operand of a binary node (what qsml_binary_scalar expresses)."""
    e = abi.Expr()
    vals = [e.input(j) for j in range(n_inputs)]
    for _ in range(n_ops):
        r = rng.random()
        x = vals[rng.integers(0, len(vals))]
        if r < 0.25:
            op = int(UN[rng.integers(0, len(UN))])
            vals.append(e.unary(op, x))
        elif r < 0.45:
            op = int(BIN[rng.integers(0, 4)])
            c = float(np.float32(rng.uniform(0.25, 2.0)))
            vals.append(e.binary(op, x, e.const(c)))
        else:
            y = vals[rng.integers(0, len(vals))]
            op = int(BIN[rng.integers(0, 4)]) if rng.random() < 0.9 else abi.OP_POW
            vals.append(e.binary(op, x, y))
    return e


def unfused(ctx, e, tensors, out_shape, dtype):
    """Evaluates the node list with one unfused call per node."""
    vals = {}
    for i, (kind, code, a, b, value) in enumerate(e.nodes):
        if kind == abi.FUSE_INPUT:
            vals[i] = tensors[code]
            continue
        if kind == abi.FUSE_CONST:
            continue
        if kind == abi.FUSE_UNARY:
            o = empty(tuple(vals[a].shape), dtype)
            ctx.unary(code, d(vals[a]), d(o))
        elif e.nodes[b][0] == abi.FUSE_CONST:
            o = empty(tuple(vals[a].shape), dtype)
            ctx.binary_scalar(code, d(vals[a]), e.nodes[b][4], d(o))
        else:
            shape = abi.broadcast_shape(tuple(vals[a].shape), tuple(vals[b].shape))
            o = empty(shape, dtype)
            ctx.binary(code, d(vals[a]), d(vals[b]), d(o))
        vals[i] = o
    last = vals[len(e.nodes) - 1]
    import torch
    return host(torch.broadcast_to(last, out_shape).contiguous())


SHAPE_SETS = [
    [(64, 256)],
    [(64, 256), (1, 256)],
    [(64, 256), (1, 256), (64, 1)],
    [(8, 16, 32), (16, 1), (8, 1, 32), (1,)],
    [(1000,), (1000,)],          # 1-D, vector path
    [(37, 33), (37, 1)],         # odd inner extent: generic path
    [(5, 6, 7), (6, 7), (5, 1, 7)],
]


@pytest.mark.parametrize("mode", [abi.FUSE_MODE_AUTO, abi.FUSE_MODE_INTERP], indirect=True)
@pytest.mark.parametrize("dtype", [np.float32, np.float16])
@pytest.mark.parametrize("sset", range(len(SHAPE_SETS)))
@pytest.mark.parametrize("seed", range(6))
def test_random_dags_match_unfused(ctx, dtype, sset, seed, mode):
    shapes = SHAPE_SETS[sset]
    rng = np.random.default_rng(1000 * sset + seed)
    xs = [rng.uniform(0.1, 1.5, s).astype(dtype) for s in shapes]
    ts = [dev(x) for x in xs]
    out_shape = tuple(np.broadcast_shapes(*shapes))
    e = random_expr(rng, len(shapes), int(rng.integers(3, 12)))
    out = empty(out_shape, dtype)
    ctx.elementwise_fused(e.nodes, [d(t) for t in ts], d(out))
    got = host(out)
    want = unfused(ctx, e, ts, out_shape, dtype)
    assert_bits_equal(got, want, f"dag {sset}/{seed}")


def test_strided_and_transposed_inputs(ctx, orc):
    rng = np.random.default_rng(7)
    X = rng.uniform(-1, 1, (96, 160)).astype(np.float32)
    Y = rng.uniform(-1, 1, (160, 96)).astype(np.float32)
    tX, tY = dev(X), dev(Y)
    yT = abi.make_desc(tY.data_ptr(), abi.F32, (96, 160), (1, 96))        # Y.T view
    xs = abi.make_desc(tX.data_ptr() + 4, abi.F32, (96, 80), (160, 2))    # X[:, 1::2]
    out = empty((96, 160), np.float32)
    e = abi.Expr()
    e.binary(abi.OP_MUL, e.binary(abi.OP_ADD, e.input(0), e.input(1)), e.const(0.5))
    ctx.elementwise_fused(e.nodes, [d(tX), yT], d(out))
    want = orc.binary_scalar(orc.MUL, orc.binary(orc.ADD, X, np.ascontiguousarray(Y.T)), 0.5)
    assert_bits_equal(host(out), want, "transposed operand")
    out2 = empty((96, 80), np.float32)
    e2 = abi.Expr()
    e2.unary(abi.UN_ABS, e2.input(0))
    ctx.elementwise_fused(e2.nodes, [xs], d(out2))
    assert_bits_equal(host(out2), np.abs(X[:, 1::2]), "strided operand")


@pytest.mark.parametrize("mode", [abi.FUSE_MODE_AUTO, abi.FUSE_MODE_INTERP], indirect=True)
def test_temporaries_two_level(ctx, orc, mode):
    rng = np.random.default_rng(12)
    A, B = (rng.uniform(0.5, 1.5, (128, 64)).astype(np.float32) for _ in range(2))
    out = empty((128, 64), np.float32)
    e = abi.Expr()
    a, b = e.input(0), e.input(1)
    num = e.binary(abi.OP_MUL, e.binary(abi.OP_ADD, a, b), e.binary(abi.OP_SUB, a, b))
    den = e.binary(abi.OP_ADD, e.binary(abi.OP_MUL, a, b), e.binary(abi.OP_SUB, b, a))
    e.binary(abi.OP_DIV, num, den)
    tA, tB = dev(A), dev(B)  # keep both alive while the kernel reads them
    ctx.elementwise_fused(e.nodes, [d(tA), d(tB)], d(out))
    ob = orc.binary
    want = ob(orc.DIV, ob(orc.MUL, ob(orc.ADD, A, B), ob(orc.SUB, A, B)),
              ob(orc.ADD, ob(orc.MUL, A, B), ob(orc.SUB, B, A)))
    assert_bits_equal(host(out), want, "two-level")


def test_temporaries(ctx, orc):
    """((A+B)*(A-B)) / ((A*B)+(B-A)) needs a temporary per level; a balanced
    tree of depth 4 with four distinct inputs needs three."""
    rng = np.random.default_rng(11)
    A, B, C, D = (rng.uniform(0.5, 1.5, (128, 64)).astype(np.float32) for _ in range(4))
    ts = [dev(x) for x in (A, B, C, D)]
    out = empty((128, 64), np.float32)
    e = abi.Expr()
    a, b = e.input(0), e.input(1)
    num = e.binary(abi.OP_MUL, e.binary(abi.OP_ADD, a, b), e.binary(abi.OP_SUB, a, b))
    den = e.binary(abi.OP_ADD, e.binary(abi.OP_MUL, a, b), e.binary(abi.OP_SUB, b, a))
    e.binary(abi.OP_DIV, num, den)
    ctx.elementwise_fused(e.nodes, [d(t) for t in ts[:2]], d(out))
    ob, ADD, SUB, MUL, DIV = orc.binary, orc.ADD, orc.SUB, orc.MUL, orc.DIV
    want = ob(DIV, ob(MUL, ob(ADD, A, B), ob(SUB, A, B)), ob(ADD, ob(MUL, A, B), ob(SUB, B, A)))
    assert_bits_equal(host(out), want, "two-level")

    def tree(e, leaves, depth, k):
        if depth == 0:
            return leaves[k % 4]
        l = tree(e, leaves, depth - 1, 2 * k)
        r = tree(e, leaves, depth - 1, 2 * k + 1)
        return e.binary(abi.OP_ADD if depth % 2 else abi.OP_MUL, l, r)

    def tree_np(depth, k):
        if depth == 0:
            return (A, B, C, D)[k % 4]
        l, r = tree_np(depth - 1, 2 * k), tree_np(depth - 1, 2 * k + 1)
        return ob(ADD if depth % 2 else MUL, l, r)

    e3 = abi.Expr()
    leaves = [e3.input(j) for j in range(4)]
    tree(e3, leaves, 4, 0)   # leaves at depth 0 are inputs: needs 3 temporaries
    ctx.elementwise_fused(e3.nodes, [d(t) for t in ts], d(out))
    assert_bits_equal(host(out), tree_np(4, 0), "depth-4 tree")
    e5 = abi.Expr()
    leaves = [e5.input(j) for j in range(4)]
    tree(e5, leaves, 5, 0)   # needs 4 temporaries: beyond the interpreter
    ctx.set_fuse_mode(abi.FUSE_MODE_INTERP)
    try:
        with pytest.raises(abi.QsmlError) as err:
            ctx.elementwise_fused(e5.nodes, [d(t) for t in ts], d(out))
        assert err.value.status == abi.E_UNSUPPORTED
    finally:
        ctx.set_fuse_mode(abi.FUSE_MODE_AUTO)
    # the runtime-compiled kernel has no temporary limit
    ctx.elementwise_fused(e5.nodes, [d(t) for t in ts], d(out))
    assert_bits_equal(host(out), tree_np(5, 0), "depth-5 tree")


def test_errors(ctx):
    x = dev(np.ones((4, 8), np.float32))
    h = dev(np.ones((4, 8), np.float16))
    out = empty((4, 8), np.float32)
    cases = [
        ([(abi.FUSE_BINARY, abi.OP_ADD, 0, 1, 0.0)], [d(x)], abi.E_INVALID),           # operand not earlier
        ([(abi.FUSE_INPUT, 3, 0, 0, 0.0)], [d(x)], abi.E_INVALID),                     # input out of range
        ([(abi.FUSE_INPUT, 0, 0, 0, 0.0), (abi.FUSE_UNARY, 99, 0, 0, 0.0)], [d(x)], abi.E_INVALID),
        ([(abi.FUSE_INPUT, 0, 0, 0, 0.0)], [d(h)], abi.E_DTYPE),                        # dtype mismatch
        ([(abi.FUSE_INPUT, 0, 0, 0, 0.0)], [d(dev(np.ones((5, 8), np.float32)))], abi.E_SHAPE),
        ([(7, 0, 0, 0, 0.0)], [d(x)], abi.E_INVALID),                                   # unknown kind
    ]
    for nodes, ins, st in cases:
        with pytest.raises(abi.QsmlError) as e:
            ctx.elementwise_fused(nodes, ins, d(out))
        assert e.value.status == st, nodes
    many = [d(x)] * 7
    with pytest.raises(abi.QsmlError) as e:
        ctx.elementwise_fused([(abi.FUSE_INPUT, 0, 0, 0, 0.0)], many, d(out))
    assert e.value.status == abi.E_INVALID
    # empty output: nothing launched, no error
    z = dev(np.ones((0, 8), np.float32))
    ctx.elementwise_fused([(abi.FUSE_INPUT, 0, 0, 0, 0.0)], [d(z)], d(empty((0, 8), np.float32)))


def test_jit_mode_and_kernel_cache(ctx):
    """JIT mode: the compiled kernel runs (or the call is refused for a layout
    it does not cover); a repeated expression reuses its compiled kernel."""
    rng = np.random.default_rng(21)
    X = dev(rng.uniform(-1, 1, (256, 512)).astype(np.float32))
    Y = dev(rng.uniform(-1, 1, (1, 512)).astype(np.float32))
    out = empty((256, 512), np.float32)
    e = abi.Expr()
    e.unary(abi.UN_TANH, e.binary(abi.OP_MUL, e.binary(abi.OP_SUB, e.input(0), e.input(1)), e.const(3.0)))
    ctx.set_fuse_mode(abi.FUSE_MODE_JIT)
    try:
        ctx.elementwise_fused(e.nodes, [d(X), d(Y)], d(out))
        first = host(out)
        _, _, k0 = ctx.fuse_stats()
        for _ in range(3):
            ctx.elementwise_fused(e.nodes, [d(X), d(Y)], d(out))
        _, _, k1 = ctx.fuse_stats()
        assert k1 == k0
        assert_bits_equal(host(out), first, "repeat")
        # a 3-D layout that does not collapse to 2-D is the interpreter's
        Z = dev(rng.uniform(-1, 1, (4, 6, 8)).astype(np.float32))
        W = dev(rng.uniform(-1, 1, (4, 1, 8)).astype(np.float32))
        o3 = empty((4, 6, 8), np.float32)
        e3 = abi.Expr()
        e3.binary(abi.OP_ADD, e3.input(0), e3.input(1))
        with pytest.raises(abi.QsmlError) as err:
            ctx.elementwise_fused(e3.nodes, [d(Z), d(W)], d(o3))
        assert err.value.status == abi.E_UNSUPPORTED
    finally:
        ctx.set_fuse_mode(abi.FUSE_MODE_AUTO)
    ctx.set_fuse_mode(abi.FUSE_MODE_INTERP)
    try:
        ctx.elementwise_fused(e.nodes, [d(X), d(Y)], d(out))
        assert_bits_equal(host(out), first, "interpreter vs compiled")
    finally:
        ctx.set_fuse_mode(abi.FUSE_MODE_AUTO)
    with pytest.raises(abi.QsmlError):
        ctx.set_fuse_mode(9)
