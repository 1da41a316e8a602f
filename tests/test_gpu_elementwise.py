"""GPU parity of the elementwise kernels (through the C ABI) against the oracle.

Tolerances (binary32): add/sub/mul/div/relu/neg/abs/sqrt bit-exact; pow with
exponent 2 bit-exact (x*x), other exponents <= 2 ulp; exp/log/sin/cos/tanh/
sigmoid/gelu (CUDA's own math functions against glibc) <= 4 ulp or 1e-6
absolute near zero.  binary16 results are the binary32 result rounded once,
so bit-exact as well.
"""
import json
import os

import numpy as np
import pytest

from helpers import assert_bits_equal, d, dev, empty, host, ulp_f32
from quasarml_b200 import abi, datagen

pytestmark = pytest.mark.gpu

BIN = {"add": abi.OP_ADD, "sub": abi.OP_SUB, "mul": abi.OP_MUL, "div": abi.OP_DIV}
UN = {"relu": abi.UN_RELU, "neg": abi.UN_NEG, "abs": abi.UN_ABS, "sqrt": abi.UN_SQRT, "exp": abi.UN_EXP,
      "log": abi.UN_LOG, "sin": abi.UN_SIN, "cos": abi.UN_COS, "tanh": abi.UN_TANH,
      "sigmoid": abi.UN_SIGMOID, "gelu": abi.UN_GELU}


def gpu_binary(ctx, op, a_np, b_np):
    a, b = dev(a_np), dev(b_np)
    out = empty(abi.broadcast_shape(a_np.shape, b_np.shape), a_np.dtype)
    ctx.binary(op, d(a), d(b), d(out))
    return host(out)


def gpu_scalar(ctx, op, a_np, s):
    a = dev(a_np)
    out = empty(a_np.shape, a_np.dtype)
    ctx.binary_scalar(op, d(a), s, d(out))
    return host(out)


def gpu_unary(ctx, op, a_np):
    a = dev(a_np)
    out = empty(a_np.shape, a_np.dtype)
    ctx.unary(op, d(a), d(out))
    return host(out)


GOLDEN = json.load(open(os.path.join(os.path.dirname(__file__), "golden", "known_answers.json")))


def _inp(spec):
    if "data" in spec:
        return np.asarray(spec["data"], dtype=np.float32).reshape(spec["shape"])
    return np.full(spec["shape"], spec["fill"], dtype=np.float32)


@pytest.mark.parametrize("case", [c for c in GOLDEN["cases"] if c["op"] not in ("matmul", "transpose", "copy",
                                                                                "sum", "mean", "max", "min")],
                         ids=lambda c: c["id"])
def test_reference_known_answers(ctx, case):
    a = _inp(case["a"])
    if case["op"] in BIN:
        out = gpu_binary(ctx, BIN[case["op"]], a, _inp(case["b"]))
    elif case["op"] == "mul_scalar":
        out = gpu_scalar(ctx, abi.OP_MUL, a, case["scalar"])
    else:
        out = gpu_unary(ctx, UN[case["op"]], a)
    assert list(out.shape) == case["out_shape"]
    flat = out.reshape(-1)
    for idx, expect, tol in case.get("check", []):
        if tol == 0:
            assert flat[idx] == np.float32(expect), case["src"]
        else:
            assert abs(float(flat[idx]) - expect) < tol, case["src"]
    for idx, lower in case.get("greater", []):
        assert flat[idx] > lower


def test_chain_4096_bitexact(ctx, orc):
    """relu(pow((A+B)*B - A, 2) / D) at 4096x4096 with B[1,4096], D[4096,1]:
    every intermediate bit-identical to the oracle."""
    A = datagen.uniform(datagen.SEEDS["ew_A"], (4096, 4096), -1.0, 1.0)
    B = datagen.uniform(datagen.SEEDS["ew_B"], (1, 4096), -1.0, 1.0)
    D = datagen.uniform(datagen.SEEDS["ew_D"], (4096, 1), 0.5, 2.0)
    tA, tB, tD = dev(A), dev(B), dev(D)
    t = [empty((4096, 4096), np.float32) for _ in range(6)]
    ctx.binary(abi.OP_ADD, d(tA), d(tB), d(t[0]))
    ctx.binary(abi.OP_MUL, d(t[0]), d(tB), d(t[1]))
    ctx.binary(abi.OP_SUB, d(t[1]), d(tA), d(t[2]))
    ctx.binary_scalar(abi.OP_POW, d(t[2]), 2.0, d(t[3]))
    ctx.binary(abi.OP_DIV, d(t[3]), d(tD), d(t[4]))
    ctx.unary(abi.UN_RELU, d(t[4]), d(t[5]))
    r1 = orc.binary(orc.ADD, A, B)
    r2 = orc.binary(orc.MUL, r1, B)
    r3 = orc.binary(orc.SUB, r2, A)
    r4 = orc.pow_scalar(r3, 2.0)
    r5 = orc.binary(orc.DIV, r4, D)
    r6 = orc.relu(r5)
    for name, g, r in zip(("add", "mul", "sub", "pow", "div", "relu"), t, (r1, r2, r3, r4, r5, r6)):
        assert_bits_equal(host(g), r, name)


SHAPES = [((4096,), (1,)), ((3, 1, 5), (4, 1)), ((1, 7), (6, 1)), ((2, 3, 4), (3, 4)), ((5, 1, 1), (1, 2, 3)),
          ((1,), (9,)), ((1001,), (1001,)), ((37, 64), (1, 64)), ((64, 37), (64, 1)), ((2, 8, 16), (2, 1, 16)),
          ((8, 1, 24), (1, 5, 24)), ((1, 1), (1, 1)), ((17, 33, 3), (17, 33, 3))]


@pytest.mark.parametrize("dtype", [np.float32, np.float16, np.int32])
@pytest.mark.parametrize("sa,sb", SHAPES)
def test_broadcast_bitexact(ctx, orc, dtype, sa, sb):
    rng = np.random.default_rng(abs(hash((sa, sb))) % 2 ** 32)
    if dtype == np.int32:
        a = rng.integers(-1000, 1000, sa).astype(np.int32)
        b = rng.integers(1, 50, sb).astype(np.int32) * rng.choice([-1, 1], sb).astype(np.int32)
    else:
        a = rng.uniform(-2, 2, sa).astype(dtype)
        b = rng.uniform(0.5, 2, sb).astype(dtype)
    for name, op in BIN.items():
        g = gpu_binary(ctx, op, a, b)
        r = orc.binary(op, a, b)
        assert_bits_equal(g, r, f"{name} {sa} {sb} {dtype}")
        g = gpu_binary(ctx, op, b, a)
        r = orc.binary(op, b, a)
        assert_bits_equal(g, r, f"{name} swapped {sa} {sb} {dtype}")


def test_strided_and_misaligned_inputs(ctx, orc):
    """Non-contiguous views go through the generic kernel, misaligned ones
    through the scalar flat kernel; both stay bit-exact."""
    rng = np.random.default_rng(7)
    X = rng.uniform(-1, 1, (64, 130)).astype(np.float32)
    Y = rng.uniform(0.5, 2, (130, 64)).astype(np.float32)
    tX, tY = dev(X), dev(Y)
    # transposed view of Y (strides (1, 64)) + X[:, 1:129]
    a = tX[:, 1:129]
    b = tY.t()[:, :128]
    out = empty((64, 128), np.float32)
    ctx.binary(abi.OP_DIV, d(a), d(b), d(out))
    ref = orc.binary(orc.DIV, np.ascontiguousarray(X[:, 1:129]), np.ascontiguousarray(Y.T[:, :128]))
    assert_bits_equal(host(out), ref, "strided div")
    # flat arrays starting 4 bytes past an aligned address
    flat = tX.reshape(-1)[1:1 + 4097]
    out2 = empty((4097,), np.float32)
    ctx.binary_scalar(abi.OP_MUL, d(flat), 3.0, d(out2))
    assert_bits_equal(host(out2), orc.binary_scalar(orc.MUL, X.reshape(-1)[1:4098], 3.0), "misaligned")


@pytest.mark.parametrize("y", [0.5, 3.0, -1.5, 2.5, 0.0, 1.0, -2.0, 7.25])
def test_pow_scalar_ulp(ctx, orc, y):
    rng = np.random.default_rng(8)
    x = np.concatenate([rng.uniform(0, 4, 20000), rng.uniform(-4, 0, 2000),
                        [0.0, -0.0, np.inf, -np.inf, np.nan, 1.0, -1.0, 1e-30, 1e30]]).astype(np.float32)
    g = gpu_scalar(ctx, abi.OP_POW, x, y)
    r = orc.pow_scalar(x, y)
    assert ulp_f32(g, r).max() <= 2, y


def test_pow_tensor_exponent(ctx, orc):
    rng = np.random.default_rng(9)
    x = rng.uniform(0, 3, (257, 33)).astype(np.float32)
    y = rng.uniform(-3, 3, (1, 33)).astype(np.float32)
    y[0, :4] = [2.0, 0.0, 1.0, -1.0]
    g = gpu_binary(ctx, abi.OP_POW, x, y)
    r = orc.binary(orc.POW, x, y)
    assert ulp_f32(g, r).max() <= 2
    assert_bits_equal(g[:, 0], (x[:, 0] * x[:, 0]), "pow 2 column")


def test_pow_chain_exponent2_bitexact(ctx, orc):
    x = datagen.uniform(11, (1 << 20,), -3, 3)
    assert_bits_equal(gpu_scalar(ctx, abi.OP_POW, x, 2.0), x * x, "pow2")


def test_relu_special_values(ctx):
    x = np.float32([-1.0, -0.0, 0.0, 1.5, np.nan, -np.inf, np.inf, -1e-45, 1e-45])
    y = gpu_unary(ctx, abi.UN_RELU, x)
    assert y[0] == 0 and not np.signbit(y[1]) and not np.signbit(y[2]) and y[3] == np.float32(1.5)
    assert np.isnan(y[4]) and y[5] == 0 and y[6] == np.inf and y[7] == 0 and y[8] == np.float32(1e-45)
    h = gpu_unary(ctx, abi.UN_RELU, x.astype(np.float16))
    assert not np.signbit(h[1]) and np.isnan(h[4]) and h[3] == np.float16(1.5)


@pytest.mark.parametrize("name", list(UN))
def test_unary_ops(ctx, orc, name):
    rng = np.random.default_rng(10)
    lo = 0.0 if name in ("sqrt", "log") else -6.0
    x = rng.uniform(lo, 6.0, 50001).astype(np.float32)
    g = gpu_unary(ctx, UN[name], x)
    r = orc.unary(UN[name], x)
    if name in ("relu", "neg", "abs", "sqrt"):
        assert_bits_equal(g, r, name)
    else:
        bad = (ulp_f32(g, r) > 4) & (np.abs(g.astype(np.float64) - r) > 1e-6)
        assert not bad.any(), (name, x[bad][:5], g[bad][:5], r[bad][:5])


@pytest.mark.parametrize("name,op", [("add", abi.OP_ADD), ("sub", abi.OP_SUB), ("mul", abi.OP_MUL),
                                     ("div", abi.OP_DIV)])
def test_scalar_ops_bitexact(ctx, orc, name, op):
    x = datagen.uniform(12, (1 << 16) + 3, -5, 5)
    for s in (0.1, -3.0, 7.5):
        assert_bits_equal(gpu_scalar(ctx, op, x, s), orc.binary_scalar(op, x, s), name)


def test_errors_are_status_codes(ctx):
    a = empty((3, 4), np.float32)
    b = empty((5,), np.float32)
    out = empty((3, 4), np.float32)
    with pytest.raises(abi.QsmlError) as e:
        ctx.binary(abi.OP_ADD, d(a), d(b), d(out))
    assert e.value.status == abi.E_SHAPE
    with pytest.raises(abi.QsmlError) as e:
        ctx.binary(abi.OP_ADD, d(a), d(empty((3, 4), np.float16)), d(out))
    assert e.value.status == abi.E_DTYPE
    wide = empty((4, 3), np.float32).t()  # non-contiguous out
    with pytest.raises(abi.QsmlError) as e:
        ctx.unary(abi.UN_RELU, d(a), d(wide))
    assert e.value.status == abi.E_SHAPE
    with pytest.raises(abi.QsmlError) as e:
        ctx.binary(abi.OP_POW, d(empty((3,), np.int32)), d(empty((3,), np.int32)), d(empty((3,), np.int32)))
    assert e.value.status == abi.E_DTYPE
    # out shape must be exactly the broadcast shape
    with pytest.raises(abi.QsmlError):
        ctx.binary(abi.OP_ADD, d(empty((1, 4), np.float32)), d(empty((1, 4), np.float32)), d(out))


def test_empty_tensors(ctx):
    a = empty((0, 4), np.float32)
    out = empty((0, 4), np.float32)
    ctx.binary(abi.OP_ADD, d(a), d(a), d(out))
    ctx.unary(abi.UN_RELU, d(a), d(out))
    ctx.synchronize()


def test_fill(ctx):
    t = empty((1000,), np.float32)
    ctx.fill(t.data_ptr(), np.float32(2.5).tobytes(), 1000)
    assert np.all(host(t) == np.float32(2.5))
    h = empty((333,), np.float16)
    ctx.fill(h.data_ptr(), np.float16(-1.0).tobytes(), 333)
    assert np.all(host(h) == np.float16(-1.0))
