"""Pins the CPU oracle before it is trusted as the checker.

1. Every known-answer vector of the reference's own unit tests
   (tests/golden/known_answers.json, transcribed with file:line citations).
2. Properties the restated semantics must have (binary16 conversion,
   IEEE maximum/minimum, pow, relu, broadcasting, strided views, layer norm,
   the reference's fma chain), checked against NumPy where NumPy defines the
   same thing.
"""
import json
import os

import numpy as np
import pytest

GOLDEN = os.path.join(os.path.dirname(__file__), "golden", "known_answers.json")
CASES = json.load(open(GOLDEN))


def _input(spec):
    shape = tuple(spec["shape"])
    if "data" in spec:
        return np.asarray(spec["data"], dtype=np.float32).reshape(shape)
    return np.full(shape, spec["fill"], dtype=np.float32)


def oracle_eval(orc, case):
    op = case["op"]
    a = _input(case["a"])
    if op in ("add", "sub", "mul", "div"):
        b = _input(case["b"])
        return orc.binary({"add": orc.ADD, "sub": orc.SUB, "mul": orc.MUL, "div": orc.DIV}[op], a, b)
    if op == "mul_scalar":
        return orc.binary_scalar(orc.MUL, a, case["scalar"])
    if op in ("relu", "neg", "abs", "sqrt", "exp", "sigmoid", "gelu", "tanh"):
        code = {"relu": orc.UN_RELU, "neg": orc.UN_NEG, "abs": orc.UN_ABS, "sqrt": orc.UN_SQRT,
                "exp": orc.UN_EXP, "sigmoid": orc.UN_SIGMOID, "gelu": orc.UN_GELU, "tanh": orc.UN_TANH}[op]
        return orc.unary(code, a)
    if op in ("sum", "mean", "max", "min"):
        code = {"sum": orc.SUM, "mean": orc.MEAN, "max": orc.MAX, "min": orc.MIN}[op]
        return orc.reduce(code, a)[0].reshape(1)
    if op == "matmul":
        return orc.matmul_fma(a, _input(case["b"]))
    if op == "transpose":
        return orc.gather(a, 0, (a.shape[1], a.shape[0]), (1, a.shape[1]))
    if op == "copy":
        return orc.gather(a, 0, a.shape, [int(s // 4) for s in a.strides])
    raise KeyError(op)


@pytest.mark.parametrize("case", CASES["cases"], ids=[c["id"] for c in CASES["cases"]])
def test_oracle_known_answers(orc, case):
    out = oracle_eval(orc, case)
    assert list(out.shape) == case["out_shape"], case["src"]
    flat = out.reshape(-1)
    for idx, expect, tol in case.get("check", []):
        if tol == 0:
            assert flat[idx] == np.float32(expect), (case["src"], flat[idx], expect)
        else:
            assert abs(float(flat[idx]) - expect) < tol, (case["src"], flat[idx], expect)
    for idx, lower in case.get("greater", []):
        assert flat[idx] > lower, case["src"]


def test_half_conversion_exhaustive(orc):
    """binary16 -> binary32 is exact and binary32 -> binary16 is RNE; NumPy
    implements both, so all 65536 half patterns and a dense float sweep must
    agree bit for bit (NaN payloads excluded)."""
    h = np.arange(65536, dtype=np.uint32).astype(np.uint16)
    f = np.empty(65536, dtype=np.float32)
    orc.lib().orc_half_to_float_n(h.ctypes.data, f.ctypes.data, 65536)
    ref = h.view(np.float16).astype(np.float32)
    nan = np.isnan(ref)
    assert np.array_equal(np.isnan(f), nan)
    assert np.array_equal(f[~nan].view(np.uint32), ref[~nan].view(np.uint32))
    rng = np.random.default_rng(0)
    bits = rng.integers(0, 2 ** 32, size=2_000_000, dtype=np.uint64).astype(np.uint32)
    xs = bits.view(np.float32)
    xs = np.concatenate([xs, np.float32([65504, 65520, 65519.99, 6.1e-5, 5.96e-8, 2.98e-8, 2.9802322e-08,
                                         -0.0, 0.0, np.inf, -np.inf])]).astype(np.float32)
    out = np.empty(xs.size, dtype=np.uint16)
    orc.lib().orc_float_to_half_n(xs.ctypes.data, out.ctypes.data, xs.size)
    with np.errstate(over="ignore"):
        ref16 = xs.astype(np.float16)
    nan = np.isnan(xs)
    assert np.array_equal(out[~nan], ref16[~nan].view(np.uint16))
    assert np.all(np.isnan(out[nan].view(np.float16)))


def test_max_min_ieee2019(orc):
    """IEEE 754-2019 maximum/minimum: NaN wins, -0 < +0, order-free."""
    nan = np.float32("nan")
    assert np.isnan(orc.lib().orc_max_f32(1.0, nan))
    assert np.isnan(orc.lib().orc_min_f32(nan, 1.0))
    assert np.signbit(np.float32(orc.lib().orc_min_f32(0.0, -0.0)))
    assert not np.signbit(np.float32(orc.lib().orc_max_f32(-0.0, 0.0)))
    x = np.float32([3, -0.0, 0.0, -7, np.inf, 2])
    for op, want in ((orc.MAX, np.inf), (orc.MIN, -7)):
        assert orc.reduce(op, x)[0] == want
        assert orc.reduce(op, x[::-1].copy())[0] == want
    assert np.isnan(orc.reduce(orc.MAX, np.float32([1, nan, 2]))[0])


def test_relu_pins(orc):
    x = np.float32([-1.0, -0.0, 0.0, 1.5, np.nan, -np.inf, np.inf])
    y = orc.relu(x)
    assert y[0] == 0 and not np.signbit(y[1]) and not np.signbit(y[2])
    assert y[3] == np.float32(1.5) and np.isnan(y[4]) and y[5] == 0 and y[6] == np.inf


def test_pow_semantics(orc):
    rng = np.random.default_rng(1)
    x = rng.uniform(-4, 4, 100000).astype(np.float32)
    # exponent 2: the single correctly rounded product
    assert np.array_equal(orc.pow_scalar(x, 2.0).view(np.uint32), (x * x).view(np.uint32))
    # other exponents follow C99 powf (checked against binary64 pow, <= 1 ulp)
    for y in (0.5, 3.0, -1.5, 2.5, 0.0, 1.0):
        got = orc.pow_scalar(np.abs(x), y)
        with np.errstate(all="ignore"):
            ref = np.power(np.abs(x).astype(np.float64), y).astype(np.float32)
        assert orc.ulp_diff_f32(got, ref).max() <= 1, y
    assert orc.lib().orc_pow_f32(-2.0, 3.0) == -8.0
    assert np.isnan(orc.lib().orc_pow_f32(-2.0, 0.5))
    assert orc.lib().orc_pow_f32(np.nan, 0.0) == 1.0


def test_binary_broadcast_matches_numpy(orc):
    rng = np.random.default_rng(2)
    shapes = [((4096,), (1,)), ((3, 1, 5), (4, 1)), ((1, 7), (6, 1)), ((2, 3, 4), (3, 4)),
              ((5, 1, 1), (1, 2, 3)), ((1,), (9,))]
    for sa, sb in shapes:
        a = rng.uniform(-2, 2, sa).astype(np.float32)
        b = rng.uniform(0.5, 2, sb).astype(np.float32)
        for op, fn in ((orc.ADD, np.add), (orc.SUB, np.subtract), (orc.MUL, np.multiply), (orc.DIV, np.divide)):
            got = orc.binary(op, a, b)
            ref = fn(a, b)
            assert got.shape == ref.shape
            assert np.array_equal(got.view(np.uint32), ref.view(np.uint32)), (sa, sb, op)
    with pytest.raises(ValueError):
        orc.binary(orc.ADD, np.zeros((3, 4), np.float32), np.zeros((5,), np.float32))


def test_reduce_axis_order_is_reference_order(orc):
    """out32 is the k-ascending binary32 chain of Reduction.cpp:328."""
    rng = np.random.default_rng(3)
    x = rng.normal(size=(3, 50, 7)).astype(np.float32)
    o32, o64, ab = orc.reduce(orc.SUM, x, axis=1)
    ref = np.zeros((3, 7), dtype=np.float32)
    for k in range(50):
        ref = (ref + x[:, k, :]).astype(np.float32)
    assert np.array_equal(o32, ref)
    assert np.allclose(o64, x.astype(np.float64).sum(axis=1))
    assert np.allclose(ab, np.abs(x.astype(np.float64)).sum(axis=1))
    m32 = orc.reduce(orc.MEAN, x, axis=1)[0]
    assert np.array_equal(m32, (ref * np.float32(1.0 / 50)).astype(np.float32))


def test_gather_matches_numpy_views(orc):
    X = np.arange(64 * 96, dtype=np.int32).reshape(64, 96)
    for view in (X[5::3, 1::2], X.T[::4, :], X[::-1, 3:50:5], X[10:11, :]):
        off = (view.__array_interface__["data"][0] - X.__array_interface__["data"][0]) // 4
        strides = [s // 4 for s in view.strides]
        got = orc.gather(X, off, view.shape, strides)
        assert np.array_equal(got, np.ascontiguousarray(view))


def test_layer_norm_matches_numpy(orc):
    rng = np.random.default_rng(4)
    x = rng.normal(0.5, 2, (16, 96)).astype(np.float32)
    g = rng.normal(1, 0.1, 96).astype(np.float32)
    b = rng.normal(0, 0.1, 96).astype(np.float32)
    y = orc.layer_norm(x, g, b, 1e-5)
    xd = x.astype(np.float64)
    mu = xd.mean(-1, keepdims=True)
    var = xd.var(-1, keepdims=True)
    ref = ((xd - mu) / np.sqrt(var + np.float64(np.float32(1e-5))) * g + b).astype(np.float32)
    assert np.max(np.abs(y - ref)) <= 1e-6


def test_matmul_fma_chain(orc):
    rng = np.random.default_rng(5)
    a = rng.uniform(-1, 1, (9, 33)).astype(np.float32)
    b = rng.uniform(-1, 1, (33, 5)).astype(np.float32)
    c = orc.matmul_fma(a, b)
    # explicit fma chain in float64 arithmetic rounded per step reproduces fmaf
    ref = np.zeros((9, 5), dtype=np.float32)
    for k in range(33):
        prod = a[:, k:k + 1].astype(np.float64) * b[k:k + 1, :].astype(np.float64)
        ref = (ref.astype(np.float64) + prod).astype(np.float32)  # exact product, one rounding
    assert np.array_equal(c, ref)
    c64 = orc.matmul_f64(a, b)
    assert np.allclose(c64, a.astype(np.float64) @ b.astype(np.float64), atol=1e-12)
    # batched
    ab = rng.uniform(-1, 1, (3, 4, 6)).astype(np.float32)
    bb = rng.uniform(-1, 1, (3, 6, 2)).astype(np.float32)
    cb = orc.matmul_f64(ab, bb)
    assert np.allclose(cb, np.einsum("bij,bjk->bik", ab.astype(np.float64), bb.astype(np.float64)))


def test_prod_reference_order(orc):
    """prod accumulates in k order like the reference's prod shader tree
    restated serially (Reduction.cpp:190-211), binary64 as the truth."""
    x = np.float32([1.5, -2.0, 0.5, 4.0, 1.25])
    o32, o64, _ = orc.reduce(orc.PROD, x)
    assert o32 == np.float32(-7.5) and o64 == -7.5
    y = np.arange(1, 11, dtype=np.float32).reshape(2, 5)
    assert np.array_equal(orc.reduce(orc.PROD, y, axis=1)[0], np.float32([120, 30240]))


def test_argreduce_matches_numpy(orc):
    """argmax/argmin: the reference's are stubs returning values
    (Reduction.cpp:388-396); the oracle restates NumPy's index semantics,
    checked here against NumPy itself, NaN and ties included."""
    rng = np.random.default_rng(3)
    for dt in (np.float32, np.float16, np.int32, np.int16, np.int8, np.uint32, np.uint16, np.uint8):
        x = rng.integers(0, 20, (7, 9, 11)).astype(dt)
        for ax in (None, 0, 1, 2, -1):
            assert np.array_equal(orc.argreduce(orc.ARGMAX, x, ax), np.argmax(x, axis=ax)), (dt, ax)
            assert np.array_equal(orc.argreduce(orc.ARGMIN, x, ax), np.argmin(x, axis=ax)), (dt, ax)
    y = np.float32([1, np.nan, 3, np.nan, -0.0, 0.0])
    assert orc.argreduce(orc.ARGMAX, y) == np.argmax(y) == 1
    assert orc.argreduce(orc.ARGMIN, y) == np.argmin(y) == 1
    z = np.float32([0.0, -0.0, 5.0, -0.0])
    assert orc.argreduce(orc.ARGMIN, z) == np.argmin(z) == 0
    with pytest.raises(ValueError):
        orc.argreduce(orc.ARGMAX, np.zeros((3, 0), np.float32), 1)


def test_matmul_check_sees_one_bad_output(orc):
    """The full-matrix matmul check accepts a binary32 product and flags a
    single output pushed outside the bar (a defect confined to one tile)."""
    rng = np.random.default_rng(3)
    a = rng.uniform(-1, 1, (2, 300, 200)).astype(np.float32)
    b = rng.uniform(-1, 1, (2, 200, 150)).astype(np.float32)
    c = np.matmul(a, b)
    worst, normwise, _ = orc.matmul_check(c, a, b, rows_per_block=64)
    assert worst <= 1e-5 and normwise <= 1e-6
    bad = c.copy()
    bad[1, 257, 149] += 1e-2 * np.abs(a[1, 257]) @ np.abs(b[1, :, 149])
    worst, _, _ = orc.matmul_check(bad, a, b, rows_per_block=64)
    assert worst >= 1e-2 * 0.99
