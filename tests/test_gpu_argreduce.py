"""GPU argmax / argmin (qsml_arg_reduce) against the oracle's first-index scan.

Indices must match exactly.  Inputs carry many ties (small integer ranges)
so the first-index rule is exercised, and float inputs carry NaN, +-0 and
infinities.  Shapes reach every kernel: the segment kernel (the flattened
tensor and a few long rows), one warp per row, and the column kernel, each
with and without 16-byte vector loads.
"""
import numpy as np
import pytest

from helpers import d, dev, empty, host
from quasarml_b200 import abi

pytestmark = pytest.mark.gpu

DTYPES = [np.float32, np.float16, np.int32, np.int16, np.int8, np.uint32, np.uint16, np.uint8]


def make(shape, dtype, seed, lo=0, hi=50, specials=True):
    rng = np.random.default_rng(seed)
    x = rng.integers(lo, hi, size=shape).astype(dtype)
    if specials and np.issubdtype(np.dtype(dtype), np.floating) and x.size >= 16:
        flat = x.reshape(-1)
        pos = rng.choice(x.size, size=max(4, x.size // 5000), replace=False)
        vals = np.array([np.nan, -0.0, 0.0, np.inf, -np.inf], dtype=dtype)
        flat[pos] = vals[rng.integers(0, len(vals), size=len(pos))]
    return x


# Unsigned inputs travel as the signed type of the same width (the bits are
# what matters); the descriptor carries the unsigned dtype code.
_SIGNED = {np.dtype(np.uint32): (np.int32, abi.U32), np.dtype(np.uint16): (np.int16, abi.U16)}


def _dev_desc(x):
    if np.dtype(x.dtype) in _SIGNED:
        st, code = _SIGNED[np.dtype(x.dtype)]
        t = dev(np.ascontiguousarray(x).view(st))
        return t, abi.make_desc(t.data_ptr(), code, tuple(t.shape), tuple(t.stride()))
    t = dev(x)
    return t, d(t)


def gpu_arg(ctx, op, x, axis, keepdims=False, out_dtype=np.int32):
    tx, dx = _dev_desc(x)
    if axis is None:
        oshape = (1,)
        ax = abi.AXIS_ALL
    else:
        ax = axis
        oshape = abi.reduced_shape(x.shape, axis, keepdims)
    out = empty(oshape, np.int32)
    do = d(out)
    if out_dtype == np.uint32:
        do = abi.make_desc(out.data_ptr(), abi.U32, tuple(out.shape), tuple(out.stride()))
    ctx.arg_reduce(op, dx, ax, keepdims, do)
    r = host(out)
    return (r.view(np.uint32) if out_dtype == np.uint32 else r).astype(np.int64)


CASES = [
    ((1000003,), None),            # segment kernel, one row, ragged tail
    ((64, 512, 1024), None),       # segment kernel, flattened 33.5M elements
    ((8, 100000), -1),             # segment kernel, several long rows
    ((4096, 300), 1),              # warp per row
    ((5000, 77), -1),              # warp per row, unaligned rows
    ((64, 512, 1024), 0),          # column kernel
    ((64, 512, 1024), 1),          # column kernel
    ((3, 1000, 7), 1),             # column kernel, scalar loads
    ((1,), 0),                     # single element
]


@pytest.mark.parametrize("dtype", DTYPES)
@pytest.mark.parametrize("case", range(len(CASES)))
@pytest.mark.parametrize("op", [abi.ARG_MAX, abi.ARG_MIN])
def test_matches_oracle(ctx, orc, dtype, case, op):
    shape, axis = CASES[case]
    if int(np.prod(shape)) > 4_000_000 and dtype not in (np.float32, np.float16, np.int8):
        pytest.skip("large shapes run for three representative dtypes")
    x = make(shape, dtype, seed=100 + case)
    got = gpu_arg(ctx, op, x, axis)
    want = orc.argreduce(op, x, axis)
    np.testing.assert_array_equal(got.reshape(-1), np.asarray(want).reshape(-1))


TIE_CASES = [((1000003,), None), ((8, 100000), -1), ((4096, 300), 1), ((64, 512, 1024), 0), ((64, 512, 1024), 1),
              ((16, 64, 520), 1)]


@pytest.mark.parametrize("case", range(len(TIE_CASES)))
@pytest.mark.parametrize("op", [abi.ARG_MAX, abi.ARG_MIN])
def test_f16_ties_zeros_and_nans(ctx, orc, case, op):
    """binary16 through the packed (two halves per instruction) scans: values
    drawn from {-0, +0, 1, -1} so that ties are everywhere and -0/+0 must
    compare equal, NaN in a few slices (sometimes first), whole slices of NaN
    and of -inf/+inf."""
    shape, axis = TIE_CASES[case]
    rng = np.random.default_rng(300 + case)
    x = rng.choice(np.array([-0.0, 0.0, 1.0, -1.0], np.float16), size=shape)
    flat = x.reshape(-1)
    flat[rng.choice(flat.size, size=max(3, flat.size // 200000), replace=False)] = np.nan
    if x.ndim >= 2:
        flat[0] = np.nan
        x[(0,) * (x.ndim - 2) + (slice(None), 1)] = np.nan                # a NaN column
        x[(min(1, x.shape[0] - 1),) + (slice(None),) * (x.ndim - 1)] = -np.inf if op == abi.ARG_MAX else np.inf
    got = gpu_arg(ctx, op, x, axis)
    want = orc.argreduce(op, x, axis)
    np.testing.assert_array_equal(got.reshape(-1), np.asarray(want).reshape(-1))


def test_nan_and_signed_zero_rules(ctx, orc):
    x = np.array([1, 5, np.nan, 5, np.nan, -0.0], np.float32)
    assert gpu_arg(ctx, abi.ARG_MAX, x, None)[0] == 2
    assert gpu_arg(ctx, abi.ARG_MIN, x, None)[0] == 2
    z = np.array([3, -0.0, 0.0, -0.0, 7], np.float32)
    assert gpu_arg(ctx, abi.ARG_MIN, z, None)[0] == 1  # -0 == +0: first one
    y = np.full(5000, -np.inf, np.float32)
    assert gpu_arg(ctx, abi.ARG_MAX, y, None)[0] == 0  # all equal: index 0
    # integer extremes
    i = np.array([np.iinfo(np.int32).min, 0, np.iinfo(np.int32).max, np.iinfo(np.int32).max], np.int32)
    assert gpu_arg(ctx, abi.ARG_MAX, i, None)[0] == 2
    assert gpu_arg(ctx, abi.ARG_MIN, i, None)[0] == 0
    u = np.array([7, np.iinfo(np.uint32).max, 0, 0], np.uint32)
    assert gpu_arg(ctx, abi.ARG_MAX, u, None)[0] == 1
    assert gpu_arg(ctx, abi.ARG_MIN, u, None)[0] == 2


WORST_SHAPES = [((1000003,), None), ((8, 100000), -1), ((4096, 300), 1), ((8, 64, 256), 1), ((3, 1000, 7), 1)]


@pytest.mark.parametrize("shape,axis", WORST_SHAPES)
@pytest.mark.parametrize("dtype,op,fill", [
    (np.float32, abi.ARG_MAX, -np.inf), (np.float32, abi.ARG_MIN, np.inf), (np.float16, abi.ARG_MAX, -np.inf),
    (np.int32, abi.ARG_MAX, np.iinfo(np.int32).min), (np.int32, abi.ARG_MIN, np.iinfo(np.int32).max),
    (np.uint32, abi.ARG_MAX, 0), (np.uint32, abi.ARG_MIN, np.iinfo(np.uint32).max), (np.int8, abi.ARG_MAX, -128)])
def test_worst_values_every_kernel(ctx, orc, shape, axis, dtype, op, fill):
    """Slices made only of the value every element is at least as good as
    (every kernel starts its running best there), then one better element."""
    x = np.full(shape, fill, dtype)
    want = orc.argreduce(op, x, axis)
    np.testing.assert_array_equal(gpu_arg(ctx, op, x, axis).reshape(-1), np.asarray(want).reshape(-1))
    flat = x.reshape(-1)
    flat[flat.size // 3] = np.array(7, dtype) if fill != 7 else np.array(8, dtype)
    want = orc.argreduce(op, x, axis)
    np.testing.assert_array_equal(gpu_arg(ctx, op, x, axis).reshape(-1), np.asarray(want).reshape(-1))


def test_keepdims_and_u32_out(ctx, orc):
    x = make((6, 33, 40), np.float32, seed=9)
    got = gpu_arg(ctx, abi.ARG_MAX, x, 1, keepdims=True, out_dtype=np.uint32)
    assert got.shape == (6, 1, 40)
    np.testing.assert_array_equal(got[:, 0, :], orc.argreduce(orc.ARGMAX, x, 1))


def test_errors(ctx):
    x = dev(np.ones((4, 0), np.float32))
    with pytest.raises(abi.QsmlError) as e:
        ctx.arg_reduce(abi.ARG_MAX, d(x), 1, False, d(empty((4,), np.int32)))
    assert e.value.status == abi.E_SHAPE
    y = dev(np.ones((4, 5), np.float32))
    with pytest.raises(abi.QsmlError) as e:
        ctx.arg_reduce(abi.ARG_MAX, d(y), 1, False, d(empty((4,), np.float32)))
    assert e.value.status == abi.E_DTYPE
    with pytest.raises(abi.QsmlError) as e:
        ctx.arg_reduce(7, d(y), 1, False, d(empty((4,), np.int32)))
    assert e.value.status == abi.E_INVALID
    with pytest.raises(abi.QsmlError) as e:
        ctx.arg_reduce(abi.ARG_MAX, d(y), 1, False, d(empty((5,), np.int32)))
    assert e.value.status == abi.E_SHAPE
    # empty outer: nothing to do
    z = dev(np.ones((0, 5), np.float32))
    ctx.arg_reduce(abi.ARG_MAX, d(z), 1, False, d(empty((0,), np.int32)))


@pytest.mark.parametrize("dtype", [np.float32, np.float16, np.int32])
@pytest.mark.parametrize("op", [abi.ARG_MAX, abi.ARG_MIN])
def test_transposed_views(ctx, orc, dtype, op):
    """A transpose is arg-reduced over an axis in place (the contiguous
    kernels on the underlying block); a full arg-reduction of it, or any other
    strided view, needs a contiguous input (QSML_E_UNSUPPORTED)."""
    x = make((300, 500), dtype, seed=31)
    t = dev(x)
    code = {np.dtype(np.float32): abi.F32, np.dtype(np.float16): abi.F16, np.dtype(np.int32): abi.I32}[np.dtype(dtype)]
    view = abi.make_desc(t.data_ptr(), code, (500, 300), (1, 500))
    xt = np.ascontiguousarray(x.T)
    oracle_op = orc.ARGMAX if op == abi.ARG_MAX else orc.ARGMIN
    for axis in (0, 1):
        out = empty(abi.reduced_shape((500, 300), axis, False), np.int32)
        ctx.arg_reduce(op, view, axis, False, d(out))
        np.testing.assert_array_equal(host(out).astype(np.int64), orc.argreduce(oracle_op, xt, axis))
    with pytest.raises(abi.QsmlError) as e:
        ctx.arg_reduce(op, view, abi.AXIS_ALL, False, d(empty((1,), np.int32)))
    assert e.value.status == abi.E_UNSUPPORTED
    sliced = abi.make_desc(t.data_ptr(), code, (150, 500), (1000, 1))  # X[::2]
    with pytest.raises(abi.QsmlError) as e:
        ctx.arg_reduce(op, sliced, 1, False, d(empty((150,), np.int32)))
    assert e.value.status == abi.E_UNSUPPORTED
