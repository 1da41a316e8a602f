"""GPU parity of the reductions (through the C ABI) against the oracle.

Tolerances:
* the bar for binary32 sum/mean, <= 1e-5 relative to the exact (binary64)
  result of EVERY output, is asserted at the configuration's shape
  X[64,512,1024] over each axis and all elements on a well-conditioned input
  (X ~ N(3,1), so no output is a cancellation), for binary32 input, binary16
  input with binary32 output, and binary16 in and out (plus the one binary16
  output rounding, 2^-11 relative);
* elsewhere (zero-mean inputs, odd shapes) sum/mean |gpu - exact| <=
  1e-5 * sum|x| (sum|x| is the scale of any summation's rounding error when
  outputs may cancel to near zero), plus one output rounding when the output
  is binary16.
max/min are order-free and bit-exact.  Results must also be bit-identical run
to run.
"""
import numpy as np
import pytest

from helpers import d, dev, empty, host
from quasarml_b200 import abi, datagen

pytestmark = pytest.mark.gpu

OPS = {"sum": abi.RED_SUM, "mean": abi.RED_MEAN, "max": abi.RED_MAX, "min": abi.RED_MIN}


def gpu_reduce(ctx, op, t, axis, keepdims=False, out_dtype=None):
    shape = abi.reduced_shape(tuple(t.shape), axis, keepdims)
    import torch
    odt = out_dtype or t.dtype
    out = torch.empty(shape, dtype=odt, device="cuda")
    ctx.reduce(op, d(t), abi.AXIS_ALL if axis is None else axis, keepdims, d(out))
    return host(out)


def check(orc, name, x_np, axis, g, out_is_half):
    o32, o64, ab = orc.reduce(OPS[name], x_np, axis)
    g = g.astype(np.float64).reshape(o64.shape)
    if name in ("max", "min"):
        ref = o32.astype(np.float16) if out_is_half else o32
        assert np.array_equal(g, ref.astype(np.float64)), name
        return
    tol = 1e-5 * ab + 1e-30
    if out_is_half:
        # a binary16 output holds the binary32 result rounded once, so a
        # result beyond the binary16 range is +-inf, as NumPy's would be
        with np.errstate(over="ignore"):
            r16 = o64.astype(np.float16)
        big = np.isinf(r16)
        assert np.array_equal(g[big], r16[big].astype(np.float64)), f"{name}: binary16 overflow"
        g, o64, ab, tol = g[~big], o64[~big], ab[~big], tol[~big]
        if g.size == 0:
            return
        tol = tol + np.abs(o64) * 2.0 ** -11
    err = np.abs(g - o64)
    worst = float(np.max(err / tol))
    assert worst <= 1.0, f"{name} axis={axis}: error {worst:.3g} x tolerance"


@pytest.fixture(scope="module")
def x3():
    return datagen.normal(datagen.SEEDS["red_X"], (64, 512, 1024), 0.0, 1.0)


@pytest.mark.parametrize("dtype", ["f32", "f16"])
@pytest.mark.parametrize("axis", [None, 0, 1, 2])
def test_workload_64x512x1024(ctx, orc, x3, dtype, axis):
    """X[64,512,1024] ~ N(0,1): sum/mean/max/min over each axis and all."""
    x = x3 if dtype == "f32" else x3.astype(np.float16)
    t = dev(x)
    for name, op in OPS.items():
        g = gpu_reduce(ctx, op, t, axis)
        check(orc, name, x, axis, g, dtype == "f16")
        g2 = gpu_reduce(ctx, op, t, axis)
        assert np.array_equal(g.view(np.uint8), g2.view(np.uint8)), "not deterministic"


@pytest.fixture(scope="module")
def x3pos():
    return datagen.normal(datagen.SEEDS["red_X"], (64, 512, 1024), 3.0, 1.0)


@pytest.mark.parametrize("case", ["f32", "f16_in_f32_out", "f16"])
@pytest.mark.parametrize("axis", [None, 0, 1, 2])
def test_workload_relative_bar(ctx, orc, x3pos, case, axis):
    """sum and mean of X[64,512,1024] ~ N(3,1): every output within 1e-5 of
    the exact result, relatively."""
    import torch
    x = x3pos if case == "f32" else x3pos.astype(np.float16)
    t = dev(x)
    for name in ("sum", "mean"):
        g = gpu_reduce(ctx, OPS[name], t, axis, out_dtype=torch.float32 if case == "f16_in_f32_out" else None)
        _, o64, _ = orc.reduce(OPS[name], x, axis)
        g = g.astype(np.float64).reshape(o64.shape)
        bar = 1e-5
        if case == "f16":
            with np.errstate(over="ignore"):
                r16 = o64.astype(np.float16)
            big = np.isinf(r16)  # beyond the binary16 range: +-inf, as NumPy's would be
            assert np.array_equal(g[big], r16[big].astype(np.float64)), f"{name}: binary16 overflow"
            g, o64 = g[~big], o64[~big]
            bar += 2.0 ** -11
            if g.size == 0:
                continue
        rel = float(np.max(np.abs(g - o64) / np.abs(o64)))
        print(f"{case} {name} axis={axis}: max relative error {rel:.3g} (bar {bar:.3g})")
        assert rel <= bar, f"{case} {name} axis={axis}: relative error {rel:.3g}"


def test_f16_input_f32_output(ctx, orc, x3):
    import torch
    x = x3[:8].astype(np.float16)
    t = dev(x)
    for axis in (None, 1, 2):
        for name, op in OPS.items():
            g = gpu_reduce(ctx, op, t, axis, out_dtype=torch.float32)
            check(orc, name, x, axis, g, False)


ODD = [((10,), None), ((10,), 0), ((4, 100003), 1), ((4, 100003), -1), ((33, 1001), 1), ((7, 13, 5), 1),
       ((7, 13, 5), 0), ((7, 13, 5), 2), ((1, 33), 0), ((5,), None), ((3, 70000), None), ((2, 3, 4, 5), 2),
       ((300, 8192), 1), ((8192, 3), 0), ((1, 1 << 20), 1), ((1000, 17), 1),
       # column kernel: long and short k, ragged tiles, unaligned rows
       ((3, 1000, 96), 1), ((2, 777, 1030), 1), ((5, 64, 2048), 0), ((9, 130, 4100), 1),
       # wide column kernel (short k, many 16-byte columns; ragged last span)
       ((37, 310000), 0), ((3, 50, 200000), 1), ((20, 620000), 0)]


@pytest.mark.parametrize("shape,axis", ODD)
@pytest.mark.parametrize("dtype", [np.float32, np.float16])
def test_odd_shapes(ctx, orc, shape, axis, dtype):
    x = datagen.normal(21, shape, 0.3, 1.5).astype(dtype)
    t = dev(x)
    for name, op in OPS.items():
        check(orc, name, x, axis, gpu_reduce(ctx, op, t, axis), dtype == np.float16)


def test_keepdims_and_shapes(ctx):
    x = dev(np.ones((4, 5, 6), np.float32))
    assert gpu_reduce(ctx, abi.RED_SUM, x, 1, keepdims=True).shape == (4, 1, 6)
    assert gpu_reduce(ctx, abi.RED_SUM, x, -1).shape == (4, 5)
    assert np.all(gpu_reduce(ctx, abi.RED_SUM, x, 2) == 6.0)
    y = dev(np.arange(1, 11, dtype=np.float32))
    # Reduction.cpp:297-305: reducing the only axis gives shape [1]
    assert gpu_reduce(ctx, abi.RED_MEAN, y, 0).shape == (1,)
    assert gpu_reduce(ctx, abi.RED_MEAN, y, 0)[0] == np.float32(5.5)
    with pytest.raises(abi.QsmlError) as e:
        ctx.reduce(abi.RED_SUM, d(x), 3, False, d(empty((4, 5), np.float32)))
    assert e.value.status == abi.E_SHAPE


def test_reference_known_answers(ctx):
    """_test_comprehensive.cpp:170-191: sum/mean/max/min of 1..10."""
    y = dev(np.arange(1, 11, dtype=np.float32))
    for op, want in ((abi.RED_SUM, 55.0), (abi.RED_MEAN, 5.5), (abi.RED_MAX, 10.0), (abi.RED_MIN, 1.0)):
        assert abs(float(gpu_reduce(ctx, op, y, None)[0]) - want) < 1e-3


def test_nan_and_signed_zero(ctx):
    x = np.zeros(100000, np.float32)
    x[::2] = -0.0
    t = dev(x)
    assert not np.signbit(gpu_reduce(ctx, abi.RED_MAX, t, None)[0])
    assert np.signbit(gpu_reduce(ctx, abi.RED_MIN, t, None)[0])
    x = datagen.normal(5, (3, 50000), 0, 1)
    x[1, 777] = np.nan
    t = dev(x)
    for op in OPS.values():
        r = gpu_reduce(ctx, op, t, 1)
        assert np.isnan(r[1]) and not np.isnan(r[0]) and not np.isnan(r[2])
    for op in (abi.RED_MAX, abi.RED_MIN):
        r = gpu_reduce(ctx, op, t, None)
        assert r.view(np.uint32)[0] == 0x7FFFFFFF  # canonical NaN
    inf = dev(np.float32([-np.inf, -np.inf, -np.inf]))
    assert gpu_reduce(ctx, abi.RED_MAX, inf, None)[0] == -np.inf


def test_empty_axis(ctx):
    x = empty((3, 0), np.float32)
    assert np.all(gpu_reduce(ctx, abi.RED_SUM, x, 1) == 0)
    assert np.all(np.isnan(gpu_reduce(ctx, abi.RED_MEAN, x, 1)))
    with pytest.raises(abi.QsmlError):
        gpu_reduce(ctx, abi.RED_MAX, x, 1)


def _view(base_np, t, offset, shape, strides):
    """A strided view of device tensor t (and the same view of base_np)."""
    es = base_np.itemsize
    code = abi.F32 if base_np.dtype == np.float32 else abi.F16
    desc = abi.make_desc(t.data_ptr() + offset * es, code, shape, strides)
    view = np.lib.stride_tricks.as_strided(base_np.reshape(-1)[offset:], shape=shape,
                                           strides=[st * es for st in strides])
    return desc, np.ascontiguousarray(view)


# (name, base shape, element offset, view shape, view strides in elements)
VIEWS = [("X[5::3, 1::2]", (64, 300), 5 * 300 + 1, (20, 150), (900, 2)),
         ("X.T", (70, 90), 0, (90, 70), (1, 90)),
         ("X.T[::4, :]", (64, 96), 0, (24, 64), (4, 96)),
         ("X.transpose(2, 0, 1)", (6, 40, 50), 0, (50, 6, 40), (1, 2000, 50)),
         ("X[::-1, :]", (30, 40), 29 * 40, (30, 40), (-40, 1)),
         ("broadcast [1,500] -> [7,500]", (1, 500), 0, (7, 500), (0, 1)),
         ("X[::3] of 300000", (300000,), 0, (100000,), (3,)),
         ("X[::2, ::-1] of [4, 70000]", (4, 70000), 69999, (2, 70000), (140000, -1)),
         ("X[1::2, ::3] of [4000, 300]", (4000, 300), 300, (2000, 100), (600, 3))]


@pytest.mark.parametrize("view", VIEWS, ids=[v[0] for v in VIEWS])
@pytest.mark.parametrize("dtype", [np.float32, np.float16])
def test_strided_views(ctx, orc, view, dtype):
    """Reductions read views in place (no gather copy): every axis and all
    elements, against the oracle on the materialised view (sum/mean within
    1e-5 * sum|x|, max/min bit-exact)."""
    import torch
    name, bshape, off, shape, strides = view
    base = datagen.normal(23, bshape, 0.3, 1.5).astype(dtype)
    t = dev(base)
    desc, x = _view(base, t, off, shape, strides)
    tdt = torch.float32 if dtype == np.float32 else torch.float16
    for axis in [None] + list(range(len(shape))):
        for oname, op in OPS.items():
            out = torch.empty(abi.reduced_shape(shape, axis, False), dtype=tdt, device="cuda")
            ctx.reduce(op, desc, abi.AXIS_ALL if axis is None else axis, False, abi.desc_of(out))
            assert ctx.last_kernel().startswith("k_reduce_"), ctx.last_kernel()
            check(orc, oname, x, axis, host(out), dtype == np.float16)


def test_strided_view_kernels(ctx):
    """Rows of a sliced matrix are read along k (a warp per output); its
    columns a lane per output, k split over warps (and, for few outputs over a
    long k, CTAs with partials combined in order)."""
    base = np.ones((64, 300), np.float32)
    t = dev(base)
    desc, _ = _view(base, t, 5 * 300 + 1, (20, 150), (900, 2))
    out = empty((20,), np.float32)
    ctx.reduce(abi.RED_SUM, desc, 1, False, d(out))
    assert ctx.last_kernel() == "k_reduce_strided_lanes"
    assert np.all(host(out) == 150.0)
    out = empty((150,), np.float32)
    ctx.reduce(abi.RED_SUM, desc, 0, False, d(out))
    assert ctx.last_kernel() == "k_reduce_strided_cols"
    assert np.all(host(out) == 20.0)
    # 2000 rows of 100 columns: k cut over CTAs (7 chunks)
    base = np.ones((4000, 300), np.float32)
    t = dev(base)
    desc, _ = _view(base, t, 300, (2000, 100), (600, 3))
    out = empty((100,), np.float32)
    for _ in range(3):  # ticket counters are reset for the next launch
        ctx.reduce(abi.RED_SUM, desc, 0, False, d(out))
        assert ctx.last_kernel() == "k_reduce_strided_cols"
        assert np.all(host(out) == 2000.0)


@pytest.mark.parametrize("dtype", [np.float32, np.float16])
def test_transposed_views_use_contiguous_kernels(ctx, orc, dtype):
    """A transpose (a permuted contiguous block) is reduced by the contiguous
    kernels: X.T over its axis 0 is X's rows, over its axis 1 X's columns (few
    column tiles over a long k: k also split over CTAs)."""
    import torch
    base = datagen.normal(24, (4096, 2048), 0.3, 1.5).astype(dtype)
    t = dev(base)
    desc, x = _view(base, t, 0, (2048, 4096), (1, 2048))
    tdt = torch.float32 if dtype == np.float32 else torch.float16
    for axis, kernel in ((0, "k_reduce_rows"), (1, "k_reduce_cols_split"), (None, "k_reduce_seg")):
        for oname, op in OPS.items():
            out = torch.empty(abi.reduced_shape((2048, 4096), axis, False), dtype=tdt, device="cuda")
            ctx.reduce(op, desc, abi.AXIS_ALL if axis is None else axis, False, abi.desc_of(out))
            assert ctx.last_kernel() == kernel, (axis, ctx.last_kernel())
            check(orc, oname, x, axis, host(out), dtype == np.float16)


def test_view_beyond_four_output_dims_is_unsupported(ctx):
    """Dims that do not merge beyond four output dims: QSML_E_UNSUPPORTED
    (the C++ layer then reduces a gathered copy)."""
    base = np.ones((2, 3, 4, 5, 6, 7), np.float32)
    t = dev(base)
    st = [3 * 4 * 5 * 6 * 7, 4 * 5 * 6 * 7, 5 * 6 * 7, 6 * 7, 7, 1]
    desc = abi.make_desc(t.data_ptr(), abi.F32, (7, 6, 5, 4, 3, 2), st[::-1])
    with pytest.raises(abi.QsmlError) as e:
        ctx.reduce(abi.RED_SUM, desc, 0, False, d(empty((6, 5, 4, 3, 2), np.float32)))
    assert e.value.status == abi.E_UNSUPPORTED


@pytest.mark.parametrize("shape,axis", [((1000,), None), ((7, 300), 1), ((5, 40, 3), 1), ((3, 100000), 1)])
def test_prod(ctx, orc, shape, axis):
    """prod (Reduction.cpp:190-211 in the reference): |err| <= n * 2^-24 * |exact|
    (the worst-case bound of n binary32 roundings)."""
    x = datagen.uniform(61, shape, 0.999, 1.001)
    g = gpu_reduce(ctx, abi.RED_PROD, dev(x), axis).astype(np.float64)
    _, o64, _ = orc.reduce(orc.PROD, x, axis)
    n = x.size if axis is None else x.shape[axis]
    assert np.all(np.abs(g.reshape(o64.shape) - o64) <= n * 2.0 ** -24 * np.abs(o64))


def test_long_column_reduction(ctx, orc):
    """A long column reduction: 2.1 million columns, k = 66."""
    x = datagen.normal(22, (66, 2_100_000), 0.3, 1.5)
    t = dev(x)
    for name, op in OPS.items():
        check(orc, name, x, 0, gpu_reduce(ctx, op, t, 0), False)


@pytest.mark.parametrize("shape,axis,kernel", [((64, 512, 1024), 0, "k_reduce_cols_wide"),
                                               ((64, 512, 1024), 1, "k_reduce_cols"),
                                               ((64, 512, 1024), 2, "k_reduce_rows"),
                                               ((64, 512, 1024), None, "k_reduce_seg"),
                                               ((37, 310000), 0, "k_reduce_cols_wide"),
                                               ((4096, 2048), 0, "k_reduce_cols_split")])
def test_kernel_choice(ctx, shape, axis, kernel):
    """The workload shapes reach the kernel each was tuned for (fp32)."""
    t = dev(np.zeros(shape, np.float32))
    gpu_reduce(ctx, abi.RED_SUM, t, axis)
    assert ctx.last_kernel() == kernel
