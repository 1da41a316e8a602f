"""Layer norm and last-axis softmax on rows streamed through shared memory by
bulk copies: one warp per row for rows of 2-8 KiB (binary16) or 2-4 KiB
(binary32); one CTA per row for binary16 rows above 8 KiB (softmax: from 8
KiB) and binary32 rows from 32 KiB, both up to 108 KiB.  The CTA has 128
threads up to 16 KiB rows, 256 for binary16 rows up to 52 KiB (layer norm
with binary32 gamma/beta on 16-32 KiB rows: 512) and 512 beyond.  The shapes
below also include rows that take the register-resident or the generic
kernels, and each case checks which kernel ran (qsml_last_kernel).  Covered:
rows whose 16-byte packs do not divide evenly over the 32 lanes, rows just
above and far above the SM count, 16 warps per CTA, and special values.
Bars as in the other layer norm and softmax tests: binary32
|y - ref| <= 1e-5 * max(|ref|, 0.1) (layer norm) or 1e-5 * ref + 1e-30
(softmax); binary16 1e-3 relative.
"""
import numpy as np
import pytest

from helpers import d, dev, empty, host
from quasarml_b200 import abi, datagen

pytestmark = pytest.mark.gpu

# (shape, dtype, kernel family: "pipe" = a warp per row, "wide" = a CTA per row,
# both streamed through shared memory; None = the register or generic kernels;
# a pair = (layer norm, softmax) where they differ)
SHAPES = [
    ((5000, 1000), np.float32, "pipe"),    # 4000-byte rows, 250 packs: ragged over the lanes
    ((3000, 1032), np.float16, "pipe"),    # 2064-byte rows, 129 packs
    ((20000, 512), np.float32, "pipe"),    # 2 KiB rows: 16 warps per CTA
    ((16384, 4096), np.float16, ("pipe", "wide")),  # 8 KiB binary16 rows: softmax a CTA per row
    ((149, 2048), np.float32, None),       # 8 KiB binary32 rows: register kernel
    ((200, 4104), np.float16, "wide"),     # 8208-byte binary16 rows: 128 threads
    ((300, 6000), np.float16, "wide"),     # 12,000-byte rows, 750 packs over 128 threads
    ((100, 6000), np.float16, "wide"),     # the same rows, fewer than the SMs
    ((150, 12288), np.float16, "wide"),    # 24 KiB binary16 rows
    ((200, 16384), np.float16, "wide"),    # 32 KiB binary16 rows: 8 packs per thread at 256
    ((300, 12000), np.float32, "wide"),    # 48,000-byte rows
    ((400, 18000), np.float16, "wide"),    # 36,000-byte rows
    ((1024, 16384), np.float32, "wide"),   # 64 KiB rows
    ((160, 27648), np.float32, "wide"),    # 108 KiB rows: the widest streamed
    ((50, 27652), np.float32, None),       # wider: generic kernels
]


def ln(ctx, x, g, b, eps=1e-5):
    tx, tg, tb = dev(x), dev(g), dev(b)
    y = empty(x.shape, x.dtype)
    ctx.layer_norm(d(tx), d(tg), d(tb), eps, d(y))
    return host(y)


def softmax(ctx, x):
    tx = dev(x)
    y = empty(x.shape, x.dtype)
    ctx.softmax(d(tx), -1, d(y))
    return host(y)


@pytest.mark.parametrize("case", range(len(SHAPES)))
def test_layer_norm(ctx, orc, case):
    shape, dtype, family = SHAPES[case]
    family = family[0] if isinstance(family, tuple) else family
    x = datagen.normal(70 + case, shape, 0.5, 2.0).astype(dtype)
    g = datagen.normal(80 + case, shape[-1:], 1.0, 0.1)
    b = datagen.normal(90 + case, shape[-1:], 0.0, 0.1)
    y = ln(ctx, x, g, b).astype(np.float64)
    want = {"pipe": "k_layer_norm_pipe", "wide": "k_layer_norm_wide"}.get(family)
    assert ctx.last_kernel() == want if want else ctx.last_kernel() not in ("k_layer_norm_pipe", "k_layer_norm_wide"), \
        ctx.last_kernel()
    ref = orc.layer_norm(x, g, b, 1e-5).astype(np.float64)
    tol = 1e-5 if dtype == np.float32 else 1e-3
    worst = np.max(np.abs(y - ref) / (tol * np.maximum(np.abs(ref), 0.1)))
    assert worst <= 1.0, (shape, dtype, worst)


@pytest.mark.parametrize("case", range(len(SHAPES)))
def test_softmax(ctx, orc, case):
    shape, dtype, family = SHAPES[case]
    family = family[1] if isinstance(family, tuple) else family
    x = datagen.normal(100 + case, shape, 0.5, 2.0).astype(dtype)
    got = softmax(ctx, x).astype(np.float64)
    want = {"pipe": "k_softmax_pipe", "wide": "k_softmax_wide"}.get(family)
    assert ctx.last_kernel() == want if want else ctx.last_kernel() not in ("k_softmax_pipe", "k_softmax_wide"), \
        ctx.last_kernel()
    ref = orc.softmax(x, -1)
    rtol, atol = (1e-5, 1e-30) if dtype == np.float32 else (1e-3, 1e-7)
    assert np.max(np.abs(got - ref) - rtol * ref) <= atol, (shape, dtype)
    if dtype == np.float32:
        assert np.max(np.abs(got.sum(axis=-1) - 1.0)) <= 1e-5


@pytest.mark.parametrize("dtype", [np.float32, np.float16])
def test_softmax_special_rows(ctx, orc, dtype):
    x = datagen.normal(111, (300, 1024), 0.0, 1.0).astype(np.float32)
    x[5, 17] = np.nan
    x[6, :] = 2.5
    x[7, :] = -np.inf
    x[7, 100] = 0.0
    x[7, 999] = 0.0
    x[8, 3] = np.inf
    x[9, 0] = 80.0
    x[9, 1] = -80.0
    x = x.astype(dtype)
    got = softmax(ctx, x)
    assert ctx.last_kernel() == "k_softmax_pipe"
    assert np.all(np.isnan(got[5]))
    assert np.all(got[6] == dtype(1.0 / 1024))
    assert got[7][100] == dtype(0.5) and got[7][999] == dtype(0.5)
    assert np.count_nonzero(got[7]) == 2
    assert np.isnan(got[8][3])  # inf - inf
    ref = orc.softmax(x, -1)
    ok = ~np.isnan(ref)
    ok[5] = ok[8] = False
    rtol, atol = (1e-5, 1e-30) if dtype == np.float32 else (1e-3, 1e-7)
    assert np.max(np.abs(got.astype(np.float64)[ok] - ref[ok]) - rtol * ref[ok]) <= atol


def test_layer_norm_constant_rows_and_determinism(ctx, orc):
    x = datagen.normal(112, (600, 1024), 0.5, 2.0)
    x[::3] = 3.0
    g = np.ones(1024, np.float32)
    b = np.full(1024, 0.25, np.float32)
    y1 = ln(ctx, x, g, b)
    assert ctx.last_kernel() == "k_layer_norm_pipe"
    y2 = ln(ctx, x, g, b)
    assert np.array_equal(y1.view(np.uint32), y2.view(np.uint32))
    assert np.all(y1[::3] == np.float32(0.25))
    ref = orc.layer_norm(x, g, b, 1e-5)
    assert np.max(np.abs(y1 - ref) / (1e-5 * np.maximum(np.abs(ref), 0.1))) <= 1.0


def test_layer_norm_f16_params_and_few_rows(ctx, orc):
    """binary16 gamma/beta through the streamed kernel, and fewer rows than SMs
    (one warp per CTA)."""
    for shape in ((2000, 1024), (5, 2048)):
        x = datagen.normal(113, shape, 0.5, 2.0).astype(np.float16)
        g = datagen.normal(114, shape[-1:], 1.0, 0.1).astype(np.float16)
        b = datagen.normal(115, shape[-1:], 0.0, 0.1).astype(np.float16)
        y = ln(ctx, x, g, b).astype(np.float64)
        assert ctx.last_kernel() == "k_layer_norm_pipe"
        ref = orc.layer_norm(x, g.astype(np.float32), b.astype(np.float32), 1e-5).astype(np.float64)
        assert np.max(np.abs(y - ref) / (1e-3 * np.maximum(np.abs(ref), 0.1))) <= 1.0, shape


@pytest.mark.parametrize("shape", [(300, 6000), (150, 12288), (100, 24576), (60, 40000)])
def test_layer_norm_wide_f16_params(ctx, orc, shape):
    """binary16 gamma/beta through each CTA-per-row variant: in registers
    (12,000-byte rows), from L1/L2 with 256 threads (24 and 48 KiB) and with
    512 threads (80,000-byte rows)."""
    x = datagen.normal(116, shape, 0.5, 2.0).astype(np.float16)
    g = datagen.normal(117, shape[-1:], 1.0, 0.1).astype(np.float16)
    b = datagen.normal(118, shape[-1:], 0.0, 0.1).astype(np.float16)
    y = ln(ctx, x, g, b).astype(np.float64)
    assert ctx.last_kernel() == "k_layer_norm_wide"
    ref = orc.layer_norm(x, g.astype(np.float32), b.astype(np.float32), 1e-5).astype(np.float64)
    assert np.max(np.abs(y - ref) / (1e-3 * np.maximum(np.abs(ref), 0.1))) <= 1.0, shape
