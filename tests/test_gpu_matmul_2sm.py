"""fp16 matmul on pairs of SMs (tcgen05 cta_group::2, 256 x 256 tiles).

QSML_GEMM_2SM selects the fp16 kernel on each call: 1 forces the SM-pair
kernel, 0 the one-SM kernel (otherwise the pair kernel runs when the
256 x 256 tiles fill the SM pairs).  Both run every shape here, which covers
tiles cut by M, N and K at every edge, the M half of the pair that lies
wholly past M, batched A with shared (stride-0) B, and fp16 output.
Tolerance: max|err| / max|ref| <= 1e-5 (fp32 output) or 1e-3 (fp16 output)
against binary64 products of the same fp16 inputs; the two kernels agree to
1e-6 of max|ref| on the same inputs.
"""
import numpy as np
import pytest

from helpers import d, dev, empty, host
from quasarml_b200 import abi, datagen

pytestmark = pytest.mark.gpu


@pytest.fixture(params=["0", "1"], ids=["one_sm", "sm_pair"])
def kernel(request, monkeypatch):
    monkeypatch.setenv("QSML_GEMM_2SM", request.param)
    return request.param


def mm(ctx, a_t, b_desc, shape, out):
    c = empty(shape, out)
    ctx.matmul(d(a_t), b_desc, d(c), abi.MM_FP16_F32ACC)
    return host(c)


SHAPES = [(128, 64, 128), (256, 512, 384), (100, 72, 200), (1, 64, 64), (300, 64, 520), (257, 136, 264),
          (513, 1024, 776), (2048, 64, 2048), (64, 4104, 8)]


@pytest.mark.parametrize("mkn", SHAPES)
@pytest.mark.parametrize("out", [np.float32, np.float16])
def test_fp16_shapes(ctx, orc, kernel, mkn, out):
    M, K, N = mkn
    a = datagen.uniform(61, (M, K), -1, 1).astype(np.float16)
    b = datagen.uniform(62, (K, N), -1, 1).astype(np.float16)
    tb = dev(b)
    c = mm(ctx, dev(a), d(tb), (M, N), out).astype(np.float64)
    assert ctx.last_kernel().startswith("k_gemm_tc2<" if kernel == "1" else "k_gemm_tc<"), ctx.last_kernel()
    ref = orc.matmul_f64(a, b)
    err = np.max(np.abs(c - ref)) / np.max(np.abs(ref))
    assert err <= (1e-5 if out == np.float32 else 1e-3), (kernel, err)


def test_batched_shared_b(ctx, orc, kernel):
    a = datagen.uniform(63, (6, 300, 128), -1, 1).astype(np.float16)
    b = datagen.uniform(64, (128, 264), -1, 1).astype(np.float16)
    tb = dev(b)
    bview = abi.make_desc(tb.data_ptr(), abi.F16, (6, 128, 264), (0, 264, 1))
    c = mm(ctx, dev(a), bview, (6, 300, 264), np.float32).astype(np.float64)
    for i in range(6):
        ref = orc.matmul_f64(a[i], b)
        err = np.max(np.abs(c[i] - ref)) / np.max(np.abs(ref))
        assert err <= 1e-5, (kernel, i, err)


def test_batched_shared_a(ctx, orc, kernel):
    a = datagen.uniform(67, (200, 136), -1, 1).astype(np.float16)
    b = datagen.uniform(68, (5, 136, 520), -1, 1).astype(np.float16)
    ta = dev(a)
    aview = abi.make_desc(ta.data_ptr(), abi.F16, (5, 200, 136), (0, 136, 1))
    c = empty((5, 200, 520), np.float32)
    ctx.matmul(aview, d(dev(b)), d(c), abi.MM_FP16_F32ACC)
    got = host(c).astype(np.float64)
    for i in range(5):
        ref = orc.matmul_f64(a, b[i])
        assert np.max(np.abs(got[i] - ref)) / np.max(np.abs(ref)) <= 1e-5, (kernel, i)


def test_kernels_agree(ctx, monkeypatch):
    s = 1.0 / np.sqrt(1024.0)
    a = datagen.uniform(65, (4, 1024, 1024), -s, s).astype(np.float16)
    b = datagen.uniform(66, (4, 1024, 1024), -s, s).astype(np.float16)
    ta, tb = dev(a), dev(b)
    outs = []
    for mode in ("0", "1"):
        monkeypatch.setenv("QSML_GEMM_2SM", mode)
        outs.append(mm(ctx, ta, d(tb), (4, 1024, 1024), np.float32))
    scale = float(np.max(np.abs(outs[0])))
    assert float(np.max(np.abs(outs[0] - outs[1]))) <= 1e-6 * scale


def test_auto_choice(ctx, monkeypatch):
    """Without QSML_GEMM_2SM the SM-pair kernel runs when the 256 x 256 tiles
    fill the SM pairs at least once, the one-SM kernel otherwise."""
    monkeypatch.delenv("QSML_GEMM_2SM", raising=False)
    big = dev(np.zeros((4096, 64), np.float16)), dev(np.zeros((64, 4096), np.float16))
    mm(ctx, big[0], d(big[1]), (4096, 4096), np.float32)
    assert ctx.last_kernel().startswith("k_gemm_tc2<"), ctx.last_kernel()
    small = dev(np.zeros((512, 64), np.float16)), dev(np.zeros((64, 512), np.float16))
    mm(ctx, small[0], d(small[1]), (512, 512), np.float32)
    assert ctx.last_kernel().startswith("k_gemm_tc<"), ctx.last_kernel()


# Column counts whose last tile holds an odd number of 128-byte output chunks
# (8 and 160 columns past the last full 256-column tile), with rows that end
# inside a tile (900: whole 32-row warps of the last tile lie past M), over
# enough tiles that every epilogue warp stores many tiles in a row.  Each
# epilogue warp alternates two staging buffers under in-flight TMA stores;
# this is the case where a buffer choice restarted per tile would overwrite a
# buffer a store is still reading.  Repeated calls into NaN-filled outputs.
@pytest.mark.parametrize("mkn", [(900, 520, 776), (1000, 264, 416)])
@pytest.mark.parametrize("out", [np.float32, np.float16])
def test_ragged_tiles_repeated(ctx, kernel, mkn, out):
    M, K, N = mkn
    E = 20
    a = datagen.uniform(71, (E, M, K), -1, 1).astype(np.float16)
    b = datagen.uniform(72, (E, K, N), -1, 1).astype(np.float16)
    ta, tb = dev(a), dev(b)
    ref = np.matmul(a.astype(np.float64), b.astype(np.float64))
    scale = np.max(np.abs(ref))
    for call in range(6):
        c = empty((E, M, N), out)
        c.fill_(float("nan"))
        ctx.matmul(d(ta), d(tb), d(c), abi.MM_FP16_F32ACC)
        got = host(c).astype(np.float64)
        assert ctx.last_kernel().startswith("k_gemm_tc2<" if kernel == "1" else "k_gemm_tc<"), ctx.last_kernel()
        err = np.max(np.abs(got - ref)) / scale  # NaN (an unwritten output) fails too
        assert err <= (1e-5 if out == np.float32 else 1e-3), (kernel, call, err)
