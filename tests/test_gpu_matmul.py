"""GPU matmul (through the C ABI).

fp32 (QSML_MM_FP32_FFMA): the kernel keeps the reference's per-output fma
chain in k order, so small cases are bit-identical to the oracle's chain.
At the configuration sizes (8192^3 and the batched
[32,2048,1024] x [32,1024,2048]) EVERY output of every path is checked
against the binary64 product (oracle.matmul_check):
  |c - ref| <= tol * (|A|.|B|) for each output  (componentwise bound), and
  ||c - ref||_F / ||ref||_F <= tol               (normwise),
with tol = 1e-4 for fp32 (FFMA, 3xTF32) and 1e-2 for fp16 inputs with fp32
accumulation (against the product of the same fp16 inputs; the fp16 paths
are also held to 1e-4, which fp32 accumulation meets).  Both fp16 kernels
(one SM and SM pairs, QSML_GEMM_2SM=0/1) are checked.
"""
import numpy as np
import pytest

from helpers import assert_bits_equal, d, dev, empty, host
from quasarml_b200 import abi, datagen

pytestmark = pytest.mark.gpu


def mm(ctx, a, b, out_dtype=np.float32, precision=abi.MM_AUTO):
    ta, tb = dev(a), dev(b)
    shape = a.shape[:-1] + (b.shape[-1],)
    c = empty(shape, out_dtype)
    ctx.matmul(d(ta), d(tb), d(c), precision)
    return host(c)


@pytest.mark.parametrize("mkn", [(1, 1, 1), (2, 3, 4), (129, 65, 257), (256, 256, 256), (300, 1000, 70),
                                 (64, 8, 128), (5, 300, 3)])
def test_fp32_bitexact_small(ctx, orc, mkn):
    M, K, N = mkn
    a = datagen.uniform(41, (M, K), -1, 1)
    b = datagen.uniform(42, (K, N), -1, 1)
    assert_bits_equal(mm(ctx, a, b, precision=abi.MM_FP32_FFMA), orc.matmul_fma(a, b), str(mkn))


def test_reference_known_answer(ctx):
    """_test_qsml_functionality.cpp:135-143: ones[2,3] @ ones[3,4] = 3."""
    c = mm(ctx, np.ones((2, 3), np.float32), np.ones((3, 4), np.float32))
    assert c.shape == (2, 4) and np.all(c == 3.0)


def _assert_full(orc, C, A, B, tol, what):
    worst, normwise, maxrel = orc.matmul_check(C, A, B)
    print(f"{what}: componentwise {worst:.3g}, normwise {normwise:.3g}, max|err|/max|ref| {maxrel:.3g} (bar {tol:g})")
    assert worst <= tol, (what, "componentwise", worst)
    assert normwise <= tol, (what, "normwise", normwise)


@pytest.fixture(scope="module")
def sq():
    s = 1.0 / np.sqrt(8192.0)
    return (datagen.uniform(datagen.SEEDS["mm_A"], (8192, 8192), -s, s),
            datagen.uniform(datagen.SEEDS["mm_B"], (8192, 8192), -s, s))


@pytest.fixture(scope="module")
def bat():
    s = 1.0 / np.sqrt(1024.0)
    return (datagen.uniform(datagen.SEEDS["mm_Ab"], (32, 2048, 1024), -s, s),
            datagen.uniform(datagen.SEEDS["mm_Bb"], (32, 1024, 2048), -s, s))


PATHS = [("ffma", abi.MM_FP32_FFMA, None, 1e-4), ("3xtf32", abi.MM_FP32_3XTF32, None, 1e-4),
         ("f16_one_sm", abi.MM_FP16_F32ACC, "0", 1e-2), ("f16_sm_pair", abi.MM_FP16_F32ACC, "1", 1e-2)]


@pytest.mark.parametrize("name,prec,two_sm,tol", PATHS, ids=[p[0] for p in PATHS])
def test_8192_every_output(ctx, orc, sq, monkeypatch, name, prec, two_sm, tol):
    A, B = sq
    if two_sm is not None:
        monkeypatch.setenv("QSML_GEMM_2SM", two_sm)
        A, B = A.astype(np.float16), B.astype(np.float16)
    C = mm(ctx, A, B, precision=prec)
    if two_sm is not None:
        assert ctx.last_kernel().startswith("k_gemm_tc2<" if two_sm == "1" else "k_gemm_tc<"), ctx.last_kernel()
    _assert_full(orc, C, A, B, tol, f"8192^3 {name}")
    if two_sm is not None:
        _assert_full(orc, C, A, B, 1e-4, f"8192^3 {name}, fp32-accumulation bar")


@pytest.mark.parametrize("name,prec,two_sm,tol", PATHS, ids=[p[0] for p in PATHS])
def test_batched_every_output(ctx, orc, bat, monkeypatch, name, prec, two_sm, tol):
    A, B = bat
    if two_sm is not None:
        monkeypatch.setenv("QSML_GEMM_2SM", two_sm)
        A, B = A.astype(np.float16), B.astype(np.float16)
    C = mm(ctx, A, B, precision=prec)
    _assert_full(orc, C, A, B, tol, f"batched 32x2048x1024x2048 {name}")
    if two_sm is not None:
        _assert_full(orc, C, A, B, 1e-4, f"batched {name}, fp32-accumulation bar")


def test_batched_small_bitexact(ctx, orc):
    a = datagen.uniform(43, (3, 33, 17), -1, 1)
    b = datagen.uniform(44, (3, 17, 9), -1, 1)
    assert_bits_equal(mm(ctx, a, b), orc.matmul_fma(a, b), "batched small")


@pytest.mark.parametrize("mkn", [(128, 64, 128), (256, 512, 384), (100, 72, 200), (1, 64, 64), (512, 1024, 256)])
@pytest.mark.parametrize("out", [np.float32, np.float16])
def test_fp16_small(ctx, orc, mkn, out):
    M, K, N = mkn
    a = datagen.uniform(45, (M, K), -1, 1).astype(np.float16)
    b = datagen.uniform(46, (K, N), -1, 1).astype(np.float16)
    c = mm(ctx, a, b, out_dtype=out, precision=abi.MM_FP16_F32ACC).astype(np.float64)
    ref = orc.matmul_f64(a, b)
    err = np.max(np.abs(c - ref)) / np.max(np.abs(ref))
    assert err <= (1e-5 if out == np.float32 else 1e-3), err


def test_shared_b_batch_stride_zero(ctx, orc):
    a = datagen.uniform(47, (4, 16, 8), -1, 1)
    b = datagen.uniform(48, (8, 12), -1, 1)
    ta, tb = dev(a), dev(b)
    bview = abi.make_desc(tb.data_ptr(), abi.F32, (4, 8, 12), (0, 12, 1))
    c = empty((4, 16, 12), np.float32)
    ctx.matmul(d(ta), bview, d(c))
    ref = orc.matmul_fma(a, np.broadcast_to(b, (4, 8, 12)).copy())
    assert_bits_equal(host(c), ref, "stride-0 B")


def test_errors(ctx):
    with pytest.raises(abi.QsmlError) as e:
        mm(ctx, np.ones((2, 3), np.float32), np.ones((4, 5), np.float32))
    assert e.value.status == abi.E_SHAPE
    with pytest.raises(abi.QsmlError) as e:
        ctx.matmul(d(dev(np.ones((2, 3), np.float32))), d(dev(np.ones((3, 2), np.float16))),
                   d(empty((2, 2), np.float32)))
    assert e.value.status == abi.E_DTYPE


@pytest.mark.parametrize("mkn", [(128, 64, 128), (256, 512, 384), (100, 72, 200), (1, 64, 64), (512, 1024, 256),
                                 (300, 1000, 72)])
def test_fp32_3xtf32_small(ctx, orc, mkn):
    """fp32 via three tf32 tensor-core products: max|err| / max|ref| <= 1e-4
    against binary64 (observed errors are near fp32 rounding)."""
    M, K, N = mkn
    a = datagen.uniform(49, (M, K), -1, 1)
    b = datagen.uniform(50, (K, N), -1, 1)
    c = mm(ctx, a, b, precision=abi.MM_FP32_3XTF32).astype(np.float64)
    ref = orc.matmul_f64(a, b)
    err = np.max(np.abs(c - ref)) / np.max(np.abs(ref))
    assert err <= 1e-4, err
    assert err <= 1e-5, err  # far tighter than the fp32 bar in practice


def test_fp32_3xtf32_rejects_unsupported_shapes(ctx):
    with pytest.raises(abi.QsmlError) as e:
        mm(ctx, np.ones((4, 33), np.float32), np.ones((33, 8), np.float32), precision=abi.MM_FP32_3XTF32)
    assert e.value.status == abi.E_UNSUPPORTED
