"""qsml_reduce_noalloc: the reduction entry point that allocates nothing.

It serves callers that cannot allocate device memory when they reduce --
latency-critical serving paths (cudaMalloc and cudaFree can synchronise the
device), hosts whose allocator owns all of HBM -- by keeping its scratch in a
fixed device array inside libqsml_cuda.so.  This file is named to be collected last.

Checked through the C ABI: two calls in a row on the same inputs must agree
with qsml_reduce (the context entry point).  Where qsml_reduce picks the same
segment kernel (the full reduction and few long rows) the results must be
bit-identical; where it picks another kernel (many short rows) they must agree
within the reduction tests' tolerance (sum/mean |diff| <= 1e-5 * sum|x|,
max/min exact).  Requests beyond the fixed scratch are rejected with a status
and a message.
"""
import ctypes

import numpy as np
import pytest

from quasarml_b200 import abi, datagen

pytestmark = pytest.mark.gpu

OPS = [abi.RED_SUM, abi.RED_MEAN, abi.RED_MAX, abi.RED_MIN]
CASES = [((64, 512, 1024), abi.AXIS_ALL), ((4, 100003), 1), ((8, 1 << 16), -1), ((3, 5000, 1), 1)]


def _noalloc(lib, stream, op, xd, axis, outd):
    return lib.qsml_reduce_noalloc(ctypes.c_void_p(stream) if stream else None, op, ctypes.byref(xd), axis, 0,
                                   ctypes.byref(outd))


@pytest.mark.parametrize("dtype", [np.float32, np.float16])
@pytest.mark.parametrize("shape,axis", CASES)
def test_noalloc_matches_context_entry_point(ctx, shape, axis, dtype):
    import torch
    lib = abi.load()
    stream = torch.cuda.current_stream().cuda_stream
    x_np = datagen.normal(51, shape, 0.25, 1.0).astype(dtype)
    scale = np.abs(x_np.astype(np.float64)).sum(axis=None if axis == abi.AXIS_ALL else axis).reshape(-1)
    x = torch.from_numpy(x_np).cuda()
    oshape = abi.reduced_shape(shape, None if axis == abi.AXIS_ALL else axis, False)
    tdt = torch.float32 if dtype == np.float32 else torch.float16
    for op in OPS:
        ref = torch.empty(oshape, dtype=tdt, device="cuda")
        ctx.reduce(op, abi.desc_of(x), axis, False, abi.desc_of(ref))
        same_kernel = ctx.last_kernel() == "k_reduce_seg"
        want_bits = ref.cpu().numpy().reshape(-1)
        want = want_bits.astype(np.float64)
        for call in range(2):
            out = torch.full(oshape, float("nan"), dtype=tdt, device="cuda")
            st = _noalloc(lib, stream, op, abi.desc_of(x), axis, abi.desc_of(out))
            assert st == abi.OK, lib.qsml_last_error(None).decode()
            got_bits = out.cpu().numpy().reshape(-1)
            got = got_bits.astype(np.float64)
            if same_kernel:
                assert np.array_equal(got_bits.view(np.uint8), want_bits.view(np.uint8)), (op, call, got[:4], want[:4])
            elif op in (abi.RED_MAX, abi.RED_MIN):
                assert np.array_equal(got, want), (op, call)
            else:
                k = x_np.size // got.size
                tol = 1e-5 * (scale if op == abi.RED_SUM else scale / k) + 1e-30
                if dtype == np.float16:
                    tol = tol + np.abs(want) * 2.0 ** -11
                # equal values (including a binary16 overflow to inf on both
                # paths) or within the tolerance
                with np.errstate(invalid="ignore"):
                    ok = (got == want) | (np.abs(got - want) <= tol)
                assert np.all(ok), (op, call, got[:4], want[:4])


def test_noalloc_rejects_beyond_its_scratch(ctx):
    import torch
    lib = abi.load()
    x = torch.zeros((65, 10), device="cuda")
    out = torch.empty((65,), device="cuda")
    st = _noalloc(lib, torch.cuda.current_stream().cuda_stream, abi.RED_SUM, abi.desc_of(x), 1, abi.desc_of(out))
    assert st == abi.E_UNSUPPORTED
    assert b"64 rows" in lib.qsml_last_error(None)
    y = torch.zeros((8, 16), device="cuda")
    st = _noalloc(lib, 0, abi.RED_SUM, abi.desc_of(y), 0, abi.desc_of(torch.empty((16,), device="cuda")))
    assert st == abi.E_UNSUPPORTED


def test_noalloc_rejects_an_empty_axis(ctx):
    import torch
    lib = abi.load()
    x = torch.zeros((3, 0), device="cuda")
    out = torch.empty((3,), device="cuda")
    st = _noalloc(lib, torch.cuda.current_stream().cuda_stream, abi.RED_SUM, abi.desc_of(x), 1, abi.desc_of(out))
    assert st == abi.E_SHAPE
