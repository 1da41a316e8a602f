"""Helpers shared by the GPU parity tests (device copies, views, tolerances)."""
import numpy as np

from quasarml_b200 import abi


def dev(x: np.ndarray):
    import torch
    return torch.from_numpy(np.ascontiguousarray(x)).cuda()


def host(t) -> np.ndarray:
    import torch
    torch.cuda.current_stream().synchronize()
    return t.cpu().numpy()


def empty(shape, np_dtype):
    import torch
    tdt = {np.dtype(np.float32): torch.float32, np.dtype(np.float16): torch.float16,
           np.dtype(np.int32): torch.int32, np.dtype(np.int16): torch.int16,
           np.dtype(np.int8): torch.int8, np.dtype(np.uint8): torch.uint8}[np.dtype(np_dtype)]
    return torch.empty(tuple(shape), dtype=tdt, device="cuda")


def d(t):
    return abi.desc_of(t)


def ulp_f32(x, y):
    """binary32 ulp distance, NaN==NaN counts 0, NaN vs number is huge."""
    x = np.ascontiguousarray(x, dtype=np.float32)
    y = np.ascontiguousarray(y, dtype=np.float32)
    xi = x.view(np.int32).astype(np.int64)
    yi = y.view(np.int32).astype(np.int64)
    xi = np.where(xi < 0, -(xi & 0x7FFFFFFF), xi)
    yi = np.where(yi < 0, -(yi & 0x7FFFFFFF), yi)
    dd = np.abs(xi - yi)
    xn, yn = np.isnan(x), np.isnan(y)
    dd = np.where(xn & yn, 0, dd)
    dd = np.where(xn ^ yn, 1 << 40, dd)
    return dd


def assert_bits_equal(gpu, ref, what=""):
    g = np.ascontiguousarray(gpu)
    r = np.ascontiguousarray(ref)
    assert g.shape == r.shape, (what, g.shape, r.shape)
    if g.dtype.kind == "f":
        gn, rn = np.isnan(g), np.isnan(r)
        assert np.array_equal(gn, rn), f"{what}: NaN positions differ"
        gv = g.view(np.uint32 if g.itemsize == 4 else np.uint16)
        rv = r.view(np.uint32 if r.itemsize == 4 else np.uint16)
        bad = (gv != rv) & ~gn
    else:
        bad = g != r
    nbad = int(np.count_nonzero(bad))
    if nbad:
        idx = np.argwhere(bad)[:5]
        raise AssertionError(f"{what}: {nbad} elements differ, first at {idx.tolist()}: "
                             f"gpu={g[tuple(idx[0])]!r} ref={r[tuple(idx[0])]!r}")
