"""GPU strided gather (through the C ABI): bit-exact against the oracle."""
import numpy as np
import pytest

from helpers import assert_bits_equal, d, dev, empty, host
from quasarml_b200 import abi, datagen

pytestmark = pytest.mark.gpu


def view_desc(t, offset, shape, strides):
    """Descriptor of a view of contiguous torch tensor t (element offset/strides)."""
    code = abi.torch_dtype_code(t.dtype)
    return abi.make_desc(t.data_ptr() + offset * t.element_size(), code, shape, strides)


def gpu_gather(ctx, t, offset, shape, strides):
    import torch
    out = torch.empty(tuple(shape), dtype=t.dtype, device="cuda")
    ctx.gather(view_desc(t, offset, shape, strides), d(out))
    return host(out)


def numpy_view(X, view):
    off = (view.__array_interface__["data"][0] - X.__array_interface__["data"][0]) // X.itemsize
    return off, view.shape, [s // X.itemsize for s in view.strides]


@pytest.fixture(scope="module")
def big():
    Xi = datagen.iota_i32((8192, 8192))
    Xf = datagen.uniform(datagen.SEEDS["gather_f32"], (8192, 8192), -1.0, 1.0)
    return Xi, Xf


@pytest.mark.parametrize("which", ["i32", "f32"])
def test_workload_8192(ctx, orc, big, which):
    """X[5::3, 1::2] -> [2729,4096] and X.T[::4, :] -> [2048,8192]."""
    X = big[0] if which == "i32" else big[1]
    t = dev(X)
    for view in (X[5::3, 1::2], X.T[::4, :]):
        off, shape, strides = numpy_view(X, view)
        g = gpu_gather(ctx, t, off, shape, strides)
        r = orc.gather(X, off, shape, strides)
        assert_bits_equal(g, r, f"{which} {shape}")
        if which == "i32":
            assert np.array_equal(g, np.ascontiguousarray(view))


CASES = [
    lambda X: X[::-1, 3:50:5],          # negative row stride
    lambda X: X[10:11, :],              # one row
    lambda X: X[:, ::-1],               # negative inner stride
    lambda X: X.T,                      # plain transpose
    lambda X: X[1:, 1:],                # unaligned row starts
    lambda X: X[:, 7],                  # a column
    lambda X: X.T[1::3, 2::5],          # strided transpose
    lambda X: X[::2, :],                # every other row (rows kernel)
]


@pytest.mark.parametrize("dtype", [np.int8, np.int16, np.float16, np.int32, np.float32])
@pytest.mark.parametrize("ci", range(len(CASES)))
def test_views_2d(ctx, orc, dtype, ci):
    X = (datagen.iota_i32((96, 200)) % 127).astype(dtype)
    view = CASES[ci](X)
    off, shape, strides = numpy_view(X, view)
    t = dev(X)
    g = gpu_gather(ctx, t, off, shape, strides)
    assert_bits_equal(g, orc.gather(X, off, shape, strides), str(ci))
    assert_bits_equal(g, np.ascontiguousarray(view), f"numpy {ci}")


def test_views_nd(ctx, orc):
    X = datagen.iota_i32((6, 40, 70))
    t = dev(X)
    for view in (X.transpose(2, 0, 1), X.transpose(1, 2, 0)[::3], X[:, ::2, 1::4], X.transpose(0, 2, 1),
                 X[::-1, :, ::-1]):
        off, shape, strides = numpy_view(X, view)
        g = gpu_gather(ctx, t, off, shape, strides)
        assert_bits_equal(g, np.ascontiguousarray(view), str(shape))


def test_broadcast_source(ctx):
    X = datagen.iota_i32((1, 64))
    t = dev(X)
    g = gpu_gather(ctx, t, 0, (32, 64), (0, 1))
    assert np.array_equal(g, np.broadcast_to(X, (32, 64)))


def test_contiguous_copy_and_errors(ctx):
    X = datagen.uniform(3, (1000,), -1, 1)
    t = dev(X)
    g = gpu_gather(ctx, t, 0, (1000,), (1,))
    assert np.array_equal(g, X)
    with pytest.raises(abi.QsmlError):
        ctx.gather(view_desc(t, 0, (10, 10), (10, 1)), d(empty((10, 11), np.float32)))
