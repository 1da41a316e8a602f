"""qsml_cast (through the C ABI): binary32 -> binary16 rounds to nearest even
and binary16 -> binary32 is exact, so both are bit-identical to NumPy's
astype; special values (NaN positions, +-inf, values beyond the binary16
range, subnormals, -0), ragged lengths and unaligned pointers (the scalar
path) included."""
import numpy as np
import pytest

from helpers import d, dev, empty, host
from quasarml_b200 import abi, datagen

pytestmark = pytest.mark.gpu


def specials():
    return np.array([0.0, -0.0, 1.0, -1.0, np.inf, -np.inf, np.nan, 65504.0, 65519.99, 65520.0, 70000.0, -70000.0,
                     6.1e-5, 5.96e-8, 2.98e-8, 2.99e-8, 1e-9, 1.0009765625, 1.00048828125, 1.00146484375],
                    np.float32)


def check_bits(got, want):
    gn, wn = np.isnan(got), np.isnan(want)
    assert np.array_equal(gn, wn)
    assert np.array_equal(got[~gn].view(np.uint16 if got.itemsize == 2 else np.uint32),
                          want[~wn].view(np.uint16 if want.itemsize == 2 else np.uint32))


@pytest.mark.parametrize("n", [1, 7, 8, 1000, 1 << 20, (1 << 20) + 5])
def test_f32_to_f16_and_back(ctx, n):
    x = datagen.normal(91, (n,), 0.0, 3000.0)
    x[: min(n, 20)] = specials()[: min(n, 20)]
    h = empty((n,), np.float16)
    ctx.cast(d(dev(x)), d(h))
    got = host(h)
    with np.errstate(over="ignore"):
        check_bits(got, x.astype(np.float16))
    back = empty((n,), np.float32)
    ctx.cast(d(h), d(back))
    check_bits(host(back), got.astype(np.float32))


def test_unaligned_and_same_dtype(ctx):
    x = datagen.uniform(92, (1001,), -2, 2)
    t = dev(x)
    view = abi.make_desc(t.data_ptr() + 4, abi.F32, (1000,), (1,))  # 4-byte offset: scalar path
    h = empty((1000,), np.float16)
    ctx.cast(view, d(h))
    check_bits(host(h), x[1:].astype(np.float16))
    c = empty((1001,), np.float32)
    ctx.cast(d(t), d(c))
    check_bits(host(c), x)


def test_errors(ctx):
    t = dev(np.ones((4, 4), np.float32))
    with pytest.raises(abi.QsmlError) as e:
        ctx.cast(d(t), d(empty((4, 5), np.float16)))
    assert e.value.status == abi.E_SHAPE
    with pytest.raises(abi.QsmlError) as e:
        ctx.cast(d(t.t()), d(empty((4, 4), np.float16)))
    assert e.value.status == abi.E_UNSUPPORTED
    with pytest.raises(abi.QsmlError) as e:
        ctx.cast(d(t), d(empty((4, 4), np.int32)))
    assert e.value.status == abi.E_DTYPE
