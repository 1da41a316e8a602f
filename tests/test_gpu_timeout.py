"""Failure detection on the device without a fault: the bounded waits.

The kernels that wait on mbarriers for data -- the one-SM tensor-core GEMM
and the layer-norm / softmax row pipelines (warp-per-row and CTA-per-row) --
give up a wait after the context's limit (qsml_set_wait_limit), let every copy
and MMA they already issued finish, record QSML_E_TIMEOUT and return.  Each
test lowers the limit to one cycle, so the first wait for a copy still in
flight runs out; qsml_synchronize must then report QSML_E_TIMEOUT once, and
with the default limit restored the next call on the same context must
succeed and match the oracle.  Nothing here faults, traps or hangs the GPU:
every wait stays bounded, and the waits that drain a kernel's own copies keep
the full limit.
"""
import numpy as np
import pytest

from helpers import d, dev, empty, host
from quasarml_b200 import abi, datagen

pytestmark = pytest.mark.gpu


@pytest.fixture
def fresh():
    """A context of its own, so a recorded timeout cannot reach another test."""
    import torch
    torch.cuda.set_device(0)
    c = abi.Context(0)
    yield c
    c.set_wait_limit(0)
    torch.cuda.synchronize()
    c.close()


def expect_timeout(c):
    with pytest.raises(abi.QsmlError) as e:
        c.synchronize()
    assert e.value.status == abi.E_TIMEOUT, e.value
    c.synchronize()  # reported once, then cleared


def test_gemm_wait_expires_then_recovers(fresh, orc, monkeypatch):
    monkeypatch.setenv("QSML_GEMM_2SM", "0")
    a = datagen.uniform(71, (512, 1024), -1, 1).astype(np.float16)
    b = datagen.uniform(72, (1024, 512), -1, 1).astype(np.float16)
    ta, tb = dev(a), dev(b)
    c = empty((512, 512), np.float32)
    fresh.set_wait_limit(1)
    fresh.matmul(d(ta), d(tb), d(c), abi.MM_FP16_F32ACC)
    assert fresh.last_kernel().startswith("k_gemm_tc<"), fresh.last_kernel()
    expect_timeout(fresh)
    fresh.set_wait_limit(0)
    fresh.matmul(d(ta), d(tb), d(c), abi.MM_FP16_F32ACC)
    fresh.synchronize()
    ref = orc.matmul_f64(a, b)
    err = np.max(np.abs(host(c).astype(np.float64) - ref)) / np.max(np.abs(ref))
    assert err <= 1e-5, err


@pytest.mark.parametrize("shape,dtype,kernel", [((4096, 2048), np.float16, "k_layer_norm_pipe"),
                                                ((64, 16384), np.float32, "k_layer_norm_wide")])
def test_layer_norm_wait_expires_then_recovers(fresh, orc, shape, dtype, kernel):
    x = datagen.normal(73, shape, 0.5, 2.0).astype(dtype)
    g = datagen.normal(74, shape[-1:], 1.0, 0.1)
    bb = datagen.normal(75, shape[-1:], 0.0, 0.1)
    tx, tg, tb = dev(x), dev(g), dev(bb)
    y = empty(shape, dtype)
    fresh.set_wait_limit(1)
    fresh.layer_norm(d(tx), d(tg), d(tb), 1e-5, d(y))
    assert fresh.last_kernel().startswith(kernel), fresh.last_kernel()
    expect_timeout(fresh)
    fresh.set_wait_limit(0)
    fresh.layer_norm(d(tx), d(tg), d(tb), 1e-5, d(y))
    fresh.synchronize()
    ref = orc.layer_norm(x, g, bb, 1e-5).astype(np.float64)
    bar = 1e-5 if dtype == np.float32 else 1e-3
    err = np.abs(host(y).astype(np.float64) - ref) / (bar * np.maximum(np.abs(ref), 0.1))
    assert np.max(err) <= 1.0


def test_softmax_wait_expires_then_recovers(fresh, orc):
    x = datagen.normal(76, (4096, 2048), 0.5, 2.0).astype(np.float16)
    tx = dev(x)
    y = empty(x.shape, np.float16)
    fresh.set_wait_limit(1)
    fresh.softmax(d(tx), -1, d(y))
    assert fresh.last_kernel().startswith("k_softmax_pipe"), fresh.last_kernel()
    expect_timeout(fresh)
    fresh.set_wait_limit(0)
    fresh.softmax(d(tx), -1, d(y))
    fresh.synchronize()
    ref = orc.softmax(x, -1).astype(np.float64)
    got = host(y).astype(np.float64)
    assert np.max(np.abs(got - ref) - 1e-3 * ref) <= 1e-7


def test_wait_limit_rejects_a_negative_value(fresh):
    with pytest.raises(abi.QsmlError) as e:
        fresh.set_wait_limit(-1)
    assert e.value.status == abi.E_INVALID
