"""GPU runtime: caching allocator, copies, streams, counters, error model and
host-side fault injection (QSML_FAULT_ALLOC_N makes a driver allocation
report out-of-memory; nothing faults on the device)."""
import ctypes
import os
import subprocess
import sys

import numpy as np
import pytest

from quasarml_b200 import abi

pytestmark = pytest.mark.gpu

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def test_device_query():
    lib = abi.load()
    n = ctypes.c_int32()
    assert lib.qsml_device_count(ctypes.byref(n)) == abi.OK and n.value >= 1
    buf = ctypes.create_string_buffer(256)
    assert lib.qsml_device_name(0, buf, 256) == abi.OK
    assert b"B200" in buf.value or len(buf.value) > 0


def test_allocator_reuses_blocks(ctx):
    s0 = ctx.allocator_stats()
    p = ctx.alloc(3 << 20)
    assert p % 256 == 0
    ctx.free(p)
    q = ctx.alloc(3 << 20)
    assert q == p
    s1 = ctx.allocator_stats()
    assert s1["hits"] >= s0["hits"] + 1
    ctx.free(q)
    small = [ctx.alloc(1000) for _ in range(8)]
    for x in small:
        ctx.free(x)
    assert ctx.allocator_stats()["live_bytes"] == s0["live_bytes"]
    with pytest.raises(abi.QsmlError) as e:
        ctx.free(0x1234)
    assert e.value.status == abi.E_INVALID


def test_pinned_roundtrip_and_fill(ctx):
    lib = abi.load()
    n = 1 << 20
    hp = ctypes.c_void_p()
    assert lib.qsml_host_alloc(n * 4, ctypes.byref(hp)) == abi.OK
    host = np.frombuffer((ctypes.c_float * n).from_address(hp.value), dtype=np.float32)
    host[:] = np.arange(n, dtype=np.float32)
    dptr = ctx.alloc(n * 4)
    ctx.h2d(dptr, hp.value, n * 4)
    back = np.zeros(n, np.float32)
    ctx.d2h(back.ctypes.data, dptr, n * 4)
    assert np.array_equal(back, host)
    ctx.fill(dptr, np.float32(-2.0).tobytes(), n)
    ctx.d2h(back.ctypes.data, dptr, n * 4)
    assert np.all(back == -2.0)
    ctx.free(dptr)
    assert lib.qsml_host_free(hp) == abi.OK


def test_ops_on_library_allocations(ctx):
    """The ABI works on its own allocations (no torch memory involved)."""
    n = 4096
    a = np.arange(n, dtype=np.float32)
    pa, pb = ctx.alloc(n * 4), ctx.alloc(n * 4)
    ctx.h2d(pa, a.ctypes.data, n * 4)
    ctx.synchronize()
    da = abi.make_desc(pa, abi.F32, (n,))
    db = abi.make_desc(pb, abi.F32, (n,))
    ctx.binary(abi.OP_ADD, da, da, db)
    out = np.zeros(n, np.float32)
    ctx.d2h(out.ctypes.data, pb, n * 4)
    assert np.array_equal(out, a + a)
    ctx.free(pa)
    ctx.free(pb)


def test_counters(ctx):
    before = ctx.launch_count()
    n = 1024
    p = ctx.alloc(n * 4)
    dsc = abi.make_desc(p, abi.F32, (n,))
    ctx.unary(abi.UN_RELU, dsc, dsc)
    ctx.synchronize()
    assert ctx.launch_count() == before + 1
    assert ctx.cpu_fallback_count() == 0
    ctx.free(p)


def test_stream_switch(ctx):
    import torch
    s = torch.cuda.Stream()
    old = ctx.stream()
    ctx.set_stream(s.cuda_stream)
    assert ctx.stream() == s.cuda_stream
    ctx.set_stream(old)
    assert ctx.stream() == old


def test_fault_injection_alloc_reports_oom():
    code = (
        "import sys; sys.path.insert(0, %r)\n"
        "from quasarml_b200 import abi\n"
        "c = abi.Context(0, use_torch_stream=False)\n"
        "try:\n"
        "    c.alloc(1 << 20)\n"
        "    print('NO-ERROR')\n"
        "except abi.QsmlError as e:\n"
        "    print('STATUS', e.status, str(e))\n"
        "p = c.alloc(1 << 20)\n"
        "c.free(p)\n"
        "print('RECOVERED')\n" % ROOT
    )
    env = dict(os.environ, QSML_FAULT_ALLOC_N="1")
    r = subprocess.run([sys.executable, "-c", code], env=env, capture_output=True, text=True, timeout=300)
    assert r.returncode == 0, r.stderr
    assert f"STATUS {abi.E_OOM}" in r.stdout and "RECOVERED" in r.stdout, r.stdout


@pytest.mark.gpu
@pytest.mark.parametrize("nbytes", [(8 << 20) - 16, 8 << 20, (40 << 20) + 12, 67 << 20])
def test_staged_pageable_copies_round_trip(ctx, nbytes):
    """Pageable host buffers of 8 MiB and more go through pinned staging in
    chunks (including a ragged last chunk); both directions are exact, and an
    upload may be followed at once by reuse of the host buffer."""
    import torch
    rng = np.random.default_rng(nbytes)
    src = rng.integers(0, 256, nbytes, dtype=np.uint8)
    dev_buf = torch.empty(nbytes, dtype=torch.uint8, device="cuda")
    ctx.h2d(dev_buf.data_ptr(), src.ctypes.data, nbytes)
    expect = src.copy()
    src[:] = 0  # the call returned: the source may be overwritten
    back = np.empty(nbytes, dtype=np.uint8)
    ctx.d2h(back.ctypes.data, dev_buf.data_ptr(), nbytes)
    assert np.array_equal(back, expect)
    # offset (unaligned) device destination and host source
    ctx.h2d(dev_buf.data_ptr() + 3, expect.ctypes.data + 5, nbytes - 8)
    part = np.empty(nbytes - 8, dtype=np.uint8)
    ctx.d2h(part.ctypes.data, dev_buf.data_ptr() + 3, nbytes - 8)
    assert np.array_equal(part, expect[5:nbytes - 3])
