"""CPU-side checks of the C ABI: the library loads without a GPU, exports
every function include/qsml_cuda.h declares, its constants agree with the
Python binding, and context-free calls fail cleanly (status + message, no
abort) when no device is present."""
import ctypes
import re

import pytest

from quasarml_b200 import abi


def test_library_exports_every_declared_symbol():
    lib = abi.load()
    names = abi.declared_functions()
    assert len(names) >= 25
    missing = [n for n in names if not hasattr(lib, n)]
    assert not missing, missing
    # the binding declares exactly the header's functions
    assert sorted(abi._SIGS) == names


def test_header_constants_match_binding():
    text = open(abi.HEADER_PATH).read()
    defs = dict((k, int(v)) for k, v in re.findall(r"#define\s+(QSML_\w+)\s+\(?(-?\d+)\)?", text))
    assert defs["QSML_MAX_DIMS"] == abi.MAX_DIMS
    for name in ("F32", "F16", "I32", "I16", "I8", "U32", "U16", "U8"):
        assert defs["QSML_" + name] == getattr(abi, name)
    for name in ("ADD", "SUB", "MUL", "DIV", "POW"):
        assert defs["QSML_OP_" + name] == getattr(abi, "OP_" + name)
    for name in ("RELU", "NEG", "ABS", "SQRT", "EXP", "LOG", "SIN", "COS", "TANH", "SIGMOID", "GELU"):
        assert defs["QSML_UN_" + name] == getattr(abi, "UN_" + name)
    for name in ("SUM", "MEAN", "MAX", "MIN", "PROD"):
        assert defs["QSML_RED_" + name] == getattr(abi, "RED_" + name)
    assert defs["QSML_AXIS_ALL"] == abi.AXIS_ALL
    for name in ("OK", "E_INVALID", "E_SHAPE", "E_DTYPE", "E_OOM", "E_CUDA", "E_NCCL", "E_TIMEOUT",
                 "E_UNSUPPORTED"):
        assert defs["QSML_" + name] == getattr(abi, name)
    # the descriptor layout is the header's
    assert ctypes.sizeof(abi.TDesc) == 8 + 4 + 4 + 8 * 8 * 2


def test_dtype_codes_follow_reference_enum():
    # QuasarML/src/Common/Types.h:80-89: F32, F16, I32, I16, I8, U32, U16, U8
    assert [abi.F32, abi.F16, abi.I32, abi.I16, abi.I8, abi.U32, abi.U16, abi.U8] == list(range(8))
    assert abi.DTYPE_SIZE == {0: 4, 1: 2, 2: 4, 3: 2, 4: 1, 5: 4, 6: 2, 7: 1}


def _has_gpu():
    try:
        import torch
        return torch.cuda.is_available()
    except Exception:
        return False


@pytest.mark.skipif(_has_gpu(), reason="checks the no-device error path")
def test_no_device_paths_return_status():
    lib = abi.load()
    n = ctypes.c_int32(-1)
    assert lib.qsml_device_count(ctypes.byref(n)) == abi.OK
    assert n.value == 0
    h = ctypes.c_void_p()
    st = lib.qsml_init(0, ctypes.byref(h))
    assert st == abi.E_INVALID
    assert h.value is None
    assert b"no CUDA device" in lib.qsml_last_error(None)
    # null context is rejected, not dereferenced
    assert lib.qsml_synchronize(None) == abi.E_INVALID
    assert lib.qsml_binary(None, 0, None, None, None) == abi.E_INVALID


def test_null_arguments_rejected():
    lib = abi.load()
    assert lib.qsml_device_count(None) == abi.E_INVALID
    assert lib.qsml_init(0, None) == abi.E_INVALID
    assert lib.qsml_host_alloc(16, None) == abi.E_INVALID


def test_shape_helpers():
    assert abi.broadcast_shape((4096, 4096), (1, 4096)) == (4096, 4096)
    assert abi.broadcast_shape((4096, 4096), (4096, 1)) == (4096, 4096)
    assert abi.broadcast_shape((3, 1, 5), (4, 1)) == (3, 4, 5)
    with pytest.raises(ValueError):
        abi.broadcast_shape((3,), (4,))
    # Ops/Reduction.cpp:297-305: axis dropped (or kept as 1); empty -> [1]
    assert abi.reduced_shape((64, 512, 1024), 0, False) == (512, 1024)
    assert abi.reduced_shape((64, 512, 1024), -1, True) == (64, 512, 1)
    assert abi.reduced_shape((10,), 0, False) == (1,)
    assert abi.reduced_shape((10,), None, False) == (1,)
