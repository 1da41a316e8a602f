"""Seeded synthetic inputs (binding of libqsml_datagen.so, csrc/datagen.c).

The generator is counter-based: element i of a stream depends only on
(seed, i), so shards and threads reproduce the global tensor exactly.
``uniform_np`` restates the uniform stream in NumPy for cross-checks.
"""
from __future__ import annotations

import ctypes
import os

import numpy as np

_HERE = os.path.dirname(os.path.abspath(__file__))
_LIB_PATH = os.path.join(_HERE, "libqsml_datagen.so")
_lib = None

# Seeds of the workloads (one per tensor).
SEEDS = {
    "ew_A": 1, "ew_B": 2, "ew_D": 3,
    "red_X": 4,
    "gather_f32": 5,
    "mm_A": 6, "mm_B": 7, "mm_Bb": 8, "mm_Ab": 9,
    "ln_X": 10, "ln_gamma": 11, "ln_beta": 12,
}


def _load():
    global _lib
    if _lib is None:
        if not os.path.exists(_LIB_PATH):
            raise OSError(f"{_LIB_PATH} missing: run `make -C quasarml_b200`")
        lib = ctypes.CDLL(_LIB_PATH)
        lib.qsml_gen_bits.restype = ctypes.c_uint64
        lib.qsml_gen_bits.argtypes = [ctypes.c_uint64, ctypes.c_uint64]
        for fn in (lib.qsml_gen_uniform_f32, lib.qsml_gen_normal_f32):
            fn.restype = None
            fn.argtypes = [ctypes.c_uint64, ctypes.c_int64, ctypes.c_int64, ctypes.c_double,
                           ctypes.c_double, ctypes.c_void_p]
        lib.qsml_gen_iota_i32.restype = None
        lib.qsml_gen_iota_i32.argtypes = [ctypes.c_int64, ctypes.c_int64, ctypes.c_void_p]
        _lib = lib
    return _lib


def _out(n, dtype, out):
    if out is None:
        return np.empty(n, dtype=dtype)
    assert out.dtype == dtype and out.flags.c_contiguous and out.size == n
    return out


def uniform(seed: int, shape, a: float, b: float, offset: int = 0, out=None) -> np.ndarray:
    n = int(np.prod(shape))
    o = _out(n, np.float32, None if out is None else out.reshape(-1))
    _load().qsml_gen_uniform_f32(seed, offset, n, a, b, o.ctypes.data)
    return o.reshape(shape)


def normal(seed: int, shape, mean: float, std: float, offset: int = 0, out=None) -> np.ndarray:
    n = int(np.prod(shape))
    o = _out(n, np.float32, None if out is None else out.reshape(-1))
    _load().qsml_gen_normal_f32(seed, offset, n, mean, std, o.ctypes.data)
    return o.reshape(shape)


def iota_i32(shape, offset: int = 0) -> np.ndarray:
    n = int(np.prod(shape))
    o = np.empty(n, dtype=np.int32)
    _load().qsml_gen_iota_i32(offset, n, o.ctypes.data)
    return o.reshape(shape)


def uniform_np(seed: int, n: int, a: float, b: float, offset: int = 0) -> np.ndarray:
    """NumPy restatement of the uniform stream (for cross-checking the C one)."""
    with np.errstate(over="ignore"):
        i = np.arange(offset, offset + n, dtype=np.uint64) + np.uint64(1)
        z = np.uint64(seed) * np.uint64(0xD1B54A32D192ED03) + i * np.uint64(0x9E3779B97F4A7C15)
        z ^= z >> np.uint64(30)
        z *= np.uint64(0xBF58476D1CE4E5B9)
        z ^= z >> np.uint64(27)
        z *= np.uint64(0x94D049BB133111EB)
        z ^= z >> np.uint64(31)
    u = (z >> np.uint64(40)).astype(np.float64) * 2.0 ** -24
    return (a + (b - a) * u).astype(np.float32)
