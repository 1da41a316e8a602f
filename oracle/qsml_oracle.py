"""NumPy-facing binding of the CPU oracle (oracle/libqsml_oracle.so).

TEST INFRASTRUCTURE ONLY: imported by the test suite, by the smoke check and
by the benchmark's CPU-baseline leg, never by the product path.  Each
function restates the reference arithmetic cited in qsml_oracle.c.
"""
from __future__ import annotations

import ctypes
import os
import subprocess

import numpy as np

_HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(_HERE, "libqsml_oracle.so")

ADD, SUB, MUL, DIV, POW = range(5)
SUM, MEAN, MAX, MIN, PROD = range(5)

_lib = None
_P = ctypes.c_void_p
_I64 = ctypes.c_int64


def build() -> None:
    subprocess.run(["make", "-s", "-C", _HERE], check=True)


def _load():
    global _lib
    if _lib is not None:
        return _lib
    if not os.path.exists(LIB_PATH):
        build()
    lib = ctypes.CDLL(LIB_PATH)
    sig = {
        "orc_half_to_float": (ctypes.c_float, [ctypes.c_uint16]),
        "orc_float_to_half": (ctypes.c_uint16, [ctypes.c_float]),
        "orc_half_to_float_n": (None, [_P, _P, _I64]),
        "orc_float_to_half_n": (None, [_P, _P, _I64]),
        "orc_broadcast_shape": (ctypes.c_int, [_P, ctypes.c_int, _P, ctypes.c_int, _P, _P]),
        "orc_binary_f32": (ctypes.c_int, [ctypes.c_int, _P, _P, ctypes.c_int, _P, _P, ctypes.c_int, _P]),
        "orc_binary_f16": (ctypes.c_int, [ctypes.c_int, _P, _P, ctypes.c_int, _P, _P, ctypes.c_int, _P]),
        "orc_binary_i32": (ctypes.c_int, [ctypes.c_int, _P, _P, ctypes.c_int, _P, _P, ctypes.c_int, _P]),
        "orc_binary_scalar_f32": (None, [ctypes.c_int, _P, _I64, ctypes.c_float, _P]),
        "orc_pow_f32": (ctypes.c_float, [ctypes.c_float, ctypes.c_float]),
        "orc_relu_f32": (ctypes.c_float, [ctypes.c_float]),
        "orc_max_f32": (ctypes.c_float, [ctypes.c_float, ctypes.c_float]),
        "orc_min_f32": (ctypes.c_float, [ctypes.c_float, ctypes.c_float]),
        "orc_relu_f32_n": (None, [_P, _I64, _P]),
        "orc_relu_f16_n": (None, [_P, _I64, _P]),
        "orc_unary_f32": (ctypes.c_int, [ctypes.c_int, _P, _I64, _P]),
        "orc_reduce_f32": (None, [ctypes.c_int, _P, _I64, _I64, _I64, _P, _P, _P]),
        "orc_reduce_f16": (None, [ctypes.c_int, _P, _I64, _I64, _I64, _P, _P, _P]),
        "orc_argreduce": (None, [ctypes.c_int, ctypes.c_int, _P, _I64, _I64, _I64, _P]),
        "orc_softmax": (None, [_P, ctypes.c_int, _I64, _I64, _I64, _P]),
        "orc_gather": (None, [_P, ctypes.c_int, ctypes.c_int, _P, _P, _P]),
        "orc_layer_norm_f32": (None, [_P, _P, _P, _I64, _I64, ctypes.c_float, _P]),
        "orc_layer_norm_f16": (None, [_P, _P, _P, _I64, _I64, ctypes.c_float, _P]),
        "orc_matmul_f32_fma": (None, [_P, _P, _P, _I64, _I64, _I64, _I64, _I64, _I64, _I64]),
        "orc_matmul_f64": (None, [_P, _P, _P, _I64, _I64, _I64, _I64, _I64, _I64, _I64]),
        "orc_matmul_f16in_f64": (None, [_P, _P, _P, _I64, _I64, _I64, _I64, _I64, _I64, _I64]),
        "orc_num_threads": (ctypes.c_int, []),
        "orc_set_num_threads": (None, [ctypes.c_int]),
        "orc_reduce_f32_par": (None, [ctypes.c_int, _P, _I64, _I64, _I64, _P]),
        "orc_reduce_f16_par": (None, [ctypes.c_int, _P, _I64, _I64, _I64, _P]),
    }
    for name, (res, args) in sig.items():
        fn = getattr(lib, name)
        fn.restype = res
        fn.argtypes = args
    _lib = lib
    return lib


def lib():
    return _load()


def _ptr(a: np.ndarray):
    return a.ctypes.data


def _shape_arr(shape):
    return np.ascontiguousarray(np.asarray(shape, dtype=np.int64).reshape(-1))


def broadcast_shape(a_shape, b_shape):
    L = _load()
    a, b = _shape_arr(a_shape), _shape_arr(b_shape)
    out = np.zeros(16, dtype=np.int64)
    nout = ctypes.c_int()
    if L.orc_broadcast_shape(_ptr(a), len(a), _ptr(b), len(b), _ptr(out), ctypes.addressof(nout)) != 0:
        raise ValueError("shapes do not broadcast")
    return tuple(int(x) for x in out[: nout.value])


def binary(op: int, a: np.ndarray, b: np.ndarray) -> np.ndarray:
    """Broadcast binary op; dtype float32 / float16 / int32."""
    L = _load()
    a = np.ascontiguousarray(a)
    b = np.ascontiguousarray(b)
    assert a.dtype == b.dtype
    shape = broadcast_shape(a.shape, b.shape)
    out = np.empty(shape, dtype=a.dtype)
    sa, sb = _shape_arr(a.shape), _shape_arr(b.shape)
    fn = {np.dtype(np.float32): L.orc_binary_f32, np.dtype(np.float16): L.orc_binary_f16,
          np.dtype(np.int32): L.orc_binary_i32}[a.dtype]
    rc = fn(op, _ptr(a), _ptr(sa), a.ndim, _ptr(b), _ptr(sb), b.ndim, _ptr(out))
    if rc != 0:
        raise ValueError("shape error")
    return out


def binary_scalar(op: int, x: np.ndarray, s: float) -> np.ndarray:
    x = np.ascontiguousarray(x, dtype=np.float32)
    out = np.empty_like(x)
    _load().orc_binary_scalar_f32(op, _ptr(x), x.size, s, _ptr(out))
    return out


def relu(x: np.ndarray) -> np.ndarray:
    x = np.ascontiguousarray(x)
    out = np.empty_like(x)
    if x.dtype == np.float32:
        _load().orc_relu_f32_n(_ptr(x), x.size, _ptr(out))
    elif x.dtype == np.float16:
        _load().orc_relu_f16_n(_ptr(x), x.size, _ptr(out))
    else:
        raise TypeError(x.dtype)
    return out


UN_RELU, UN_NEG, UN_ABS, UN_SQRT, UN_EXP, UN_LOG, UN_SIN, UN_COS, UN_TANH, UN_SIGMOID, UN_GELU = range(11)


def unary(op: int, x: np.ndarray) -> np.ndarray:
    x = np.ascontiguousarray(x, dtype=np.float32)
    out = np.empty_like(x)
    if _load().orc_unary_f32(op, _ptr(x), x.size, _ptr(out)) != 0:
        raise ValueError("unknown unary op")
    return out


def pow_scalar(x: np.ndarray, y: float) -> np.ndarray:
    return binary_scalar(POW, x, y)


def reduce(op: int, x: np.ndarray, axis=None):
    """Returns (out32, out64, absum) shaped like the reduced output (no
    keepdims).  axis None = all elements."""
    L = _load()
    x = np.ascontiguousarray(x)
    if axis is None:
        outer, k, inner, oshape = 1, x.size, 1, ()
    else:
        ax = axis + x.ndim if axis < 0 else axis
        outer = int(np.prod(x.shape[:ax], dtype=np.int64))
        k = x.shape[ax]
        inner = int(np.prod(x.shape[ax + 1:], dtype=np.int64))
        oshape = tuple(d for i, d in enumerate(x.shape) if i != ax)
    n = outer * inner
    o32 = np.empty(n, dtype=np.float32)
    o64 = np.empty(n, dtype=np.float64)
    ab = np.empty(n, dtype=np.float64)
    fn = L.orc_reduce_f32 if x.dtype == np.float32 else L.orc_reduce_f16
    fn(op, _ptr(x), outer, k, inner, _ptr(o32), _ptr(o64), _ptr(ab))
    return o32.reshape(oshape), o64.reshape(oshape), ab.reshape(oshape)


ARGMAX, ARGMIN = 0, 1
_QSML_DTYPE = {np.dtype(np.float32): 0, np.dtype(np.float16): 1, np.dtype(np.int32): 2, np.dtype(np.int16): 3,
               np.dtype(np.int8): 4, np.dtype(np.uint32): 5, np.dtype(np.uint16): 6, np.dtype(np.uint8): 7}


def argreduce(op: int, x: np.ndarray, axis=None) -> np.ndarray:
    """Index (int64) of the first max (op ARGMAX) or min (ARGMIN) over `axis`
    (None = the flattened array); NaN beats every number."""
    L = _load()
    x = np.ascontiguousarray(x)
    if axis is None:
        outer, k, inner, oshape = 1, x.size, 1, ()
    else:
        ax = axis + x.ndim if axis < 0 else axis
        outer = int(np.prod(x.shape[:ax], dtype=np.int64))
        k = x.shape[ax]
        inner = int(np.prod(x.shape[ax + 1:], dtype=np.int64))
        oshape = tuple(d for i, d in enumerate(x.shape) if i != ax)
    if k == 0:
        raise ValueError("argreduce of an empty axis")
    out = np.empty(outer * inner, dtype=np.int64)
    L.orc_argreduce(op, _QSML_DTYPE[x.dtype], _ptr(x), outer, k, inner, _ptr(out))
    return out.reshape(oshape)


def softmax(x: np.ndarray, axis: int = -1) -> np.ndarray:
    """binary64 softmax over `axis` of a float32 / float16 array."""
    x = np.ascontiguousarray(x)
    ax = axis + x.ndim if axis < 0 else axis
    outer = int(np.prod(x.shape[:ax], dtype=np.int64))
    k = x.shape[ax]
    inner = int(np.prod(x.shape[ax + 1:], dtype=np.int64))
    out = np.empty(x.shape, dtype=np.float64)
    _load().orc_softmax(_ptr(x), 1 if x.dtype == np.float16 else 0, outer, k, inner, _ptr(out))
    return out


def gather(base: np.ndarray, offset: int, shape, strides) -> np.ndarray:
    """Materialises the view of `base` (flat, contiguous) starting at element
    `offset` with element strides."""
    base = np.ascontiguousarray(base).reshape(-1)
    out = np.empty(tuple(shape), dtype=base.dtype)
    if out.size == 0:
        return out
    sh, st = _shape_arr(shape), _shape_arr(strides)
    ptr = base.ctypes.data + offset * base.itemsize
    _load().orc_gather(ctypes.c_void_p(ptr), base.itemsize, len(sh), _ptr(sh), _ptr(st), _ptr(out))
    return out


def layer_norm(x: np.ndarray, gamma: np.ndarray, beta: np.ndarray, eps: float) -> np.ndarray:
    x = np.ascontiguousarray(x)
    g = np.ascontiguousarray(gamma, dtype=np.float32)
    b = np.ascontiguousarray(beta, dtype=np.float32)
    cols = x.shape[-1]
    rows = x.size // cols
    out = np.empty_like(x)
    fn = _load().orc_layer_norm_f32 if x.dtype == np.float32 else _load().orc_layer_norm_f16
    fn(_ptr(x), _ptr(g), _ptr(b), rows, cols, eps, _ptr(out))
    return out


def _mm_dims(a, b):
    if a.ndim == 2:
        return 1, a.shape[0], a.shape[1], b.shape[1], 0, 0
    return a.shape[0], a.shape[1], a.shape[2], b.shape[2], a.shape[1] * a.shape[2], b.shape[1] * b.shape[2]


def matmul_fma(a: np.ndarray, b: np.ndarray) -> np.ndarray:
    a = np.ascontiguousarray(a, dtype=np.float32)
    b = np.ascontiguousarray(b, dtype=np.float32)
    bt, M, K, N, sA, sB = _mm_dims(a, b)
    out = np.empty(((bt,) if a.ndim == 3 else ()) + (M, N), dtype=np.float32)
    _load().orc_matmul_f32_fma(_ptr(a), _ptr(b), _ptr(out), bt, M, K, N, sA, sB, M * N)
    return out


def matmul_f64(a: np.ndarray, b: np.ndarray) -> np.ndarray:
    bt, M, K, N, sA, sB = _mm_dims(a, b)
    out = np.empty(((bt,) if a.ndim == 3 else ()) + (M, N), dtype=np.float64)
    if a.dtype == np.float16:
        a = np.ascontiguousarray(a)
        b = np.ascontiguousarray(b)
        _load().orc_matmul_f16in_f64(_ptr(a), _ptr(b), _ptr(out), bt, M, K, N, sA, sB, M * N)
    else:
        a = np.ascontiguousarray(a, dtype=np.float32)
        b = np.ascontiguousarray(b, dtype=np.float32)
        _load().orc_matmul_f64(_ptr(a), _ptr(b), _ptr(out), bt, M, K, N, sA, sB, M * N)
    return out


def ulp_diff_f32(x: np.ndarray, y: np.ndarray) -> np.ndarray:
    """Distance in binary32 units in the last place (NaN pairs count 0)."""
    xi = np.ascontiguousarray(x, dtype=np.float32).view(np.int32).astype(np.int64)
    yi = np.ascontiguousarray(y, dtype=np.float32).view(np.int32).astype(np.int64)
    xi = np.where(xi < 0, -(xi & 0x7FFFFFFF), xi)
    yi = np.where(yi < 0, -(yi & 0x7FFFFFFF), yi)
    d = np.abs(xi - yi)
    both_nan = np.isnan(x) & np.isnan(y)
    return np.where(both_nan, 0, d)


def matmul_check(c: np.ndarray, a: np.ndarray, b: np.ndarray, rows_per_block: int = 1024):
    """Every output of a product c = a @ b (rank 2, or rank 3 batched) against
    binary64, for the floating-point matmul bars (LinAlg.cpp:84-158 computes
    each output as one dot product over k).  The binary64 product and the
    componentwise error scale |a| @ |b| (the factor in the classical bound
    |fl(a.b) - a.b| <= gamma_k |a|.|b| of any summation order) come from
    NumPy's binary64 matmul, a block of rows at a time.  a and b are the
    inputs as the kernel saw them (binary16 inputs widen exactly).

    Returns (worst componentwise error / scale, normwise error
    ||c - ref||_F / ||ref||_F, max|err| / max|ref|)."""
    a3 = a[None] if a.ndim == 2 else a
    b3 = b[None] if b.ndim == 2 else b
    c3 = c[None] if c.ndim == 2 else c
    worst = 0.0
    err2 = 0.0
    ref2 = 0.0
    maxerr = 0.0
    maxref = 0.0
    for bi in range(a3.shape[0]):
        B = b3[bi].astype(np.float64)
        Babs = np.abs(B)
        for r0 in range(0, a3.shape[1], rows_per_block):
            A = a3[bi, r0:r0 + rows_per_block].astype(np.float64)
            ref = A @ B
            scale = np.abs(A) @ Babs
            err = np.abs(c3[bi, r0:r0 + rows_per_block].astype(np.float64) - ref)
            with np.errstate(divide="ignore", invalid="ignore"):
                q = np.where(scale > 0, err / scale, np.where(err > 0, np.inf, 0.0))
            worst = max(worst, float(q.max()))
            err2 += float(np.sum(err * err))
            ref2 += float(np.sum(ref * ref))
            maxerr = max(maxerr, float(err.max()))
            maxref = max(maxref, float(np.abs(ref).max()))
    return worst, (err2 ** 0.5) / (ref2 ** 0.5 if ref2 > 0 else 1.0), maxerr / (maxref if maxref > 0 else 1.0)
