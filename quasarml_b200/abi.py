"""ctypes binding of libqsml_cuda.so, the extern "C" ABI of include/qsml_cuda.h.

This is how Python code (the test suite and bench.py) reaches the CUDA
backend: every call goes through the same C entry points the C++ QuasarML
layer uses.  Device buffers may come from the library's own caching
allocator (``Context.alloc``) or from torch tensors (``desc_of``); torch is
only plumbing for memory, streams and events.

There is no fallback: if the shared library is missing the import of this
module raises.
"""
from __future__ import annotations

import ctypes
import os
from typing import Iterable, Optional, Sequence

_HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(_HERE, "libqsml_cuda.so")
HEADER_PATH = os.path.join(os.path.dirname(_HERE), "include", "qsml_cuda.h")

# ---- constants (mirror include/qsml_cuda.h; tests check they agree) -------
OK, E_INVALID, E_SHAPE, E_DTYPE, E_OOM, E_CUDA, E_NCCL, E_TIMEOUT, E_UNSUPPORTED = range(9)
F32, F16, I32, I16, I8, U32, U16, U8 = range(8)
MAX_DIMS = 8
OP_ADD, OP_SUB, OP_MUL, OP_DIV, OP_POW = range(5)
(UN_RELU, UN_NEG, UN_ABS, UN_SQRT, UN_EXP, UN_LOG, UN_SIN, UN_COS, UN_TANH,
 UN_SIGMOID, UN_GELU) = range(11)
RED_SUM, RED_MEAN, RED_MAX, RED_MIN, RED_PROD = range(5)
AXIS_ALL = -1000
ARG_MAX, ARG_MIN = 0, 1
MM_AUTO, MM_FP32_FFMA, MM_FP32_3XTF32, MM_FP16_F32ACC = range(4)

DTYPE_SIZE = {F32: 4, F16: 2, I32: 4, I16: 2, I8: 1, U32: 4, U16: 2, U8: 1}
STATUS_NAME = {OK: "OK", E_INVALID: "E_INVALID", E_SHAPE: "E_SHAPE", E_DTYPE: "E_DTYPE",
               E_OOM: "E_OOM", E_CUDA: "E_CUDA", E_NCCL: "E_NCCL", E_TIMEOUT: "E_TIMEOUT",
               E_UNSUPPORTED: "E_UNSUPPORTED"}


class TDesc(ctypes.Structure):
    _fields_ = [
        ("data", ctypes.c_void_p),
        ("dtype", ctypes.c_int32),
        ("ndim", ctypes.c_int32),
        ("shape", ctypes.c_int64 * MAX_DIMS),
        ("stride", ctypes.c_int64 * MAX_DIMS),
    ]


FUSE_INPUT, FUSE_CONST, FUSE_BINARY, FUSE_UNARY = range(4)
FUSE_MODE_AUTO, FUSE_MODE_INTERP, FUSE_MODE_JIT = range(3)
FUSE_MAX_NODES, FUSE_MAX_INPUTS = 64, 6


class FuseNode(ctypes.Structure):
    """One node of a qsml_elementwise_fused expression."""
    _fields_ = [
        ("kind", ctypes.c_int32),
        ("code", ctypes.c_int32),
        ("a", ctypes.c_int32),
        ("b", ctypes.c_int32),
        ("value", ctypes.c_float),
    ]


class Expr:
    """Builds a qsml_elementwise_fused node list:

        e = Expr(); A, B = e.input(0), e.input(1)
        root = e.unary(UN_RELU, e.binary(OP_ADD, A, e.const(2.0)))
        ctx.elementwise_fused(e.nodes, [dA, dB], dOut)   # root = last node
    """

    def __init__(self):
        self.nodes = []

    def _add(self, kind, code=0, a=0, b=0, value=0.0) -> int:
        self.nodes.append((kind, code, a, b, value))
        return len(self.nodes) - 1

    def input(self, j: int) -> int:
        return self._add(FUSE_INPUT, j)

    def const(self, v: float) -> int:
        return self._add(FUSE_CONST, value=float(v))

    def binary(self, op: int, a: int, b: int) -> int:
        return self._add(FUSE_BINARY, op, a, b)

    def unary(self, op: int, a: int) -> int:
        return self._add(FUSE_UNARY, op, a)


class QsmlError(RuntimeError):
    def __init__(self, status: int, message: str):
        super().__init__(f"{STATUS_NAME.get(status, status)}: {message}")
        self.status = status


_P = ctypes.POINTER
_c = ctypes
# name -> (restype, argtypes)
_SIGS = {
    "qsml_device_count": (_c.c_int32, [_P(_c.c_int32)]),
    "qsml_device_name": (_c.c_int32, [_c.c_int32, _c.c_char_p, _c.c_size_t]),
    "qsml_init": (_c.c_int32, [_c.c_int32, _P(_c.c_void_p)]),
    "qsml_destroy": (_c.c_int32, [_c.c_void_p]),
    "qsml_set_stream": (_c.c_int32, [_c.c_void_p, _c.c_void_p]),
    "qsml_get_stream": (_c.c_int32, [_c.c_void_p, _P(_c.c_void_p)]),
    "qsml_synchronize": (_c.c_int32, [_c.c_void_p]),
    "qsml_set_wait_limit": (_c.c_int32, [_c.c_void_p, _c.c_int64]),
    "qsml_set_overlap": (_c.c_int32, [_c.c_void_p, _c.c_int32]),
    "qsml_overlap_stats": (_c.c_int32, [_c.c_void_p, _c.POINTER(_c.c_uint64), _c.POINTER(_c.c_uint64)]),
    "qsml_last_error": (_c.c_char_p, [_c.c_void_p]),
    "qsml_alloc": (_c.c_int32, [_c.c_void_p, _c.c_size_t, _P(_c.c_void_p)]),
    "qsml_free": (_c.c_int32, [_c.c_void_p, _c.c_void_p]),
    "qsml_empty_cache": (_c.c_int32, [_c.c_void_p]),
    "qsml_h2d": (_c.c_int32, [_c.c_void_p, _c.c_void_p, _c.c_void_p, _c.c_size_t]),
    "qsml_d2h": (_c.c_int32, [_c.c_void_p, _c.c_void_p, _c.c_void_p, _c.c_size_t]),
    "qsml_d2h_async": (_c.c_int32, [_c.c_void_p, _c.c_void_p, _c.c_void_p, _c.c_size_t]),
    "qsml_d2d": (_c.c_int32, [_c.c_void_p, _c.c_void_p, _c.c_void_p, _c.c_size_t]),
    "qsml_host_alloc": (_c.c_int32, [_c.c_size_t, _P(_c.c_void_p)]),
    "qsml_host_free": (_c.c_int32, [_c.c_void_p]),
    "qsml_fill": (_c.c_int32, [_c.c_void_p, _c.c_void_p, _c.c_void_p, _c.c_int32, _c.c_int64]),
    "qsml_binary": (_c.c_int32, [_c.c_void_p, _c.c_int32, _P(TDesc), _P(TDesc), _P(TDesc)]),
    "qsml_binary_scalar": (_c.c_int32, [_c.c_void_p, _c.c_int32, _P(TDesc), _c.c_float, _P(TDesc)]),
    "qsml_unary": (_c.c_int32, [_c.c_void_p, _c.c_int32, _P(TDesc), _P(TDesc)]),
    "qsml_reduce": (_c.c_int32, [_c.c_void_p, _c.c_int32, _P(TDesc), _c.c_int32, _c.c_int32, _P(TDesc)]),
    "qsml_arg_reduce": (_c.c_int32, [_c.c_void_p, _c.c_int32, _P(TDesc), _c.c_int32, _c.c_int32, _P(TDesc)]),
    "qsml_elementwise_fused": (_c.c_int32, [_c.c_void_p, _P(FuseNode), _c.c_int32, _P(TDesc), _c.c_int32,
                                            _P(TDesc)]),
    "qsml_set_fuse_mode": (_c.c_int32, [_c.c_void_p, _c.c_int32]),
    "qsml_fuse_stats": (_c.c_int32, [_c.c_void_p, _P(_c.c_uint64), _P(_c.c_uint64), _P(_c.c_uint64)]),
    "qsml_group_unique_id": (_c.c_int32, [_c.c_void_p]),
    "qsml_group_init_rank": (_c.c_int32, [_c.c_void_p, _c.c_void_p, _c.c_int32, _c.c_int32, _P(_c.c_void_p)]),
    "qsml_group_init_all": (_c.c_int32, [_P(_c.c_void_p), _c.c_int32, _P(_c.c_void_p)]),
    "qsml_group_size": (_c.c_int32, [_c.c_void_p, _P(_c.c_int32), _P(_c.c_int32)]),
    "qsml_group_start": (_c.c_int32, []),
    "qsml_group_end": (_c.c_int32, []),
    "qsml_allreduce": (_c.c_int32, [_c.c_void_p, _c.c_int32, _c.c_void_p, _c.c_int64, _c.c_int32, _c.c_int32]),
    "qsml_group_destroy": (_c.c_int32, [_c.c_void_p]),
    "qsml_gather": (_c.c_int32, [_c.c_void_p, _P(TDesc), _P(TDesc)]),
    "qsml_cast": (_c.c_int32, [_c.c_void_p, _P(TDesc), _P(TDesc)]),
    "qsml_softmax": (_c.c_int32, [_c.c_void_p, _P(TDesc), _c.c_int32, _P(TDesc)]),
    "qsml_layer_norm": (_c.c_int32, [_c.c_void_p, _P(TDesc), _P(TDesc), _P(TDesc), _c.c_float, _P(TDesc)]),
    "qsml_matmul": (_c.c_int32, [_c.c_void_p, _P(TDesc), _P(TDesc), _P(TDesc), _c.c_int32]),
    "qsml_reduce_noalloc": (_c.c_int32, [_c.c_void_p, _c.c_int32, _P(TDesc), _c.c_int32, _c.c_int32, _P(TDesc)]),
    "qsml_allreduce_partials": (_c.c_int32, [_c.c_void_p, _c.c_int32, _c.c_int32, _c.c_void_p, _c.c_int64]),
    "qsml_finish_partial": (_c.c_int32, [_c.c_void_p, _c.c_int32, _P(TDesc), _c.c_int64, _P(TDesc)]),
    "qsml_reduce_sharded": (_c.c_int32, [_c.c_void_p, _c.c_int32, _c.c_int32, _P(TDesc), _c.c_int32, _c.c_int32,
                                         _P(TDesc), _c.c_int64]),
    "qsml_shard_rows": (_c.c_int32, [_c.c_int64, _c.c_int32, _c.c_int32, _P(_c.c_int64), _P(_c.c_int64)]),
    "qsml_launch_count": (_c.c_int32, [_c.c_void_p, _P(_c.c_uint64)]),
    "qsml_last_kernel": (_c.c_int32, [_c.c_void_p, _c.c_char_p, _c.c_size_t]),
    "qsml_cpu_fallback_count": (_c.c_int32, [_c.c_void_p, _P(_c.c_uint64)]),
    "qsml_allocator_stats": (_c.c_int32, [_c.c_void_p, _P(_c.c_uint64), _P(_c.c_uint64),
                                          _P(_c.c_uint64), _P(_c.c_uint64)]),
}

_lib = None


def load() -> ctypes.CDLL:
    """Loads libqsml_cuda.so once; raises if it has not been built."""
    global _lib
    if _lib is not None:
        return _lib
    if not os.path.exists(LIB_PATH):
        raise OSError(f"{LIB_PATH} is missing: build it with `make -C quasarml_b200` "
                      "(or __graft_entry__.build()); there is no CPU fallback")
    lib = ctypes.CDLL(LIB_PATH)
    for name, (res, args) in _SIGS.items():
        fn = getattr(lib, name)
        fn.restype = res
        fn.argtypes = args
    _lib = lib
    return lib


UNIQUE_ID_BYTES = 128


def _check_global(st: int) -> None:
    if st != OK:
        raise QsmlError(st, load().qsml_last_error(None).decode())


def group_unique_id() -> bytes:
    """A new NCCL unique id (one rank makes it, every rank of the group uses it)."""
    buf = (ctypes.c_uint8 * UNIQUE_ID_BYTES)()
    _check_global(load().qsml_group_unique_id(buf))
    return bytes(buf)


class Group:
    """A qsml_group: init_rank(ctx, uid, nranks, rank) for one process per
    GPU, or init_all([ctx, ...]) for one process driving several GPUs."""

    def __init__(self, handle, ctxs):
        self.h, self.ctxs = handle, list(ctxs)

    @classmethod
    def init_rank(cls, ctx, uid: bytes, nranks: int, rank: int) -> "Group":
        h = ctypes.c_void_p()
        buf = (ctypes.c_uint8 * UNIQUE_ID_BYTES).from_buffer_copy(uid)
        ctx.check(ctx.lib.qsml_group_init_rank(ctx.h, buf, int(nranks), int(rank), ctypes.byref(h)))
        return cls(h, [ctx])

    @classmethod
    def init_all(cls, ctxs) -> "Group":
        h = ctypes.c_void_p()
        arr = (ctypes.c_void_p * len(ctxs))(*[c.h.value for c in ctxs])
        _check_global(load().qsml_group_init_all(arr, len(ctxs), ctypes.byref(h)))
        return cls(h, ctxs)

    def size(self) -> tuple:
        n, loc = ctypes.c_int32(), ctypes.c_int32()
        _check_global(load().qsml_group_size(self.h, ctypes.byref(n), ctypes.byref(loc)))
        return n.value, loc.value

    def allreduce(self, local: int, ptr: int, count: int, dtype: int, op: int) -> None:
        st = load().qsml_allreduce(self.h, int(local), ctypes.c_void_p(ptr), int(count), int(dtype), int(op))
        if st != OK:
            raise QsmlError(st, load().qsml_last_error(self.ctxs[local].h).decode())

    def _check_local(self, st: int, local: int) -> None:
        if st != OK:
            raise QsmlError(st, load().qsml_last_error(self.ctxs[local].h).decode())

    def allreduce_partials(self, local: int, op: int, ptr: int, count: int) -> None:
        """Combines `count` binary32 partials of reduction `op` across the group, in place."""
        self._check_local(load().qsml_allreduce_partials(self.h, int(local), int(op), ctypes.c_void_p(ptr),
                                                         int(count)), local)

    def reduce_sharded(self, local: int, op: int, a: TDesc, axis: int, keepdims: bool, out: TDesc,
                       global_rows: int = 0) -> None:
        """One reduction of a tensor whose rows are split over the group's ranks."""
        self._check_local(load().qsml_reduce_sharded(self.h, int(local), int(op), ctypes.byref(a), int(axis),
                                                     int(bool(keepdims)), ctypes.byref(out), int(global_rows)),
                          local)

    def destroy(self) -> None:
        if self.h:
            _check_global(load().qsml_group_destroy(self.h))
            self.h = None


def shard_rows(rows: int, nranks: int, rank: int) -> tuple:
    """(begin, count) of rank `rank`'s rows under the library's balanced split."""
    b, c = ctypes.c_int64(), ctypes.c_int64()
    _check_global(load().qsml_shard_rows(int(rows), int(nranks), int(rank), ctypes.byref(b), ctypes.byref(c)))
    return b.value, c.value


def group_start() -> None:
    _check_global(load().qsml_group_start())


def group_end() -> None:
    _check_global(load().qsml_group_end())


def declared_functions() -> list:
    """Names of the functions include/qsml_cuda.h declares."""
    import re
    text = open(HEADER_PATH).read()
    return sorted(set(re.findall(r"QSML_API\s+[\w\s\*]+?\b(qsml_\w+)\s*\(", text)))


def make_desc(ptr: int, dtype: int, shape: Sequence[int], strides: Optional[Sequence[int]] = None) -> TDesc:
    shape = [int(s) for s in shape]
    if len(shape) > MAX_DIMS:
        raise ValueError("too many dims")
    if strides is None:
        strides, s = [0] * len(shape), 1
        for i in range(len(shape) - 1, -1, -1):
            strides[i] = s
            s *= shape[i]
    d = TDesc()
    d.data = ctypes.c_void_p(int(ptr)) if ptr else None
    d.dtype = dtype
    d.ndim = len(shape)
    for i, (n, st) in enumerate(zip(shape, strides)):
        d.shape[i] = n
        d.stride[i] = int(st)
    return d


def torch_dtype_code(dt) -> int:
    import torch
    table = {torch.float32: F32, torch.float16: F16, torch.int32: I32, torch.int16: I16,
             torch.int8: I8, torch.uint8: U8}
    if hasattr(torch, "uint16"):
        table[torch.uint16] = U16
        table[torch.uint32] = U32
    return table[dt]


def desc_of(t) -> TDesc:
    """Descriptor of a torch CUDA tensor (any strides; storage offset applied)."""
    return make_desc(t.data_ptr(), torch_dtype_code(t.dtype), tuple(t.shape), tuple(t.stride()))


class Context:
    """One qsml_ctx: a device, a stream and a caching allocator."""

    def __init__(self, device: int = 0, use_torch_stream: bool = True):
        self.lib = load()
        h = ctypes.c_void_p()
        st = self.lib.qsml_init(int(device), ctypes.byref(h))
        if st != OK:
            raise QsmlError(st, self.lib.qsml_last_error(None).decode())
        self.h = h
        self.device = device
        if use_torch_stream:
            import torch
            self.set_stream(torch.cuda.current_stream(device).cuda_stream)

    # -- plumbing ------------------------------------------------------------
    def check(self, st: int) -> None:
        if st != OK:
            raise QsmlError(st, self.lib.qsml_last_error(self.h).decode())

    def close(self) -> None:
        if self.h:
            self.check(self.lib.qsml_destroy(self.h))
            self.h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def set_stream(self, stream_ptr: int) -> None:
        """Enqueue on this cudaStream_t (0 = the legacy default stream, which is
        what torch reports for its default stream)."""
        self.check(self.lib.qsml_set_stream(self.h, ctypes.c_void_p(int(stream_ptr)) if stream_ptr else None))

    def stream(self) -> int:
        s = ctypes.c_void_p()
        self.check(self.lib.qsml_get_stream(self.h, ctypes.byref(s)))
        return s.value or 0

    def synchronize(self) -> None:
        self.check(self.lib.qsml_synchronize(self.h))

    def set_wait_limit(self, cycles: int) -> None:
        """SM cycles after which a kernel waiting for data gives up with
        QSML_E_TIMEOUT (0 = the default, about 1 s)."""
        self.check(self.lib.qsml_set_wait_limit(self.h, cycles))

    def set_overlap(self, enable: bool) -> None:
        """Let independent reductions, arg-reductions, layer norms, softmaxes
        and gathers on this context's stream overlap (each starts reading
        while the library kernels before it that share no buffer with it
        still run).  Only for streams on which nothing else launches kernels
        that trigger programmatic dependent launch early."""
        self.check(self.lib.qsml_set_overlap(self.h, 1 if enable else 0))

    def overlap_stats(self) -> tuple:
        """(launches planned for overlap, of which overlapped the kernels before them)."""
        p, d = ctypes.c_uint64(), ctypes.c_uint64()
        self.check(self.lib.qsml_overlap_stats(self.h, ctypes.byref(p), ctypes.byref(d)))
        return p.value, d.value

    def finish_partial(self, op: int, partial: TDesc, n: int, out: TDesc) -> None:
        """out from combined binary32 partials (a mean divides by n)."""
        self.check(self.lib.qsml_finish_partial(self.h, int(op), ctypes.byref(partial), int(n), ctypes.byref(out)))

    def launch_count(self) -> int:
        n = ctypes.c_uint64()
        self.check(self.lib.qsml_launch_count(self.h, ctypes.byref(n)))
        return n.value

    def last_kernel(self) -> str:
        """Name of the last kernel this context launched ("" before any)."""
        buf = ctypes.create_string_buffer(128)
        self.check(self.lib.qsml_last_kernel(self.h, buf, len(buf)))
        return buf.value.decode()

    def cpu_fallback_count(self) -> int:
        n = ctypes.c_uint64()
        self.check(self.lib.qsml_cpu_fallback_count(self.h, ctypes.byref(n)))
        return n.value

    def allocator_stats(self) -> dict:
        v = [ctypes.c_uint64() for _ in range(4)]
        self.check(self.lib.qsml_allocator_stats(self.h, *[ctypes.byref(x) for x in v]))
        return dict(zip(["misses", "hits", "reserved_bytes", "live_bytes"], [x.value for x in v]))

    # -- memory --------------------------------------------------------------
    def alloc(self, nbytes: int) -> int:
        p = ctypes.c_void_p()
        self.check(self.lib.qsml_alloc(self.h, int(nbytes), ctypes.byref(p)))
        return p.value

    def free(self, ptr: int) -> None:
        self.check(self.lib.qsml_free(self.h, ctypes.c_void_p(ptr)))

    def h2d(self, dst: int, src: int, nbytes: int) -> None:
        self.check(self.lib.qsml_h2d(self.h, ctypes.c_void_p(dst), ctypes.c_void_p(src), int(nbytes)))

    def d2h(self, dst: int, src: int, nbytes: int, sync: bool = True) -> None:
        fn = self.lib.qsml_d2h if sync else self.lib.qsml_d2h_async
        self.check(fn(self.h, ctypes.c_void_p(dst), ctypes.c_void_p(src), int(nbytes)))

    def fill(self, dst: int, value_bytes: bytes, count: int) -> None:
        buf = ctypes.create_string_buffer(value_bytes, len(value_bytes))
        self.check(self.lib.qsml_fill(self.h, ctypes.c_void_p(dst), buf, len(value_bytes), int(count)))

    # -- ops (descriptors) ---------------------------------------------------
    def binary(self, op: int, a: TDesc, b: TDesc, out: TDesc) -> None:
        self.check(self.lib.qsml_binary(self.h, op, ctypes.byref(a), ctypes.byref(b), ctypes.byref(out)))

    def binary_scalar(self, op: int, a: TDesc, s: float, out: TDesc) -> None:
        self.check(self.lib.qsml_binary_scalar(self.h, op, ctypes.byref(a), ctypes.c_float(s), ctypes.byref(out)))

    def unary(self, op: int, a: TDesc, out: TDesc) -> None:
        self.check(self.lib.qsml_unary(self.h, op, ctypes.byref(a), ctypes.byref(out)))

    def reduce(self, op: int, a: TDesc, axis: int, keepdims: bool, out: TDesc) -> None:
        self.check(self.lib.qsml_reduce(self.h, op, ctypes.byref(a), int(axis), int(bool(keepdims)), ctypes.byref(out)))

    def arg_reduce(self, op: int, a: TDesc, axis: int, keepdims: bool, out: TDesc) -> None:
        self.check(self.lib.qsml_arg_reduce(self.h, op, ctypes.byref(a), int(axis), int(bool(keepdims)),
                                            ctypes.byref(out)))

    def elementwise_fused(self, nodes, inputs: Sequence[TDesc], out: TDesc) -> None:
        """nodes: FuseNode array or (kind, code, a, b, value) tuples; the
        last node is the result."""
        if not isinstance(nodes, ctypes.Array):
            arr = (FuseNode * max(len(nodes), 1))()
            for i, n in enumerate(nodes):
                arr[i] = FuseNode(*n)
            n_nodes = len(nodes)
        else:
            arr, n_nodes = nodes, len(nodes)
        ins = (TDesc * max(len(inputs), 1))(*inputs)
        self.check(self.lib.qsml_elementwise_fused(self.h, arr, n_nodes, ins, len(inputs), ctypes.byref(out)))

    def set_fuse_mode(self, mode: int) -> None:
        self.check(self.lib.qsml_set_fuse_mode(self.h, int(mode)))

    def fuse_stats(self) -> tuple:
        """(runtime-compiled launches, interpreter launches, kernels compiled)."""
        j, i, k = ctypes.c_uint64(), ctypes.c_uint64(), ctypes.c_uint64()
        self.check(self.lib.qsml_fuse_stats(self.h, ctypes.byref(j), ctypes.byref(i), ctypes.byref(k)))
        return j.value, i.value, k.value

    def gather(self, src: TDesc, out: TDesc) -> None:
        self.check(self.lib.qsml_gather(self.h, ctypes.byref(src), ctypes.byref(out)))

    def cast(self, src: TDesc, out: TDesc) -> None:
        """out = src converted to out's dtype (F32 <-> F16)."""
        self.check(self.lib.qsml_cast(self.h, ctypes.byref(src), ctypes.byref(out)))

    def softmax(self, x: TDesc, axis: int, y: TDesc) -> None:
        self.check(self.lib.qsml_softmax(self.h, ctypes.byref(x), int(axis), ctypes.byref(y)))

    def layer_norm(self, x: TDesc, g: TDesc, b: TDesc, eps: float, y: TDesc) -> None:
        self.check(self.lib.qsml_layer_norm(self.h, ctypes.byref(x), ctypes.byref(g), ctypes.byref(b),
                                            ctypes.c_float(eps), ctypes.byref(y)))

    def matmul(self, a: TDesc, b: TDesc, c: TDesc, precision: int = MM_AUTO) -> None:
        self.check(self.lib.qsml_matmul(self.h, ctypes.byref(a), ctypes.byref(b), ctypes.byref(c), precision))


def broadcast_shape(a: Iterable[int], b: Iterable[int]) -> tuple:
    """NumPy broadcasting of two shapes (raises ValueError if incompatible)."""
    a, b = list(a), list(b)
    n = max(len(a), len(b))
    a = [1] * (n - len(a)) + a
    b = [1] * (n - len(b)) + b
    out = []
    for x, y in zip(a, b):
        if x != y and x != 1 and y != 1:
            raise ValueError(f"shapes {a} and {b} do not broadcast")
        out.append(y if x == 1 else x)
    return tuple(out)


def reduced_shape(shape: Sequence[int], axis: Optional[int], keepdims: bool) -> tuple:
    """Output shape of a reduction, following Ops/Reduction.cpp:297-305."""
    if axis is None or axis == AXIS_ALL:
        return (1,)
    ax = axis + len(shape) if axis < 0 else axis
    if not 0 <= ax < len(shape):
        raise ValueError("invalid axis")
    out = [d if i != ax else 1 for i, d in enumerate(shape) if i != ax or keepdims]
    return tuple(out) if out else (1,)
