"""QuasarML B200 backend: sm_100a CUDA kernels behind QuasarML's op API.

The product is native code: libqsml_cuda.so (extern "C" ABI, include/qsml_cuda.h)
and the C++ QuasarML layer in quasarml_b200/cpp.  This Python package only
binds the ABI (``abi``) and provides the seeded input generator (``datagen``)
used by the tests and the benchmark.
"""
from . import abi  # noqa: F401

__all__ = ["abi"]
