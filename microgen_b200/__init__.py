"""B200-native (sm_100a) decode-step hot path for MicroGen.

INT8 weight-only tensor-parallel linears and paged-KV decode attention as
hand-written CUDA kernels behind a C-ABI shared library
(``libmicrogen_b200.so``, declared in ``include/microgen_b200.h``), with the
reference's backend and paged-allocator interfaces mirrored on the host side:

* ``microgen_b200.backends``  — ``QuantizedLinear`` / ``ColumnParallelLinear`` /
  ``RowParallelLinear`` modules and the ``InferenceBackend`` implementations;
* ``microgen_b200.runtime``   — ``PagedKVCacheAllocator`` with a device KV pool;
* ``microgen_b200.kernels``   — thin ctypes wrappers over the C-ABI.

Importing this package does not load the library; the first kernel call does,
and raises if it is missing (there is no CPU fallback).
"""

__version__ = "0.1.0"
