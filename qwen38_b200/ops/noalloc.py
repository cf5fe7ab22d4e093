"""ctypes binding of the allocation-free GEMM entry point (``csrc/q38_noalloc.h``).

``q38_linear_noalloc`` serves callers that cannot allocate device memory at call time: its
scratch lives in a fixed device array inside the extension (see the header for the rules of use).
The argument types below follow the header's prototypes; ``tests/test_noalloc_header.py`` parses
the header and checks them, so the two cannot drift apart silently.
"""
from __future__ import annotations

import ctypes

# C prototypes, as declared in csrc/q38_noalloc.h (parameter C types in order)
PROTOTYPES = {
    "q38_linear_noalloc": ("int", ["const void*", "int", "int", "const void*", "int", "void*", "int", "int",
                                   "cudaStream_t"]),
    "q38_linear_noalloc_status": ("int", []),
}

_CTYPES = {"int": ctypes.c_int, "const void*": ctypes.c_void_p, "void*": ctypes.c_void_p,
           "cudaStream_t": ctypes.c_void_p}

OK, EARG, ESIZE, ECUDA = 0, 1, 2, 3
EPI_BF16, EPI_F32, EPI_ADD_F32 = 0, 1, 2


def bind(so_path: str):
    """(q38_linear_noalloc, q38_linear_noalloc_status) from the built extension at ``so_path``."""
    lib = ctypes.CDLL(so_path)
    out = []
    for name, (ret, args) in PROTOTYPES.items():
        fn = getattr(lib, name)
        fn.restype = _CTYPES[ret]
        fn.argtypes = [_CTYPES[a] for a in args]
        out.append(fn)
    return tuple(out)
