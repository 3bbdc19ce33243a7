"""blackwell_gemm_b200 -- BF16 GEMM (C = A @ B, B given as the (K, N) view of an
N x K buffer) as hand-written sm_100a CUDA for B200.

Drop-in for the reference's extension module (src/matmul.cpp:109-124): the
harness calls ``getattr(module, f"matmul_{version}")(A, B)``
(src/bench_core.py:115,120); here ``version = "b200"``:

    from blackwell_gemm_b200 import module
    C = module.matmul_b200(A, B)
    C = module.profile_matmul_b200(A, B, profiler, num_entries)

``matmul_b200`` / ``profile_matmul_b200`` come from the torch extension
``_C`` (csrc/matmul.cpp), which calls the C ABI of libb200gemm.so
(include/b200_gemm.h, ctypes binding in ``capi``).  Both are built in-tree by
``blackwell_gemm_b200.build``; importing raises if they are missing.  There is
no CPU or library fallback.
"""
from __future__ import annotations

import importlib
import types

from . import capi  # noqa: F401

__all__ = ["module", "matmul_b200", "profile_matmul_b200", "profile_rows", "capi", "load"]

_ext = None


def load():
    """Import the torch extension (after torch, whose libraries it links)."""
    global _ext
    if _ext is None:
        import torch  # noqa: F401  (loads libc10/libtorch for the extension)

        capi.lib()  # libb200gemm.so must be present and loadable
        try:
            _ext = importlib.import_module("blackwell_gemm_b200._C")
        except ImportError as e:
            raise ImportError("blackwell_gemm_b200._C is not built; run "
                              "`python -m blackwell_gemm_b200.build`") from e
    return _ext


def matmul_b200(A, B):
    """C = A @ B.  A: (M, K) bf16 CUDA, B: (K, N) bf16 CUDA (normally the .T of
    an N x K tensor).  Returns a new contiguous (M, N) bf16 tensor computed on
    the current stream with fp32 accumulation."""
    return load().matmul_b200(A, B)


def profile_matmul_b200(A, B, profiler, num_entries: int):
    """matmul_b200 with the intra-kernel profiler on: ``profiler`` is an int64
    CUDA tensor with at least ``profile_rows(M, N, K) * (1 + 4 * num_entries)``
    elements (see ``blackwell_gemm_b200.profiler``)."""
    return load().profile_matmul_b200(A, B, profiler, int(num_entries))


def profile_rows(M: int, N: int, K: int) -> int:
    return capi.profile_rows(M, N, K)


module = types.SimpleNamespace(matmul_b200=matmul_b200, profile_matmul_b200=profile_matmul_b200)
