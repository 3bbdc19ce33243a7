"""CPU oracle for the BF16 GEMM  C = A * B^T  -- TEST INFRASTRUCTURE ONLY.

Only tests/, ``__graft_entry__.smoke()`` and bench.py's CPU-baseline /
reference legs may import this package, and only as the checker or the
baseline being reported; the product (``blackwell_gemm_b200``) never does.

Contents
  gemm_f32 / gemm_bf16   the C restatement in gemm_oracle.c (liboracle.so):
                         bf16 products, fp32 accumulation in a fixed order,
                         round-to-nearest-even to bf16 (reference semantics:
                         src/kernels/kernel_v8.cu:450-455,554-589,716)
  numpy_gemm_f32         independent cross-check through numpy/BLAS sgemm
  round_bf16, bf16_to_f32 bit-level conversions
  exact_inputs           operands whose products and sums are exact in fp32,
                         so every correct implementation returns identical
                         bits (known-answer tests)
  ref_lib / ref_gemm     the reference's own kernels built from its sources
                         (oracle/_ref/libref_gemm.so, GPU only)

Parity pins: tests/test_oracle.py checks this oracle against the golden
vectors in tests/golden/, which were produced by running the reference's own
v8 kernel (tests/golden/make_golden.py).
"""
from __future__ import annotations

import ctypes
import os
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
ORACLE_SO = HERE / "liboracle.so"
REF_SO = HERE / "_ref" / "libref_gemm.so"

_lib = None
_ref = None


def lib() -> ctypes.CDLL:
    global _lib
    if _lib is None:
        if not ORACLE_SO.exists():
            raise ImportError("oracle/liboracle.so is not built; run `python oracle/build.py`")
        h = ctypes.CDLL(str(ORACLE_SO))
        vp, i = ctypes.c_void_p, ctypes.c_int
        h.oracle_gemm_f32.argtypes = [vp, vp, vp, i, i, i, i, i, i, i]
        h.oracle_gemm_f32.restype = i
        h.oracle_gemm_bf16.argtypes = [vp, vp, vp, i, i, i, i, i, i, i]
        h.oracle_gemm_bf16.restype = i
        h.oracle_round_bf16.argtypes = [vp, vp, ctypes.c_int64]
        h.oracle_round_bf16.restype = None
        h.oracle_bf16_to_f32.argtypes = [vp, vp, ctypes.c_int64]
        h.oracle_bf16_to_f32.restype = None
        _lib = h
    return _lib


def _u16(x) -> np.ndarray:
    x = np.ascontiguousarray(x)
    if x.dtype != np.uint16:
        raise TypeError("bf16 operands are passed as uint16 bit patterns")
    return x


def default_threads() -> int:
    return max(1, len(os.sched_getaffinity(0)) if hasattr(os, "sched_getaffinity") else
               (os.cpu_count() or 1))


def gemm_f32(A: np.ndarray, B: np.ndarray, nthreads: int | None = None) -> np.ndarray:
    """fp32 C = A * B^T for bf16 bit patterns A (M x K) and B (N x K)."""
    A, B = _u16(A), _u16(B)
    M, K = A.shape
    N, K2 = B.shape
    assert K == K2, "inner dimensions differ"
    C = np.empty((M, N), dtype=np.float32)
    st = lib().oracle_gemm_f32(A.ctypes.data, B.ctypes.data, C.ctypes.data, M, N, K, K, K, N,
                               nthreads or default_threads())
    if st != 0:
        raise RuntimeError(f"oracle_gemm_f32 failed ({st})")
    return C


def gemm_bf16(A: np.ndarray, B: np.ndarray, nthreads: int | None = None) -> np.ndarray:
    """bf16 (uint16 bits) C = rne_bf16(A * B^T)."""
    return round_bf16(gemm_f32(A, B, nthreads))


def round_bf16(x: np.ndarray) -> np.ndarray:
    x = np.ascontiguousarray(x, dtype=np.float32)
    y = np.empty(x.shape, dtype=np.uint16)
    lib().oracle_round_bf16(x.ctypes.data, y.ctypes.data, x.size)
    return y


def bf16_to_f32(x: np.ndarray) -> np.ndarray:
    return (_u16(x).astype(np.uint32) << 16).view(np.float32)


def numpy_gemm_f32(A: np.ndarray, B: np.ndarray) -> np.ndarray:
    """Independent restatement through numpy (BLAS sgemm, fp32)."""
    return bf16_to_f32(A) @ bf16_to_f32(B).T


def exact_inputs(M: int, N: int, K: int, seed: int = 0):
    """bf16 operands with entries in {-4..4}/4: every product is a multiple of
    1/16 and |partial sum| <= K, so fp32 accumulation is exact in any order
    while K * 16 < 2^24.  The bf16 result is then unique: identical bits from
    the oracle, the reference and any correct kernel."""
    assert K * 16 < (1 << 24)
    rng = np.random.default_rng(seed)
    a = rng.integers(-4, 5, size=(M, K)).astype(np.float32) / 4
    b = rng.integers(-4, 5, size=(N, K)).astype(np.float32) / 4
    return round_bf16(a), round_bf16(b)


# ----------------------------------------------------------------- reference
def ref_lib() -> ctypes.CDLL:
    """The reference's kernels (GPU).  torch must be imported first (libc10)."""
    global _ref
    if _ref is None:
        if not REF_SO.exists():
            raise ImportError("oracle/_ref/libref_gemm.so is not built (needs the reference "
                              "checkout at build time); run `python oracle/build.py`")
        import torch  # noqa: F401

        h = ctypes.CDLL(str(REF_SO), mode=ctypes.RTLD_GLOBAL)
        vp, i = ctypes.c_void_p, ctypes.c_int
        h.ref_gemm.argtypes = [ctypes.c_char_p, vp, vp, vp, i, i, i]
        h.ref_gemm.restype = i
        h.ref_supports.argtypes = [ctypes.c_char_p, i, i, i]
        h.ref_supports.restype = i
        _ref = h
    return _ref


def ref_supports(version: str, M: int, N: int, K: int) -> bool:
    return bool(ref_lib().ref_supports(version.encode(), M, N, K))


def ref_gemm(version: str, a_ptr: int, bt_ptr: int, c_ptr: int, M: int, N: int, K: int) -> None:
    """Run the reference's matmul_<version> on device pointers (A M x K, B^T
    N x K, C M x N, all contiguous bf16) on the legacy default stream."""
    st = ref_lib().ref_gemm(version.encode(), a_ptr, bt_ptr, c_ptr, M, N, K)
    if st != 0:
        raise RuntimeError(f"reference {version} refused {M}x{N}x{K} (status {st})")
