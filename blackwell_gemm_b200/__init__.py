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

__all__ = ["module", "matmul_b200", "profile_matmul_b200", "matmul_b200_epilogue",
           "matmul_b200_host", "profile_rows", "capi", "load"]

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


def _row_major(t):
    """Row-major view with a 16-byte aligned row stride (copies if needed)."""
    rows, cols = t.shape
    ok = (cols <= 1 or t.stride(1) == 1) and (rows <= 1 or (t.stride(0) % 8 == 0 and
                                                           t.stride(0) >= cols))
    if ok and t.data_ptr() % 16 == 0:
        return t, (t.stride(0) if rows > 1 else (cols + 7) // 8 * 8)
    import torch
    ld = (cols + 7) // 8 * 8
    buf = torch.empty(rows, ld, dtype=t.dtype, device=t.device)
    buf[:, :cols].copy_(t)
    return buf[:, :cols], ld


def matmul_b200_epilogue(A, B, *, alpha: float = 1.0, bias=None, beta: float = 1.0,
                         residual=None):
    """C = round_bf16(alpha * (A @ B) + bias + beta * residual) in one pass.

    A: (M, K) bf16 CUDA; B: (K, N) bf16 CUDA (the (K, N) view of an N x K
    buffer, as for matmul_b200); bias: (N,) bf16 or None; residual: (M, N)
    bf16 or None.  Accumulation and the epilogue arithmetic are fp32; the
    result is rounded to bf16 once."""
    import torch

    if A.dim() != 2 or B.dim() != 2 or B.shape[0] != A.shape[1]:
        raise RuntimeError("matmul_b200_epilogue: A must be (M, K) and B (K, N)")
    for t in (A, B) + tuple(x for x in (bias, residual) if x is not None):
        if not t.is_cuda or t.dtype != torch.bfloat16 or t.device != A.device:
            raise RuntimeError("matmul_b200_epilogue: operands must be bfloat16 CUDA tensors "
                               "on one device")
    M, K = A.shape
    N = B.shape[1]
    a, lda = _row_major(A)
    bt, ldb = _row_major(B.t())
    ldc = (N + 7) // 8 * 8
    Cbuf = torch.empty(M, ldc, dtype=torch.bfloat16, device=A.device)
    bias_ptr = 0
    if bias is not None:
        if bias.shape != (N,):
            raise RuntimeError("matmul_b200_epilogue: bias must have shape (N,)")
        bias = bias.contiguous()
        if bias.data_ptr() % 16:
            bias = bias.clone()
        bias_ptr = bias.data_ptr()
    resid_ptr, ldr = 0, 0
    if residual is not None:
        if residual.shape != (M, N):
            raise RuntimeError("matmul_b200_epilogue: residual must have shape (M, N)")
        residual, ldr = _row_major(residual)
        resid_ptr = residual.data_ptr()
    with torch.cuda.device(A.device):
        st = capi.gemm_bf16_epilogue(a.data_ptr(), bt.data_ptr(), Cbuf.data_ptr(), M, N, K, lda,
                                     ldb, ldc, alpha, bias_ptr, beta, resid_ptr, ldr,
                                     torch.cuda.current_stream(A.device).cuda_stream)
    capi.check(st, "matmul_b200_epilogue")
    return Cbuf[:, :N] if ldc == N else Cbuf[:, :N].contiguous()


def matmul_b200_host(A, B, *, block_rows: int = 0, out=None):
    """C = A @ B for operands in host memory (CPU bf16 tensors; page-locked
    memory lets the transfers overlap).  A: (M, K); B: (K, N), normally the .T
    of an (N, K) tensor.  B is copied to the current CUDA device once, A is
    streamed in blocks of rows with uploads, GEMMs and downloads overlapped
    (b200_gemm_bf16_host).  Returns `out` or a new page-locked (M, N) tensor;
    waits for the result."""
    import torch

    if A.dim() != 2 or B.dim() != 2 or B.shape[0] != A.shape[1]:
        raise RuntimeError("matmul_b200_host: A must be (M, K) and B (K, N)")
    for t in (A, B):
        if t.is_cuda or t.dtype != torch.bfloat16:
            raise RuntimeError("matmul_b200_host: A and B must be bfloat16 CPU tensors")
    M, K = A.shape
    N = B.shape[1]
    a = A if A.stride(1) == 1 else A.contiguous()
    bt = B.t()
    if bt.stride(1) != 1:
        bt = bt.contiguous()
    if out is None:
        out = torch.empty(M, N, dtype=torch.bfloat16).pin_memory()
    if out.shape != (M, N) or out.stride(1) != 1:
        raise RuntimeError("matmul_b200_host: out must be a row-major (M, N) tensor")
    stream = torch.cuda.current_stream()
    st = capi.gemm_bf16_host(a.data_ptr(), bt.data_ptr(), out.data_ptr(), M, N, K,
                             a.stride(0) if M > 1 else K, bt.stride(0) if N > 1 else K,
                             out.stride(0) if M > 1 else N, block_rows, stream.cuda_stream)
    capi.check(st, "matmul_b200_host")
    stream.synchronize()
    return out


def profile_rows(M: int, N: int, K: int) -> int:
    return capi.profile_rows(M, N, K)


module = types.SimpleNamespace(matmul_b200=matmul_b200, profile_matmul_b200=profile_matmul_b200)
