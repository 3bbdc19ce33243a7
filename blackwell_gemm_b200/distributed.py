"""Multi-GPU GEMM on one node: one process per GPU, ``torch.distributed``.

The reference is single-GPU; these are the two multi-GPU configurations the
build is measured on:

* **Row-sharded** (``row_shard_gemm``): each rank owns ``M/P`` rows of A and
  a replicated B and computes its rows of C.  No collective touches the data
  path; work per GPU is fixed as P grows when M grows with it.
* **K-split** (``k_split_gemm``): each rank owns the K-slice ``A[:, Kr]`` and
  ``B[:, Kr]``, computes the fp32 partial ``A[:, Kr] B[:, Kr]^T`` (M x N, not
  rounded) with ``b200_gemm_bf16_f32out``, the partials are summed by an NCCL
  reduce-scatter over NVLink (``op=SUM``; rank r receives rows
  ``[r M/P, (r+1) M/P)``) and rank r rounds its rows to bf16 once
  (``b200_cast_f32_bf16``).  Rounding once after the sum keeps the result
  equal, up to fp32 summation order, to the single-GPU GEMM.

The local GEMM and the cast are arguments so the collective logic can be
exercised on CPU ranks (``gloo``) with a plain fp32 GEMM; the GPU path always
uses this package's kernels.
"""
from __future__ import annotations

from typing import Callable, Optional

import torch
import torch.distributed as dist


def gemm_f32_cuda(A: torch.Tensor, Bt: torch.Tensor) -> torch.Tensor:
    """fp32 A @ Bt^T on the GPU through the C ABI (bf16 in, fp32 out)."""
    from . import capi

    M, K = A.shape
    N = Bt.shape[0]
    assert A.is_contiguous() and Bt.is_contiguous() and A.dtype == Bt.dtype == torch.bfloat16
    C = torch.empty(M, N, dtype=torch.float32, device=A.device)
    st = capi.gemm_bf16_f32out(A.data_ptr(), Bt.data_ptr(), C.data_ptr(), M, N, K, K, K, N,
                               torch.cuda.current_stream(A.device).cuda_stream)
    capi.check(st, "b200_gemm_bf16_f32out")
    return C


def cast_bf16_cuda(W: torch.Tensor) -> torch.Tensor:
    """bf16 round-to-nearest-even of a contiguous fp32 CUDA matrix."""
    from . import capi

    M, N = W.shape
    C = torch.empty(M, N, dtype=torch.bfloat16, device=W.device)
    st = capi.cast_f32_bf16(W.data_ptr(), N, C.data_ptr(), N, M, N,
                            torch.cuda.current_stream(W.device).cuda_stream)
    capi.check(st, "b200_cast_f32_bf16")
    return C


def gemm_bf16_cuda(A: torch.Tensor, Bt: torch.Tensor) -> torch.Tensor:
    from . import capi

    M, K = A.shape
    N = Bt.shape[0]
    C = torch.empty(M, N, dtype=torch.bfloat16, device=A.device)
    st = capi.gemm_bf16(A.data_ptr(), Bt.data_ptr(), C.data_ptr(), M, N, K, K, K, N,
                        torch.cuda.current_stream(A.device).cuda_stream)
    capi.check(st, "b200_gemm_bf16")
    return C


def row_shard_gemm(A_rows: torch.Tensor, Bt: torch.Tensor,
                   gemm: Callable = gemm_bf16_cuda) -> torch.Tensor:
    """This rank's rows of C = A B^T: A_rows is its (M/P, K) block, Bt the
    replicated (N, K) operand.  No communication."""
    return gemm(A_rows, Bt)


def k_split_gemm(A_k: torch.Tensor, Bt_k: torch.Tensor, group: Optional[dist.ProcessGroup] = None,
                 gemm_f32: Callable = gemm_f32_cuda,
                 cast: Callable = cast_bf16_cuda) -> torch.Tensor:
    """Rank r's rows ``[r M/P, (r+1) M/P)`` of C = A B^T, where A_k = A[:, Kr]
    (M x K/P) and Bt_k = B[:, Kr] (N x K/P) are this rank's K-slices.  M must
    be divisible by the group size."""
    world = dist.get_world_size(group)
    M = A_k.shape[0]
    if M % world:
        raise ValueError(f"M={M} is not divisible by the {world} ranks of the K-split")
    partial = gemm_f32(A_k, Bt_k)                     # M x N fp32, unrounded
    out = torch.empty(M // world, partial.shape[1], dtype=torch.float32, device=partial.device)
    dist.reduce_scatter_tensor(out, partial, op=dist.ReduceOp.SUM, group=group)
    return cast(out)


def k_slice(K: int, world: int, rank: int) -> slice:
    """Rank's contiguous K range; K must be divisible by world."""
    if K % world:
        raise ValueError(f"K={K} is not divisible by {world} ranks")
    k = K // world
    return slice(rank * k, (rank + 1) * k)
