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
* **Fused K-split** (``FusedKSplit``): the same decomposition in one kernel
  per rank (``b200_ksplit_gemm_bf16``): each rank writes the fp32 tiles of
  other owners' rows straight into the owner's memory over NVLink while it
  computes, and adds the peers' tiles to its own rows in the epilogue, so the
  exchange overlaps the tensor-core work and nothing is rounded twice.

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


class FusedKSplit:
    """Rank's rows of C = A B^T from K-slices, reduced over NVLink inside the
    GEMM kernel (``b200_ksplit_gemm_bf16``).

    Construction is a collective over ``group`` (each rank on its own GPU,
    the current device): every rank allocates its receive area for problems
    up to ``max_m`` x ``max_n``, the IPC handles are all-gathered and mapped.
    Calls are collectives too: every rank, same order, same M and N.
    ``close()`` (also a collective) synchronizes, waits for every rank and
    unmaps."""

    def __init__(self, max_m: int, max_n: int, group: Optional[dist.ProcessGroup] = None):
        from . import capi

        self.group = group
        # Without an initialised process group this is a one-rank instance.
        self.collective = dist.is_available() and dist.is_initialized()
        self.world = dist.get_world_size(group) if self.collective else 1
        self.rank = dist.get_rank(group) if self.collective else 0
        self.device = torch.device("cuda", torch.cuda.current_device())
        self.comm, handle = capi.ksplit_create(self.rank, self.world, max_m, max_n)
        handles = [handle]
        try:
            if self.collective:
                handles = [None] * self.world
                dist.all_gather_object(handles, handle, group=group)
            capi.ksplit_connect(self.comm, b"".join(handles))
        except BaseException:
            capi.ksplit_destroy(self.comm)       # unmaps what was mapped, frees the area
            self.comm = None
            raise
        if self.collective:
            dist.barrier(group)

    def __call__(self, A_k: torch.Tensor, Bt_k: torch.Tensor,
                 out: Optional[torch.Tensor] = None) -> torch.Tensor:
        """A_k = A[:, Kr] (M x K_r), Bt_k = B[:, Kr] (N x K_r), both contiguous
        bf16 on this rank's GPU; returns (or fills) rows [r M/P, (r+1) M/P)."""
        from . import capi

        if self.comm is None:
            raise RuntimeError("FusedKSplit is closed")
        self._check_operands(A_k, Bt_k)
        M, K = A_k.shape
        N = Bt_k.shape[0]
        if out is None:
            out = torch.empty(M // self.world, N, dtype=torch.bfloat16, device=A_k.device)
        else:
            self._check_out(out, M, N, A_k.device)
        st = capi.ksplit_gemm_bf16(self.comm, A_k.data_ptr(), Bt_k.data_ptr(), out.data_ptr(),
                                   M, N, K, K, K, out.stride(0),
                                   torch.cuda.current_stream(A_k.device).cuda_stream)
        capi.check(st, "b200_ksplit_gemm_bf16")
        return out

    def _check_operands(self, A_k: torch.Tensor, Bt_k: torch.Tensor) -> None:
        if A_k.dim() != 2 or Bt_k.dim() != 2 or Bt_k.shape[1] != A_k.shape[1]:
            raise ValueError("A_k must be M x K_r and Bt_k N x K_r")
        if A_k.dtype != torch.bfloat16 or Bt_k.dtype != torch.bfloat16:
            raise TypeError("A_k and Bt_k must be bfloat16")
        if A_k.device != Bt_k.device or A_k.device.type != "cuda":
            raise ValueError("A_k and Bt_k must be on one CUDA device")
        if A_k.device != self.device:
            # The communicator's receive area, its peer mappings and the
            # kernel's launch belong to self.device: operands on another GPU
            # must not reach the C ABI.
            raise ValueError(f"A_k and Bt_k must be on this rank's GPU {self.device}, "
                             f"not {A_k.device}")
        if not (A_k.is_contiguous() and Bt_k.is_contiguous()):
            raise ValueError("A_k (M x K_r) and Bt_k (N x K_r) must be contiguous")

    def _check_out(self, out: torch.Tensor, M: int, N: int, device: torch.device) -> None:
        # The kernel writes M/P rows of N columns at out's row stride: a
        # smaller or differently typed buffer would be written past its end.
        if out.dtype != torch.bfloat16 or out.device != device:
            raise TypeError("out must be bfloat16 on the operands' GPU")
        if tuple(out.shape) != (M // self.world, N) or out.stride(1) != 1:
            raise ValueError(f"out must be ({M // self.world}, {N}) with unit column stride")

    def close(self) -> None:
        from . import capi

        if self.comm is None:
            return
        torch.cuda.synchronize(self.device)
        if self.collective:
            dist.barrier(self.group)
        capi.ksplit_destroy(self.comm)
        self.comm = None


def k_slice(K: int, world: int, rank: int) -> slice:
    """Rank's contiguous K range; K must be divisible by world."""
    if K % world:
        raise ValueError(f"K={K} is not divisible by {world} ranks")
    k = K // world
    return slice(rank * k, (rank + 1) * k)


def k_split_sampled_parity(out_rows: torch.Tensor, A_k: torch.Tensor, Bt_k: torch.Tensor,
                           group: Optional[dist.ProcessGroup] = None, per_owner: int = 32,
                           seed: int = 1) -> dict:
    """Parity of a K-split GEMM's output against an fp32 GEMM of the same bf16
    inputs over the WHOLE K, on sampled rows, although no rank holds all of K.

    ``out_rows`` is this rank's (M/P, N) block of C; ``A_k`` (M x K_r) and
    ``Bt_k`` (N x K_r) its K-slices.  Every rank draws the same ``per_owner``
    rows from each owner's block, computes their fp32 partial over its own
    K-slice (no TF32) together with the squared row norms of its slices, and
    the partials and norms are summed across ranks (all_reduce), which gives
    the full-K fp32 reference of the sampled rows and the full-K norms.  Each
    rank then compares its own sampled rows; the metrics of ``parity.metrics``
    are combined across ranks (max of ``max_scaled``; ``rel_fro`` over all
    sampled rows).  A collective: every rank calls it.  Returns the same dict
    on every rank."""
    from . import parity

    collective = dist.is_available() and dist.is_initialized()
    world = dist.get_world_size(group) if collective else 1
    rank = dist.get_rank(group) if collective else 0
    M, N = A_k.shape[0], Bt_k.shape[0]
    rows = M // world
    if out_rows.shape[0] != rows or out_rows.shape[1] != N:
        raise ValueError(f"out_rows must be ({rows}, {N})")
    take = min(per_owner, rows)
    g = torch.Generator().manual_seed(seed)
    sample = torch.cat([q * rows + torch.randperm(rows, generator=g)[:take]
                        for q in range(world)]).to(A_k.device)
    a = A_k.index_select(0, sample)
    prev = torch.backends.cuda.matmul.allow_tf32
    torch.backends.cuda.matmul.allow_tf32 = False
    try:
        ref = a.float() @ Bt_k.float().T                       # |S| x N partial over K_r
    finally:
        torch.backends.cuda.matmul.allow_tf32 = prev
    na2 = a.double().square().sum(1)
    nb2 = Bt_k.double().square().sum(1)
    if collective:
        for t in (ref, na2, nb2):
            dist.all_reduce(t, op=dist.ReduceOp.SUM, group=group)
    mine = slice(rank * take, (rank + 1) * take)
    C = out_rows.index_select(0, sample[mine] - rank * rows).double()
    R = ref[mine].double()
    diff = (C - R).abs()
    scale = na2[mine].sqrt()[:, None] * nb2.sqrt()[None, :]
    ratio = torch.where(scale > 0, diff / scale.clamp_min(1e-300),
                        torch.where(diff > 0, torch.full_like(diff, float("inf")),
                                    torch.zeros_like(diff)))
    finite = bool(torch.isfinite(C).all())
    stats = torch.tensor([float(ratio.max()) if finite and ratio.numel() else
                          (0.0 if finite else float("inf")),
                          float(diff.square().sum()), float(R.square().sum())],
                         dtype=torch.float64, device=A_k.device)
    if collective:
        mx = stats[:1].clone()
        sums = stats[1:].clone()
        dist.all_reduce(mx, op=dist.ReduceOp.MAX, group=group)
        dist.all_reduce(sums, op=dist.ReduceOp.SUM, group=group)
        stats = torch.cat([mx, sums])
    max_scaled, sq_diff, sq_ref = (float(v) for v in stats)
    rel_fro = (sq_diff / sq_ref) ** 0.5 if sq_ref > 0 else (0.0 if sq_diff == 0 else float("inf"))
    m = {"max_scaled": max_scaled, "rel_fro": rel_fro}
    return {**m, "pass": parity.passes(m), "rows_checked": take * world,
            "against": "fp32 GEMM of the same bf16 inputs over the whole K (sampled rows; "
                       "partials summed across ranks, no TF32)"}
