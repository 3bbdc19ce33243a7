"""Synthetic workloads of the benchmark configurations (seeded).

The shapes and value distributions are the ones the configurations name:
A iid N(0, 1) and B iid N(0, 1) -- or N(0, 0.02) for the weight operand of
the projection and skinny configurations -- drawn in fp32 from a fixed seed
and cast to bf16; B is generated as (N, K) and passed as its (K, N) view,
as the reference's harness does (src/bench_core.py:110-111).
"""
from __future__ import annotations

import torch

# (M, N, K) per configuration.
SQUARE_1024 = [(1024, 1024, 1024)]
SQUARE = [(2048, 2048, 2048), (4096, 4096, 4096), (8192, 8192, 8192), (16384, 16384, 16384)]
PROJECTION = [(8192, 6144, 4096), (8192, 4096, 4096), (8192, 28672, 4096), (8192, 4096, 14336)]
SKINNY = [(16, 8192, 8192), (64, 8192, 8192), (128, 8192, 8192), (256, 8192, 8192)]
M_SHARD = (131072, 8192, 8192)   # rows split across GPUs, B replicated
K_SPLIT = (8192, 8192, 131072)   # K split across GPUs, fp32 partials reduce-scattered

CONFIGS = {
    "square_1024": SQUARE_1024,
    "square": SQUARE,
    "projection": PROJECTION,
    "skinny": SKINNY,
    "m_shard": [M_SHARD],
    "k_split": [K_SPLIT],
}

# Weight operand standard deviation per configuration (1.0 = N(0, 1)).
WEIGHT_STD = {"square_1024": 1.0, "square": 1.0, "projection": 0.02, "skinny": 0.02,
              "m_shard": 1.0, "k_split": 1.0}


def flops(M: int, N: int, K: int) -> int:
    return 2 * M * N * K


def min_bytes(M: int, N: int, K: int) -> int:
    """Algorithmic HBM bytes: read A and B once, write C once (bf16)."""
    return 2 * (M * K + N * K + M * N)


def make_operands(M: int, N: int, K: int, seed: int = 0, weight_std: float = 1.0,
                  device="cuda"):
    """Returns (A, Bt): A is (M, K) bf16, Bt is (N, K) bf16; the GEMM operand
    in the reference's convention is ``Bt.T``."""
    g = torch.Generator(device=device)
    g.manual_seed(seed)
    A = torch.randn(M, K, generator=g, device=device, dtype=torch.float32).to(torch.bfloat16)
    Bt = torch.randn(N, K, generator=g, device=device, dtype=torch.float32)
    if weight_std != 1.0:
        Bt.mul_(weight_std)
    return A, Bt.to(torch.bfloat16)
