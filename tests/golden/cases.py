"""Golden-vector cases: inputs are regenerated deterministically from a seed
(numpy PCG64 + the oracle's bf16 rounding); the fixture files hold the
reference kernel's bf16 output and a SHA-256 of the regenerated inputs so a
change in input generation is caught instead of silently comparing different
problems."""
from __future__ import annotations

import hashlib
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent

# Shapes the reference's v8 supports (M, N multiples of 256, K of 64).
CASES = [
    dict(name="exact_256x256x128", kind="exact", M=256, N=256, K=128, seed=11, std=1.0),
    dict(name="exact_512x512x320", kind="exact", M=512, N=512, K=320, seed=12, std=1.0),
    dict(name="randn_256x256x256", kind="randn", M=256, N=256, K=256, seed=13, std=1.0),
    dict(name="randn_w002_256x512x1024", kind="randn", M=256, N=512, K=1024, seed=14, std=0.02),
]


def inputs(case):
    import oracle

    M, N, K = case["M"], case["N"], case["K"]
    if case["kind"] == "exact":
        return oracle.exact_inputs(M, N, K, seed=case["seed"])
    rng = np.random.default_rng(case["seed"])
    A = oracle.round_bf16(rng.standard_normal((M, K), dtype=np.float32))
    Bt = oracle.round_bf16(rng.standard_normal((N, K), dtype=np.float32) * np.float32(case["std"]))
    return A, Bt


def input_digest(A: np.ndarray, Bt: np.ndarray) -> str:
    h = hashlib.sha256()
    h.update(np.ascontiguousarray(A).tobytes())
    h.update(np.ascontiguousarray(Bt).tobytes())
    return h.hexdigest()


def path(case) -> Path:
    return HERE / f"{case['name']}.npz"


def load(case):
    """Returns (A, Bt, C_reference) or raises if the fixture is missing or its
    inputs no longer regenerate identically."""
    z = np.load(path(case))
    A, Bt = inputs(case)
    if str(z["input_sha256"]) != input_digest(A, Bt):
        raise AssertionError(f"{case['name']}: regenerated inputs differ from the fixture's")
    return A, Bt, z["C"]
