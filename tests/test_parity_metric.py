"""The tolerance metric itself, fed results with known injected errors."""
import math

import torch

from blackwell_gemm_b200 import parity


def operands(M=64, N=48, K=96, seed=0):
    g = torch.Generator().manual_seed(seed)
    A = torch.randn(M, K, generator=g).to(torch.bfloat16)
    Bt = torch.randn(N, K, generator=g).to(torch.bfloat16)
    R = A.float() @ Bt.float().T
    return A, Bt, R


def test_exact_result_scores_zero():
    A, Bt, R = operands()
    m = parity.metrics(R.clone(), R, A, Bt)
    assert m == {"max_scaled": 0.0, "rel_fro": 0.0}
    assert parity.passes(m)


def test_bf16_rounding_alone_passes():
    A, Bt, R = operands()
    m = parity.metrics(R.to(torch.bfloat16), R, A, Bt)
    assert 0 < m["max_scaled"] < 5e-3
    assert 0 < m["rel_fro"] < 3e-3
    assert parity.passes(m)


def test_single_large_error_fails_max_scaled():
    A, Bt, R = operands()
    C = R.clone()
    i, j = 5, 7
    C[i, j] += 0.02 * float(A[i].float().norm() * Bt[j].float().norm())
    m = parity.metrics(C, R, A, Bt)
    assert math.isclose(m["max_scaled"], 0.02, rel_tol=1e-3)
    assert not parity.passes(m)


def test_diffuse_error_fails_frobenius():
    A, Bt, R = operands()
    C = R * (1 + 6e-3)
    m = parity.metrics(C, R, A, Bt)
    assert math.isclose(m["rel_fro"], 6e-3, rel_tol=1e-3)
    assert not parity.passes(m)


def test_nan_and_inf_fail():
    A, Bt, R = operands()
    for bad in (float("nan"), float("inf")):
        C = R.clone()
        C[0, 0] = bad
        assert not parity.passes(parity.metrics(C, R, A, Bt))


def test_zero_rows_handled():
    A, Bt, R = operands()
    A[3] = 0
    R = A.float() @ Bt.float().T
    assert parity.passes(parity.metrics(R.clone(), R, A, Bt))
    C = R.clone()
    C[3, 0] = 1e-3   # nonzero output where the exact answer must be zero
    assert not parity.passes(parity.metrics(C, R, A, Bt))


def test_row_subset():
    A, Bt, R = operands()
    rows = torch.tensor([0, 9, 17])
    m = parity.metrics(R, R.index_select(0, rows), A, Bt, rows=rows)
    assert m["max_scaled"] == 0.0
