"""The CPU oracle (oracle/gemm_oracle.c): conversions, known answers, an
independent cross-check, and the pin against the reference's own outputs
stored in tests/golden/ (produced by running the reference's v8 kernel,
tests/golden/make_golden.py)."""
import struct
from pathlib import Path

import numpy as np
import pytest

import oracle
from golden import cases


def f32_bits(x: float) -> int:
    return struct.unpack("<I", struct.pack("<f", x))[0]


def bits_f32(u: int) -> float:
    return struct.unpack("<f", struct.pack("<I", u))[0]


@pytest.mark.parametrize("x,expect", [
    (1.0, 0x3F80),
    (-2.0, 0xC000),
    (0.0, 0x0000),
    (-0.0, 0x8000),
    (bits_f32(0x3F808000), 0x3F80),   # tie, even kept part -> down
    (bits_f32(0x3F818000), 0x3F82),   # tie, odd kept part -> up
    (bits_f32(0x3F808001), 0x3F81),   # above the tie -> up
    (bits_f32(0x3F807FFF), 0x3F80),   # below the tie -> down
    (bits_f32(0x7F7FFFFF), 0x7F80),   # max float rounds to +inf
    (float("inf"), 0x7F80),
    (float("-inf"), 0xFF80),
    (bits_f32(0x00000001), 0x0000),   # smallest subnormal rounds to zero
    (bits_f32(0x00018000), 0x0002),   # subnormal tie, odd kept part -> up
])
def test_round_to_nearest_even(x, expect):
    assert int(oracle.round_bf16(np.array([x], np.float32))[0]) == expect


def test_round_nan_stays_nan():
    y = int(oracle.round_bf16(np.array([float("nan")], np.float32))[0])
    assert (y & 0x7F80) == 0x7F80 and (y & 0x7F) != 0


def test_round_matches_torch_on_random_values():
    import torch
    x = np.random.default_rng(3).standard_normal(100_000).astype(np.float32) * 1e3
    ours = oracle.round_bf16(x)
    theirs = torch.from_numpy(x).to(torch.bfloat16).view(torch.int16).numpy().view(np.uint16)
    assert np.array_equal(ours, theirs)


def test_bf16_roundtrip():
    u = np.arange(0, 1 << 16, dtype=np.uint16)
    f = oracle.bf16_to_f32(u)
    back = oracle.round_bf16(f)
    finite = (u & 0x7F80) != 0x7F80
    assert np.array_equal(back[finite], u[finite])


@pytest.mark.parametrize("M,N,K", [(1, 1, 1), (3, 5, 7), (17, 33, 65), (64, 64, 128),
                                    (5, 9, 1000)])
def test_exact_inputs_give_exact_results(M, N, K):
    A, B = oracle.exact_inputs(M, N, K, seed=M + N + K)
    exact = (oracle.bf16_to_f32(A).astype(np.float64) @ oracle.bf16_to_f32(B).astype(np.float64).T)
    C = oracle.gemm_f32(A, B)
    assert np.array_equal(C.astype(np.float64), exact)


def test_thread_count_does_not_change_bits():
    rng = np.random.default_rng(0)
    A = oracle.round_bf16(rng.standard_normal((37, 300)).astype(np.float32))
    B = oracle.round_bf16(rng.standard_normal((29, 300)).astype(np.float32))
    c1 = oracle.gemm_f32(A, B, nthreads=1)
    c7 = oracle.gemm_f32(A, B, nthreads=7)
    assert np.array_equal(c1.view(np.uint32), c7.view(np.uint32))


def test_matches_numpy_blas():
    rng = np.random.default_rng(1)
    A = oracle.round_bf16(rng.standard_normal((128, 512)).astype(np.float32))
    B = oracle.round_bf16(rng.standard_normal((96, 512)).astype(np.float32))
    C = oracle.gemm_f32(A, B)
    R = oracle.numpy_gemm_f32(A, B)
    scale = np.linalg.norm(oracle.bf16_to_f32(A), axis=1)[:, None] * \
        np.linalg.norm(oracle.bf16_to_f32(B), axis=1)[None, :]
    assert np.max(np.abs(C - R) / scale) < 1e-6


def test_empty_and_degenerate():
    A = np.zeros((0, 4), np.uint16)
    B = np.zeros((3, 4), np.uint16)
    assert oracle.gemm_f32(A, B).shape == (0, 3)
    A = np.zeros((2, 0), np.uint16)
    B = np.zeros((3, 0), np.uint16)
    assert np.array_equal(oracle.gemm_f32(A, B), np.zeros((2, 3), np.float32))


def golden_available():
    return [c for c in cases.CASES if cases.path(c).exists()]


def test_golden_fixtures_present():
    missing = [c["name"] for c in cases.CASES if not cases.path(c).exists()]
    assert not missing, f"missing golden fixtures {missing} (tests/golden/make_golden.py)"


@pytest.mark.parametrize("case", golden_available(), ids=lambda c: c["name"])
def test_oracle_matches_reference_golden(case):
    A, Bt, C_ref = cases.load(case)
    ours = oracle.gemm_bf16(A, Bt)
    if case["kind"] == "exact":
        # exact arithmetic: the reference kernel and the oracle agree bit for bit
        assert np.array_equal(ours, C_ref)
        return
    a = oracle.bf16_to_f32(ours).astype(np.float64)
    r = oracle.bf16_to_f32(C_ref).astype(np.float64)
    scale = np.linalg.norm(oracle.bf16_to_f32(A).astype(np.float64), axis=1)[:, None] * \
        np.linalg.norm(oracle.bf16_to_f32(Bt).astype(np.float64), axis=1)[None, :]
    assert np.max(np.abs(a - r) / scale) <= 1e-2
    assert np.linalg.norm(a - r) / np.linalg.norm(r) <= 5e-3
    # different summation orders: almost all elements within one bf16 ulp,
    # most of them identical
    same_sign = (ours >> 15) == (C_ref >> 15)
    ulp = np.abs(ours.astype(np.int32) - C_ref.astype(np.int32))
    assert np.mean(same_sign & (ulp <= 1)) > 0.99
    assert np.mean(ours == C_ref) > 0.9
