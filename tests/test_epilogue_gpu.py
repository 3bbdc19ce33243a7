"""Fused epilogue C = round(alpha A B^T + bias + beta R) on every path the
launcher can take (256-wide pair kernel, split-K and skinny rounding passes),
with exact-arithmetic known answers (bit-exact) and random inputs within the
parity tolerance."""
import numpy as np
import pytest
import torch

import oracle
import blackwell_gemm_b200 as bg
from blackwell_gemm_b200 import capi, parity

pytestmark = pytest.mark.gpu


def dev(x):
    return torch.from_numpy(np.ascontiguousarray(x).view(np.int16)).cuda().view(torch.bfloat16)


def bits(t):
    return t.contiguous().view(torch.int16).cpu().numpy().view(np.uint16)


SHAPES = {
    "pair_kernel": (1024, 768, 512),
    "ragged_n": (300, 1000, 200),
    "split_k": (512, 512, 8192),
    "skinny": (16, 8192, 1024),
    "skinny_ragged": (100, 4104, 2048),
}


@pytest.mark.parametrize("alpha,beta", [(1.0, 1.0), (0.5, -1.0), (2.0, 0.5)])
@pytest.mark.parametrize("path", list(SHAPES))
def test_epilogue_exact_bits(path, alpha, beta):
    M, N, K = SHAPES[path]
    A, Bt = oracle.exact_inputs(M, N, K, seed=K)
    rng = np.random.default_rng(N)
    bias = oracle.round_bf16(rng.integers(-8, 9, N).astype(np.float32) / 4)
    R = oracle.round_bf16(rng.integers(-8, 9, (M, N)).astype(np.float32) / 4)
    C = bg.matmul_b200_epilogue(dev(A), dev(Bt).T, alpha=alpha, bias=dev(bias), beta=beta,
                                residual=dev(R))
    torch.cuda.synchronize()
    # every term is a small multiple of 1/16: the fp32 arithmetic is exact
    want = (np.float32(alpha) * oracle.gemm_f32(A, Bt) + oracle.bf16_to_f32(bias)[None, :]
            + np.float32(beta) * oracle.bf16_to_f32(R))
    assert np.array_equal(bits(C), oracle.round_bf16(want.astype(np.float32)))
    assert capi.device_status(True) == 0


@pytest.mark.parametrize("path", list(SHAPES))
def test_epilogue_random_within_tolerance(path):
    M, N, K = SHAPES[path]
    g = torch.Generator(device="cuda").manual_seed(M + N)
    A = torch.randn(M, K, device="cuda", generator=g).bfloat16()
    Bt = (torch.randn(N, K, device="cuda", generator=g) * 0.02).bfloat16()
    bias = torch.randn(N, device="cuda", generator=g).bfloat16()
    R = torch.randn(M, N, device="cuda", generator=g).bfloat16()
    C = bg.matmul_b200_epilogue(A, Bt.T, alpha=0.7, bias=bias, beta=0.3, residual=R)
    ref = 0.7 * (A.float() @ Bt.float().T) + bias.float()[None, :] + 0.3 * R.float()
    # per element: one bf16 rounding of the total (half an ulp, 2^-9 relative)
    # plus the GEMM term's norm-scaled parity bound
    gemm_bound = parity.MAX_SCALED_TOL * 0.7 * (A.float().norm(dim=1)[:, None] *
                                               Bt.float().norm(dim=1)[None, :])
    err = (C.float() - ref).abs()
    assert bool((err <= 2.0 ** -9 * ref.abs() + gemm_bound).all())
    rel_fro = float((C.float() - ref).norm() / ref.norm())
    assert rel_fro <= parity.REL_FRO_TOL, rel_fro


def test_epilogue_residual_in_place_and_optional_terms():
    M, N, K = 512, 768, 1024
    A, Bt = oracle.exact_inputs(M, N, K, seed=3)
    R = oracle.round_bf16(np.random.default_rng(0).integers(-4, 5, (M, N)).astype(np.float32) / 4)
    Rd = dev(R)
    C = bg.matmul_b200_epilogue(dev(A), dev(Bt).T, residual=Rd)   # beta defaults to 1
    want = oracle.gemm_f32(A, Bt) + oracle.bf16_to_f32(R)
    assert np.array_equal(bits(C), oracle.round_bf16(want))
    # residual aliasing the output through the C ABI: C = A B^T + C
    Cbuf = Rd.clone()
    st = capi.gemm_bf16_epilogue(dev(A).data_ptr(), dev(Bt).data_ptr(), Cbuf.data_ptr(), M, N, K,
                                 K, K, N, 1.0, 0, 1.0, Cbuf.data_ptr(), N, 0)
    assert st == capi.OK
    torch.cuda.synchronize()
    assert np.array_equal(bits(Cbuf), oracle.round_bf16(want))
    # no optional terms = the plain GEMM
    C0 = bg.matmul_b200_epilogue(dev(A), dev(Bt).T)
    assert np.array_equal(bits(C0), oracle.gemm_bf16(A, Bt))


def test_epilogue_rejects_misaligned_bias():
    A = torch.zeros(256, 64, dtype=torch.bfloat16, device="cuda")
    Bt = torch.zeros(256, 64, dtype=torch.bfloat16, device="cuda")
    C = torch.empty(256, 256, dtype=torch.bfloat16, device="cuda")
    b = torch.zeros(264, dtype=torch.bfloat16, device="cuda")
    st = capi.gemm_bf16_epilogue(A.data_ptr(), Bt.data_ptr(), C.data_ptr(), 256, 256, 64, 64, 64,
                                 256, 1.0, b.data_ptr() + 2, 0.0, 0, 0, 0)
    assert st == capi.ERR_ALIGNMENT
