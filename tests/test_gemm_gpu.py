"""GPU parity tests of the sm_100a GEMM, through the C ABI (libb200gemm.so)
and through the reference-compatible torch binding.

Checkers: the CPU oracle (oracle/gemm_oracle.c) at sizes it finishes in
seconds, the golden vectors produced by the reference's own v8 kernel
(tests/golden), bit-exact known answers (inputs whose fp32 accumulation is
exact in any order), and at full configuration sizes a GPU fp32 GEMM of the
same bf16 inputs on sampled rows.  Tolerance (the build's parity bar):
max |C - R| / (|A_i| |B_j|) <= 1e-2 and ||C - R||_F / ||R||_F <= 5e-3.
"""
import numpy as np
import pytest
import torch

import oracle
from blackwell_gemm_b200 import capi, parity, workloads
from golden import cases

pytestmark = pytest.mark.gpu

TOL_MAX_SCALED = 1e-2
TOL_REL_FRO = 5e-3


def u16_to_dev(x: np.ndarray) -> torch.Tensor:
    return torch.from_numpy(np.ascontiguousarray(x).view(np.int16)).cuda().view(torch.bfloat16)


def dev_to_u16(t: torch.Tensor) -> np.ndarray:
    return t.contiguous().view(torch.int16).cpu().numpy().view(np.uint16)


def capi_gemm(A: torch.Tensor, Bt: torch.Tensor, C: torch.Tensor | None = None, stream=None):
    """C = A Bt^T through the C ABI; C may be wider than N (padded rows)."""
    M, K = A.shape
    N = Bt.shape[0]
    if C is None:
        C = torch.empty(M, N, dtype=torch.bfloat16, device="cuda")
    s = stream.cuda_stream if stream is not None else torch.cuda.current_stream().cuda_stream
    st = capi.gemm_bf16(A.data_ptr(), Bt.data_ptr(), C.data_ptr(), M, N, K, A.stride(0),
                        Bt.stride(0), C.stride(0), s)
    assert st == capi.OK, capi.status_string(st)
    return C


def ulp_close_fraction(a: np.ndarray, b: np.ndarray) -> float:
    """Fraction of bf16 elements (bit patterns) equal or one ulp apart."""
    same_sign = (a >> 15) == (b >> 15)
    d = np.abs(a.astype(np.int32) - b.astype(np.int32))
    return float(np.mean(same_sign & (d <= 1)))


def assert_no_device_error():
    assert capi.device_status(True) == 0


def within_tol(C, R, A, Bt, rows=None):
    m = parity.metrics(C, R, A, Bt, rows=rows)
    assert m["max_scaled"] <= TOL_MAX_SCALED and m["rel_fro"] <= TOL_REL_FRO, m
    return m


CONFIGS = {"n256_bk64": (256, 1), "n256_bk128": (256, 2), "n512_bk64": (512, 1),
           "n128_bk64": (128, 1), "n64_bk64": (64, 1)}


@pytest.fixture(autouse=True, params=list(CONFIGS), ids=list(CONFIGS))
def kernel_config(request):
    """Every test runs on every kernel configuration (pair-tile width and
    stage depth), forced regardless of the per-shape choice."""
    tile_n, slabs = CONFIGS[request.param]
    capi.set_tuning(tile_n, slabs, 0)
    yield request.param
    capi.set_tuning(-1, 1, 0)


# ------------------------------------------------------------ small shapes
SMALL = [(256, 256, 64), (512, 256, 128), (256, 512, 1024), (1, 8, 8), (7, 24, 40),
         (129, 264, 72), (300, 520, 200), (1000, 8, 16), (8, 1000, 520), (1024, 1024, 1024)]


@pytest.mark.parametrize("M,N,K", SMALL)
def test_random_inputs_match_cpu_oracle(M, N, K):
    rng = np.random.default_rng(M * 31 + N * 7 + K)
    A = oracle.round_bf16(rng.standard_normal((M, K), dtype=np.float32))
    Bt = oracle.round_bf16(rng.standard_normal((N, K), dtype=np.float32))
    C = capi_gemm(u16_to_dev(A), u16_to_dev(Bt))
    torch.cuda.synchronize()
    assert_no_device_error()
    R = torch.from_numpy(oracle.gemm_f32(A, Bt))
    within_tol(C.cpu(), R, torch.from_numpy(oracle.bf16_to_f32(A)),
               torch.from_numpy(oracle.bf16_to_f32(Bt)))
    # different fp32 summation orders, one bf16 rounding each: almost every
    # element is within one bf16 ulp of the oracle's bits (outputs near zero
    # after cancellation may differ by more ulps while staying inside the
    # norm-scaled bound above)
    assert ulp_close_fraction(dev_to_u16(C), oracle.round_bf16(oracle.gemm_f32(A, Bt))) > 0.99


@pytest.mark.parametrize("M,N,K", [(256, 256, 64), (384, 640, 192), (33, 17, 264),
                                    (513, 257, 1000), (1024, 1024, 4096)])
def test_exact_inputs_bit_exact(M, N, K):
    A, Bt = oracle.exact_inputs(M, N, K, seed=K)
    ldc = (N + 7) // 8 * 8                 # C rows must start 16-byte aligned
    Cbuf = torch.zeros(M, ldc, dtype=torch.bfloat16, device="cuda")
    C = capi_gemm(u16_to_dev(A), u16_to_dev(Bt), Cbuf)[:, :N]
    torch.cuda.synchronize()
    assert np.array_equal(dev_to_u16(C), oracle.gemm_bf16(A, Bt))


@pytest.mark.parametrize("case", cases.CASES, ids=lambda c: c["name"])
def test_reference_golden_vectors(case):
    A, Bt, C_ref = cases.load(case)
    C = dev_to_u16(capi_gemm(u16_to_dev(A), u16_to_dev(Bt)))
    if case["kind"] == "exact":
        assert np.array_equal(C, C_ref)
        return
    within_tol(torch.from_numpy(oracle.bf16_to_f32(C)), torch.from_numpy(oracle.bf16_to_f32(C_ref)),
               torch.from_numpy(oracle.bf16_to_f32(A)), torch.from_numpy(oracle.bf16_to_f32(Bt)))
    assert ulp_close_fraction(C, C_ref) > 0.99


# ------------------------------------------------------- full-size configs
def full_size_check(M, N, K, std, seed=0, nrows=256):
    A, Bt = workloads.make_operands(M, N, K, seed=seed, weight_std=std)
    C = capi_gemm(A, Bt)
    torch.cuda.synchronize()
    assert_no_device_error()
    g = torch.Generator().manual_seed(seed + 1)
    rows = torch.randperm(M, generator=g)[:nrows].cuda()
    rows = torch.cat([rows, torch.tensor([0, M - 1], device="cuda")])
    R = A.index_select(0, rows).float() @ Bt.float().T
    return within_tol(C, R, A, Bt, rows=rows)


@pytest.mark.parametrize("shape", workloads.SQUARE + workloads.PROJECTION + workloads.SKINNY,
                         ids=lambda s: "x".join(map(str, s)))
def test_configuration_shapes(shape):
    M, N, K = shape
    std = 0.02 if shape in workloads.PROJECTION + workloads.SKINNY else 1.0
    full_size_check(M, N, K, std)


@pytest.mark.parametrize("shape", [workloads.M_SHARD, workloads.K_SPLIT],
                         ids=["m_shard_131072x8192x8192", "k_split_8192x8192x131072"])
def test_multi_gpu_shapes_on_one_gpu(shape):
    full_size_check(*shape, std=1.0, nrows=128)


@pytest.mark.parametrize("M,N,K", [(8192, 8192, 8192), (4096, 28672, 4096)])
def test_full_size_exact_inputs_bit_exact(M, N, K):
    # entries in {-4..4}/4: every fp32 partial sum is exact, so the fp32 GEMM
    # on the GPU is exact too and the bf16 results must agree bit for bit
    g = torch.Generator(device="cuda").manual_seed(7)
    A = (torch.randint(-4, 5, (M, K), generator=g, device="cuda").float() / 4).bfloat16()
    Bt = (torch.randint(-4, 5, (N, K), generator=g, device="cuda").float() / 4).bfloat16()
    C = capi_gemm(A, Bt)
    prev = torch.backends.cuda.matmul.allow_tf32
    torch.backends.cuda.matmul.allow_tf32 = False
    try:
        R = (A.float() @ Bt.float().T).bfloat16()
    finally:
        torch.backends.cuda.matmul.allow_tf32 = prev
    assert torch.equal(C.view(torch.int16), R.view(torch.int16))


def test_against_cublas_and_deterministic():
    A, Bt = workloads.make_operands(4096, 4096, 4096, seed=3)
    C1 = capi_gemm(A, Bt)
    C2 = capi_gemm(A, Bt)
    ref = torch.matmul(A, Bt.T)
    torch.cuda.synchronize()
    assert torch.equal(C1.view(torch.int16), C2.view(torch.int16))   # same bits every call
    within_tol(C1.float(), ref.float(), A, Bt)


def test_reference_kernel_cross_check():
    try:
        oracle.ref_lib()
    except ImportError:
        pytest.skip("reference build (oracle/_ref) not present")
    for M, N, K in [(1024, 1024, 1024), (2048, 4096, 512)]:
        A, Bt = workloads.make_operands(M, N, K, seed=5)
        C = capi_gemm(A, Bt)
        Cr = torch.empty_like(C)
        oracle.ref_gemm("v8", A.data_ptr(), Bt.data_ptr(), Cr.data_ptr(), M, N, K)
        torch.cuda.synchronize()
        within_tol(C.float(), Cr.float(), A, Bt)
        diff = (C.view(torch.int16).int() - Cr.view(torch.int16).int()).abs()
        assert (diff <= 1).float().mean() > 0.999


# ----------------------------------------------------------- edge cases
def test_empty_and_zero_k():
    for M, N in [(0, 16), (16, 0)]:
        A = torch.empty(M, 8, dtype=torch.bfloat16, device="cuda")
        Bt = torch.empty(N, 8, dtype=torch.bfloat16, device="cuda")
        C = torch.empty(M, N, dtype=torch.bfloat16, device="cuda")
        assert capi.gemm_bf16(A.data_ptr(), Bt.data_ptr(), C.data_ptr(), M, N, 8, 8, 8, 8, 0) == 0
    C = torch.full((24, 40), 3.0, dtype=torch.bfloat16, device="cuda")
    assert capi.gemm_bf16(0, 0, C.data_ptr(), 24, 40, 0, 8, 8, 40, 0) == 0
    torch.cuda.synchronize()
    assert torch.count_nonzero(C.float()) == 0


def test_strided_operands_via_leading_dimensions():
    M, N, K = 300, 136, 200
    Ab = torch.randn(M, K + 24, device="cuda").bfloat16()
    Bb = torch.randn(N, K + 56, device="cuda").bfloat16()
    A, Bt = Ab[:, :K], Bb[:, :K]
    Cb = torch.zeros(M, N + 8, dtype=torch.bfloat16, device="cuda")
    st = capi.gemm_bf16(A.data_ptr(), Bt.data_ptr(), Cb.data_ptr(), M, N, K, K + 24, K + 56,
                        N + 8, 0)
    assert st == 0
    torch.cuda.synchronize()
    within_tol(Cb[:, :N].float(), A.float() @ Bt.float().T, A, Bt)
    assert torch.count_nonzero(Cb[:, N:].float()) == 0          # padding untouched


def test_misaligned_operands_rejected():
    buf = torch.zeros(64 * 64 + 8, dtype=torch.bfloat16, device="cuda")
    p = buf.data_ptr()
    assert capi.gemm_bf16(p + 2, p, p, 8, 8, 8, 8, 8, 8, 0) == capi.ERR_ALIGNMENT
    assert capi.gemm_bf16(p, p, p, 8, 8, 12, 12, 16, 8, 0) == capi.ERR_ALIGNMENT


def test_runs_on_caller_stream():
    s = torch.cuda.Stream()
    A, Bt = workloads.make_operands(512, 768, 256, seed=9)
    torch.cuda.synchronize()
    with torch.cuda.stream(s):
        C = capi_gemm(A, Bt, stream=s)
    s.synchronize()
    within_tol(C.float(), A.float() @ Bt.float().T, A, Bt)


# ------------------------------------------------------ failure detection
def test_bounded_wait_records_timeout_and_context_survives():
    assert capi.device_status(True) == 0
    assert capi.wait_probe(50_000_000) == capi.OK      # 50 ms wait nothing releases
    torch.cuda.synchronize()
    assert capi.device_status(True) == 0x1006
    assert capi.device_status(True) == 0               # cleared
    A, Bt = workloads.make_operands(256, 256, 128, seed=2)
    C = capi_gemm(A, Bt)
    torch.cuda.synchronize()
    within_tol(C.float(), A.float() @ Bt.float().T, A, Bt)


# ------------------------------------------------ reference-shaped binding
def test_torch_binding_reference_layout():
    import blackwell_gemm_b200 as bg
    A, Bt = workloads.make_operands(1024, 768, 512, seed=4)
    C = bg.module.matmul_b200(A, Bt.T)                 # B = randn(N, K).T as the harness
    assert C.shape == (1024, 768) and C.dtype == torch.bfloat16 and C.is_contiguous()
    within_tol(C.float(), A.float() @ Bt.float().T, A, Bt)


@pytest.mark.parametrize("layout", ["B_row_major_KN", "A_transposed_view", "odd_N", "odd_K"])
def test_torch_binding_other_layouts(layout):
    import blackwell_gemm_b200 as bg
    M, N, K = 200, 136, 96
    if layout == "odd_N":
        N = 131
    if layout == "odd_K":
        K = 99
    A = torch.randn(M, K, device="cuda").bfloat16()
    B = torch.randn(K, N, device="cuda").bfloat16()        # contiguous (K, N)
    if layout == "A_transposed_view":
        A = torch.randn(K, M, device="cuda").bfloat16().T
    C = bg.matmul_b200(A, B)
    assert C.shape == (M, N) and C.is_contiguous()
    within_tol(C.float(), A.float() @ B.float(), A, B.T)


def test_torch_binding_rejects_bad_inputs():
    import blackwell_gemm_b200 as bg
    a = torch.randn(16, 16, device="cuda").bfloat16()
    with pytest.raises(RuntimeError, match="bfloat16"):
        bg.matmul_b200(a.float(), a)
    with pytest.raises(RuntimeError, match="inner dimensions"):
        bg.matmul_b200(a, torch.randn(8, 16, device="cuda").bfloat16())
    with pytest.raises(RuntimeError, match="CUDA"):
        bg.matmul_b200(a, a.cpu())


def test_profiler_variant_matches_and_records():
    import blackwell_gemm_b200 as bg
    from blackwell_gemm_b200 import profiler
    M, N, K = 1024, 1024, 2048
    A, Bt = workloads.make_operands(M, N, K, seed=6)
    buf = profiler.alloc(M, N, K, 256)
    C = bg.profile_matmul_b200(A, Bt.T, buf, 256)
    capi.set_splits(1)          # the profiled kernel never splits K; compare like with like
    try:
        C0 = bg.matmul_b200(A, Bt.T)
        torch.cuda.synchronize()
    finally:
        capi.set_splits(0)
    assert torch.equal(C.view(torch.int16), C0.view(torch.int16))
    warps = profiler.warps_per_cta(M, N, K)
    ev = list(profiler.decode(buf, warps))
    tags = {e["tag"] for e in ev}
    assert {"Setup", "IssueTMA", "IssueMMA", "Epilogue"} <= tags
    assert all(e["dur_ns"] >= 0 for e in ev)
    s = profiler.summary(buf, warps)
    assert s["span_ns"] > 0
    # a tiny capacity must truncate, never overrun
    buf2 = profiler.alloc(M, N, K, 2)
    bg.profile_matmul_b200(A, Bt.T, buf2, 2)
    torch.cuda.synchronize()
    assert int(buf2[:, 0].max()) <= 2
