"""fp32-output GEMM (K-split partials), split-K with the fp32 workspace, the
fp32 -> bf16 cast, and the K-split / row-sharded multi-GPU paths.

Tolerances: bf16 outputs use the build's parity bar (norm-scaled max 1e-2,
relative Frobenius 5e-3); fp32 outputs differ from the fp32 oracle only by
summation order, so they are held to 1e-5 on both measures.  Exact-arithmetic
inputs must match bit for bit in every mode.
"""
import os
import socket

import numpy as np
import pytest
import torch

import oracle
from blackwell_gemm_b200 import capi, parity, workloads

pytestmark = pytest.mark.gpu


def dev(x: np.ndarray) -> torch.Tensor:
    return torch.from_numpy(np.ascontiguousarray(x).view(np.int16)).cuda().view(torch.bfloat16)


def bits(t: torch.Tensor) -> np.ndarray:
    return t.contiguous().view(torch.int16).cpu().numpy().view(np.uint16)


def f32out(A, Bt):
    M, K = A.shape
    N = Bt.shape[0]
    ldc = (N + 3) // 4 * 4
    C = torch.zeros(M, ldc, dtype=torch.float32, device="cuda")
    st = capi.gemm_bf16_f32out(A.data_ptr(), Bt.data_ptr(), C.data_ptr(), M, N, K, K, K, ldc,
                               torch.cuda.current_stream().cuda_stream)
    assert st == capi.OK, capi.status_string(st)
    torch.cuda.synchronize()
    return C[:, :N]


def bf16_gemm(A, Bt):
    M, K = A.shape
    N = Bt.shape[0]
    ldc = (N + 7) // 8 * 8
    C = torch.zeros(M, ldc, dtype=torch.bfloat16, device="cuda")
    st = capi.gemm_bf16(A.data_ptr(), Bt.data_ptr(), C.data_ptr(), M, N, K, K, K, ldc,
                        torch.cuda.current_stream().cuda_stream)
    assert st == capi.OK, capi.status_string(st)
    torch.cuda.synchronize()
    return C[:, :N]


@pytest.fixture(autouse=True)
def reset_splits():
    capi.set_splits(0)
    yield
    capi.set_splits(0)
    assert capi.device_status(True) == 0


@pytest.mark.parametrize("M,N,K", [(256, 256, 64), (300, 520, 1000), (7, 36, 72),
                                    (1024, 1024, 2048)])
def test_f32out_exact_and_random(M, N, K):
    A, Bt = oracle.exact_inputs(M, N, K, seed=K)
    C = f32out(dev(A), dev(Bt))
    assert np.array_equal(C.cpu().numpy(), oracle.gemm_f32(A, Bt))
    rng = np.random.default_rng(M + K)
    A = oracle.round_bf16(rng.standard_normal((M, K), dtype=np.float32))
    Bt = oracle.round_bf16(rng.standard_normal((N, K), dtype=np.float32))
    C = f32out(dev(A), dev(Bt)).cpu()
    m = parity.metrics(C, torch.from_numpy(oracle.gemm_f32(A, Bt)),
                       torch.from_numpy(oracle.bf16_to_f32(A)), torch.from_numpy(oracle.bf16_to_f32(Bt)))
    assert m["max_scaled"] <= 1e-5 and m["rel_fro"] <= 1e-5, m


@pytest.mark.parametrize("splits", [2, 3, 7, 64])
@pytest.mark.parametrize("M,N,K", [(16, 8192, 8192), (100, 520, 1000), (256, 256, 4096)])
def test_forced_split_k_exact_bits(M, N, K, splits):
    capi.set_splits(splits)
    A, Bt = oracle.exact_inputs(M, N, K, seed=splits)
    C = bf16_gemm(dev(A), dev(Bt))
    assert np.array_equal(bits(C), oracle.gemm_bf16(A, Bt))


@pytest.mark.parametrize("shape", workloads.SKINNY, ids=lambda s: "x".join(map(str, s)))
def test_auto_split_k_skinny_configs(shape):
    M, N, K = shape
    assert capi.get_splits(M, N, K) > 1            # skinny grids take the split-K path
    A, Bt = workloads.make_operands(M, N, K, seed=2, weight_std=0.02)
    C = bf16_gemm(A, Bt)
    m = parity.metrics(C, A.float() @ Bt.float().T, A, Bt)
    assert parity.passes(m), m


def test_split_choice():
    assert capi.get_splits(8192, 8192, 8192) == 1
    assert capi.get_splits(2048, 2048, 2048) == 1
    assert capi.get_splits(16, 8192, 8192) > 1
    assert capi.get_splits(16, 8192, 64) == 1        # nothing to split
    assert capi.get_splits(1024, 1024, 1024) == 1    # too shallow to pay for the extra passes
    capi.set_splits(1)
    assert capi.get_splits(16, 8192, 8192) == 1


def test_split_k_on_two_streams_concurrently():
    A1, B1 = workloads.make_operands(64, 4096, 8192, seed=3)
    A2, B2 = workloads.make_operands(64, 4096, 8192, seed=4)
    s1, s2 = torch.cuda.Stream(), torch.cuda.Stream()
    torch.cuda.synchronize()
    C1 = torch.empty(64, 4096, dtype=torch.bfloat16, device="cuda")
    C2 = torch.empty_like(C1)
    for s, A, Bt, C in ((s1, A1, B1, C1), (s2, A2, B2, C2)):
        assert capi.gemm_bf16(A.data_ptr(), Bt.data_ptr(), C.data_ptr(), 64, 4096, 8192, 8192,
                              8192, 4096, s.cuda_stream) == capi.OK
    torch.cuda.synchronize()
    for A, Bt, C in ((A1, B1, C1), (A2, B2, C2)):
        assert parity.passes(parity.metrics(C, A.float() @ Bt.float().T, A, Bt))


def test_cast_kernel_rounding():
    x = torch.randn(37, 203, device="cuda") * 1000
    W = torch.zeros(37, 204, device="cuda")
    W[:, :203] = x
    C = torch.zeros(37, 208, dtype=torch.bfloat16, device="cuda")
    assert capi.cast_f32_bf16(W.data_ptr(), 204, C.data_ptr(), 208, 37, 203, 0) == capi.OK
    torch.cuda.synchronize()
    assert torch.equal(C[:, :203].view(torch.int16), x.to(torch.bfloat16).view(torch.int16))
    assert capi.cast_f32_bf16(W.data_ptr() + 4, 204, C.data_ptr(), 208, 37, 203, 0) == \
        capi.ERR_ALIGNMENT


# ------------------------------------------------------------ multi-GPU
def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _ksplit_worker(rank, world, port, q):
    import traceback
    try:
        os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
        from datetime import timedelta
        import torch.distributed as dist
        from blackwell_gemm_b200 import distributed as bdist
        torch.cuda.set_device(rank)
        dev_ = torch.device("cuda", rank)
        dist.init_process_group("nccl", rank=rank, world_size=world,
                                timeout=timedelta(seconds=60), device_id=dev_)
        M, N, K = 1024, 768, 4096
        A, Bt = workloads.make_operands(M, N, K, seed=11, device=dev_)
        ks = bdist.k_slice(K, world, rank)
        rows = bdist.k_split_gemm(A[:, ks].contiguous(), Bt[:, ks].contiguous())
        rs = slice(rank * M // world, (rank + 1) * M // world)
        R = A[rs].float() @ Bt.float().T
        m = parity.metrics(rows, R, A[rs], Bt)
        rows2 = bdist.row_shard_gemm(A[rs].contiguous(), Bt)
        m2 = parity.metrics(rows2, R, A[rs], Bt)
        torch.cuda.synchronize()
        dist.barrier()
        dist.destroy_process_group()
        q.put((rank, parity.passes(m) and parity.passes(m2), str((m, m2))))
    except Exception:
        q.put((rank, False, traceback.format_exc()))


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs 2 GPUs")
def test_k_split_and_row_shard_on_two_gpus():
    import torch.multiprocessing as mp
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    ps = [ctx.Process(target=_ksplit_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in ps:
        p.start()
    res = [q.get(timeout=300) for _ in ps]
    for p in ps:
        p.join(timeout=60)
    assert all(ok for _, ok, _ in res), res


# ------------------------------------------------------- skinny-M kernel
SKINNY_MODES = {"auto": 1, "cluster": 2, "stream": 3, "pair_stream": 4, "pair_cluster": 5}


@pytest.fixture(params=list(SKINNY_MODES))
def skinny_mode(request):
    """The skinny path's kernels: chosen per shape, the cluster split-K kernel,
    the stream-K kernel, and the stream-K and cluster kernels on 2-CTA pairs,
    each forced for every M."""
    capi.set_skinny_mode(SKINNY_MODES[request.param])
    yield request.param
    capi.set_skinny_mode(1)


@pytest.mark.parametrize("M", [1, 16, 17, 32, 50, 64, 100, 128, 200, 256])
@pytest.mark.parametrize("N,K", [(1024, 512), (1032, 520), (8200, 1000), (2048, 8192)])
def test_skinny_kernel_exact_bits(M, N, K, skinny_mode):
    # M <= 256, N >= 1024, K >= 512 take the C^T = B A^T kernels
    A, Bt = oracle.exact_inputs(M, N, K, seed=M)
    C = bf16_gemm(dev(A), dev(Bt))
    assert np.array_equal(bits(C), oracle.gemm_bf16(A, Bt))


@pytest.mark.parametrize("M,N,K", [(16, 8192, 8192), (100, 3000, 4000), (256, 1024, 65536)])
def test_skinny_kernels_random(M, N, K, skinny_mode):
    A, Bt = workloads.make_operands(M, N, K, seed=M + K, weight_std=0.02)
    C = bf16_gemm(A, Bt)
    assert parity.passes(parity.metrics(C, A.float() @ Bt.float().T, A, Bt))


@pytest.mark.parametrize("splits", [1, 5, 64])
def test_skinny_kernel_forced_splits_random(splits):
    capi.set_splits(splits)
    M, N, K = 48, 4096, 8192
    A, Bt = workloads.make_operands(M, N, K, seed=splits, weight_std=0.02)
    C = bf16_gemm(A, Bt)
    assert parity.passes(parity.metrics(C, A.float() @ Bt.float().T, A, Bt))


@pytest.mark.parametrize("M,N,K", [(256, 8192, 2048), (200, 16384, 1024), (256, 4096, 14336)])
def test_skinny_auto_takes_cluster_kernels_exact_bits(M, N, K):
    """Per shape, above M = 128: the cluster kernel on 2-CTA pairs (two
    slices at 8192 and one at 16384 rows of B) or on single CTAs (4096 rows
    and K = 14336, where pairs would fill fewer SMs): exact results there."""
    capi.set_skinny_mode(1)
    capi.set_splits(0)
    A, Bt = oracle.exact_inputs(M, N, K, seed=M + N)
    C = bf16_gemm(dev(A), dev(Bt))
    assert np.array_equal(bits(C), oracle.gemm_bf16(A, Bt))
    assert capi.device_status(True) == 0


@pytest.mark.parametrize("slices", [1, 2, 4])
@pytest.mark.parametrize("M,N,K", [(64, 8192, 2048), (200, 4096, 4096), (40, 28672, 1024),
                                   (256, 1280, 3008), (48, 2048, 520)])
def test_skinny_pair_cluster_slices_exact_bits(M, N, K, slices):
    """The cluster kernel on 2-CTA pairs with K split over 1, 2 and 4 pairs
    (clusters of 2, 4 and 8 CTAs): whole and ragged pair blocks, grids of
    more clusters than fit at once, and a slice left without K blocks (K =
    520: 9 blocks over 4 slices of 3)."""
    capi.set_skinny_mode(5)
    capi.set_splits(slices)
    try:
        A, Bt = oracle.exact_inputs(M, N, K, seed=M + K)
        C = bf16_gemm(dev(A), dev(Bt))
        assert np.array_equal(bits(C), oracle.gemm_bf16(A, Bt))
    finally:
        capi.set_skinny_mode(1)
        capi.set_splits(0)


@pytest.mark.parametrize("mode", [3, 4], ids=["cta", "pair"])
@pytest.mark.parametrize("M,N,K", [(128, 24576, 1024), (128, 12288, 1024), (100, 4096, 2048),
                                   (256, 8192, 1024), (64, 1024, 8192), (32, 2048, 16384)])
def test_skinny_stream_k_fixup_exact_bits(M, N, K, mode):
    """The stream-K skinny kernel (one CTA, or 2-CTA pairs) over its fix-up
    structures: blocks of B split between two workers (the second finishes
    the block alone), between three to six (every contributor finishes a
    share), mixtures of both, and about twenty contributors to a block (more
    than its pieces, so some contributors finish nothing)."""
    capi.set_skinny_mode(mode)
    try:
        A, Bt = oracle.exact_inputs(M, N, K, seed=M + N)
        C = bf16_gemm(dev(A), dev(Bt))
        assert np.array_equal(bits(C), oracle.gemm_bf16(A, Bt))
    finally:
        capi.set_skinny_mode(1)


@pytest.mark.parametrize("M", [48, 128])
def test_skinny_stream_k_graph_replays_and_streams(M):
    """The stream-K skinny kernel (16 < M <= 128 by default) raises per-stream
    epoch flags outside capture and clears its own flags when captured."""
    N, K = 4096, 8192
    A, Bt = workloads.make_operands(M, N, K, seed=31, weight_std=0.02)
    ref = bf16_gemm(A, Bt).clone()
    C = torch.zeros(M, N, dtype=torch.bfloat16, device="cuda")

    def call(out, stream):
        assert capi.gemm_bf16(A.data_ptr(), Bt.data_ptr(), out.data_ptr(), M, N, K, K, K, N,
                              stream) == capi.OK

    side = torch.cuda.Stream()
    side.wait_stream(torch.cuda.current_stream())  # C's zero fill
    call(C, side.cuda_stream)
    torch.cuda.synchronize()
    assert torch.equal(C.view(torch.int16), ref.view(torch.int16))
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        call(C, torch.cuda.current_stream().cuda_stream)
    for _ in range(3):
        C.zero_()
        g.replay()
        torch.cuda.synchronize()
        assert torch.equal(C.view(torch.int16), ref.view(torch.int16))
    outs = [torch.zeros_like(C) for _ in range(2)]
    streams = [torch.cuda.Stream(), torch.cuda.Stream()]
    for st in streams:
        st.wait_stream(torch.cuda.current_stream())
    for _ in range(3):
        for s, out in zip(streams, outs):
            call(out, s.cuda_stream)
    torch.cuda.synchronize()
    for out in outs:
        assert torch.equal(out.view(torch.int16), ref.view(torch.int16))


@pytest.mark.parametrize("tiles", [1, 2])
@pytest.mark.parametrize("M,N,K", [(1, 1032, 520), (17, 8200, 1000), (64, 1024, 8192),
                                   (100, 4096, 2048), (128, 24576, 1024), (128, 8192, 8192),
                                   (128, 1160, 4096)])
def test_skinny_stream_k_tiles_exact_bits(M, N, K, tiles):
    """The stream-K skinny kernel with tiles of one or two 128-row blocks of
    B (two blocks share each A slab): exact results whatever the split of a
    tile between CTAs, including a last tile whose second block lies partly
    or wholly past N."""
    capi.set_skinny_mode(3)
    capi.set_skinny_tiles(tiles)
    try:
        A, Bt = oracle.exact_inputs(M, N, K, seed=M + N + tiles)
        C = bf16_gemm(dev(A), dev(Bt))
        assert np.array_equal(bits(C), oracle.gemm_bf16(A, Bt))
        assert capi.device_status(True) == 0
    finally:
        capi.set_skinny_mode(1)
        capi.set_skinny_tiles(0)


@pytest.mark.parametrize("M,N,K", [(200, 24576, 1024), (256, 40960, 1024)])
def test_skinny_wide_n_takes_pair_stream_k_exact_bits(M, N, K):
    """Above M = 128 with B too wide for one wave of cluster kernels and an
    fp32 workspace of 16 MB or more, the per-shape choice runs the stream-K
    kernel on 2-CTA pairs: exact results there."""
    capi.set_skinny_mode(1)
    A, Bt = oracle.exact_inputs(M, N, K, seed=M + 3)
    C = bf16_gemm(dev(A), dev(Bt))
    assert np.array_equal(bits(C), oracle.gemm_bf16(A, Bt))
    assert capi.device_status(True) == 0
