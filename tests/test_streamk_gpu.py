"""Stream-K tail of the 256 x 256 pair kernels (b200_gemm_set_stream_k).

Whole waves of tiles run as usual; the remaining tiles' (tile, K block)
items are split evenly over all pairs, and a tile cut between pairs is summed
by the pair holding its last K blocks from fp32 pieces the others leave in a
workspace.  Exact-arithmetic inputs must match the oracle bit for bit (every
partial sum is exact); random inputs meet the parity bar and agree with the
whole-tile kernel to within rounding of the different summation grouping.
Shapes include ragged edges, K of a single block (nothing to cut) and a lone
tail tile cut across every pair of the grid.
"""
import numpy as np
import pytest
import torch

import oracle
from blackwell_gemm_b200 import capi, parity, workloads

pytestmark = pytest.mark.gpu


@pytest.fixture(autouse=True)
def restore():
    yield
    capi.set_stream_k(1)
    capi.set_tuning(-1, 1, 0)
    capi.set_splits(0)
    assert capi.device_status(True) == 0


def gemm(A, Bt):
    M, K = A.shape
    N = Bt.shape[0]
    ldc = (N + 7) // 8 * 8
    C = torch.zeros(M, ldc, dtype=torch.bfloat16, device="cuda")
    st = capi.gemm_bf16(A.data_ptr(), Bt.data_ptr(), C.data_ptr(), M, N, K, K, K, ldc,
                        torch.cuda.current_stream().cuda_stream)
    assert st == capi.OK, capi.status_string(st)
    torch.cuda.synchronize()
    return C[:, :N]


def u16_dev(x):
    return torch.from_numpy(np.ascontiguousarray(x).view(np.int16)).cuda().view(torch.bfloat16)


def tail_applies(M, N, K, tile_n):
    s = capi.launch_shape(M, N, K)
    pairs = s["grid"] // 2
    return s["tiles"] > pairs and s["tiles"] % pairs != 0


# 256 x 256 pair tiles (the stream-K configurations), more than one wave of
# 74 pairs and not a whole number of waves
SHAPES = [(4096, 4096, 1024), (4100, 4000, 1000), (768, 6400, 8192), (2560, 8192, 64),
          (3072, 3072, 3072), (8192, 6144, 520)]


@pytest.mark.parametrize("slabs", [1, 2])
@pytest.mark.parametrize("idx", range(len(SHAPES)))
def test_exact_inputs_bit_exact(slabs, idx):
    M, N, K = SHAPES[idx]
    tile_n = 256
    capi.set_tuning(tile_n, slabs, 0)
    capi.set_splits(1)
    capi.set_stream_k(2)
    assert tail_applies(M, N, K, tile_n)
    A, Bt = oracle.exact_inputs(M, N, K, seed=idx + slabs)
    C = gemm(u16_dev(A), u16_dev(Bt))
    assert np.array_equal(C.contiguous().view(torch.int16).cpu().numpy().view(np.uint16),
                          oracle.gemm_bf16(A, Bt))


@pytest.mark.parametrize("idx", [0, 2])   # 2: a lone tail tile cut across every pair
def test_random_against_fp32_and_whole_tiles(idx):
    M, N, K = SHAPES[idx]
    tile_n = 256
    capi.set_tuning(tile_n, 1, 0)
    capi.set_splits(1)
    A, Bt = workloads.make_operands(M, N, K, seed=idx)
    capi.set_stream_k(2)
    C = gemm(A, Bt)
    capi.set_stream_k(0)
    W = gemm(A, Bt)
    m = parity.metrics(C, A.float() @ Bt.float().T, A, Bt)
    assert parity.passes(m), m
    diff = (C.float() - W.float()).abs()
    ulp = W.float().abs().clamp_min(1e-30) * 2.0 ** -7
    assert (diff <= ulp).float().mean().item() > 0.99


def test_graph_replays_and_concurrent_streams():
    """Outside capture each stream keeps its own epoch-numbered flags; a
    captured call clears flags of its own, so every replay is correct."""
    M, N, K = SHAPES[0]
    capi.set_tuning(256, 1, 0)
    capi.set_splits(1)
    capi.set_stream_k(2)
    A, Bt = workloads.make_operands(M, N, K, seed=21)
    ref = gemm(A, Bt).clone()
    C = torch.zeros(M, N, dtype=torch.bfloat16, device="cuda")

    def call():
        st = capi.gemm_bf16(A.data_ptr(), Bt.data_ptr(), C.data_ptr(), M, N, K, K, K, N,
                            torch.cuda.current_stream().cuda_stream)
        assert st == capi.OK

    side = torch.cuda.Stream()
    with torch.cuda.stream(side):
        call()
    torch.cuda.synchronize()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        call()
    for _ in range(3):
        C.zero_()
        g.replay()
        torch.cuda.synchronize()
        assert torch.equal(C.view(torch.int16), ref.view(torch.int16))
    outs = [torch.zeros(M, N, dtype=torch.bfloat16, device="cuda") for _ in range(2)]
    streams = [torch.cuda.Stream(), torch.cuda.Stream()]
    torch.cuda.synchronize()
    for _ in range(3):
        for s, out in zip(streams, outs):
            st = capi.gemm_bf16(A.data_ptr(), Bt.data_ptr(), out.data_ptr(), M, N, K, K, K, N,
                                s.cuda_stream)
            assert st == capi.OK
    torch.cuda.synchronize()
    for out in outs:
        assert torch.equal(out.view(torch.int16), ref.view(torch.int16))
