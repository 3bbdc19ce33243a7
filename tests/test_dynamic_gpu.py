"""Dynamic dealing of whole tiles (b200_gemm_set_dynamic(1)): the pair
leader's producer takes tickets from a per-stream device counter and
publishes each tile in a shared-memory ring that every role of the pair
reads.  Only the order in which pairs take tiles changes, not any tile's
arithmetic, so every result must equal the static deal's bit for bit (for
split-K, whose slices meet in an fp32 sum in completion order, on exact
inputs): on
whole-wave and ragged grids, every tile width, split-K, stream-K tails, the
fused K-split on one rank, the allocation-free entry point, several calls in
a row (the counters must be back at zero after each launch), two streams at
once, and a captured CUDA graph replayed several times.
"""
import pytest
import torch

from blackwell_gemm_b200 import capi, workloads

pytestmark = pytest.mark.gpu


@pytest.fixture(autouse=True)
def restore_dealing():
    yield
    capi.set_dynamic(0)
    capi.set_tuning(-1, 1, 0)
    capi.set_splits(0)


def call(fn, A, Bt, C, stream=None):
    M, K = A.shape
    N = Bt.shape[0]
    s = (stream or torch.cuda.current_stream()).cuda_stream
    st = fn(A.data_ptr(), Bt.data_ptr(), C.data_ptr(), M, N, K, K, K, C.stride(0), s)
    assert st == capi.OK, capi.status_string(st)


def bits(C):
    return C.view(torch.int16)


@pytest.mark.parametrize("M,N,K,tile_n", [
    (4096, 4096, 1024, 256), (4096, 4096, 1024, 512), (2048, 2048, 2048, 128),
    (2048, 2048, 1024, 64), (3000, 5000, 704, -1), (8192, 6144, 4096, -1),
    (256, 2048, 8192, -1)])
def test_dynamic_equals_static(M, N, K, tile_n):
    if capi.get_splits(M, N, K) > 1:
        # split-K adds slices into an fp32 workspace in whatever order they
        # finish: exact inputs (entries in {-4..4}/4, every partial sum exact)
        # make the result unique, so a lost or repeated unit still shows
        g = torch.Generator(device="cuda").manual_seed(M + N + K)
        A = (torch.randint(-4, 5, (M, K), generator=g, device="cuda").float() / 4).bfloat16()
        Bt = (torch.randint(-4, 5, (N, K), generator=g, device="cuda").float() / 4).bfloat16()
    else:
        A, Bt = workloads.make_operands(M, N, K, seed=M ^ N ^ K)
    ldc = (N + 7) // 8 * 8
    capi.set_tuning(tile_n, 1, 0)
    ref = torch.zeros(M, ldc, dtype=torch.bfloat16, device="cuda")
    capi.set_dynamic(0)
    call(capi.gemm_bf16, A, Bt, ref)
    capi.set_dynamic(1)
    for _ in range(3):
        C = torch.zeros_like(ref)
        call(capi.gemm_bf16, A, Bt, C)
        torch.cuda.synchronize()
        assert torch.equal(bits(C), bits(ref))
    assert capi.device_status(True) == 0


def test_dynamic_noalloc_and_two_streams():
    M, N, K = 4096, 4096, 1024
    A, Bt = workloads.make_operands(M, N, K, seed=3)
    # the allocation-free path runs whole tiles (no stream-K tail): its
    # static deal is the reference for its dynamic one
    ref_na = torch.zeros(M, N, dtype=torch.bfloat16, device="cuda")
    call(capi.gemm_bf16_noalloc, A, Bt, ref_na)
    capi.set_dynamic(1)
    for _ in range(2):
        C = torch.zeros_like(ref_na)
        call(capi.gemm_bf16_noalloc, A, Bt, C)
        torch.cuda.synchronize()
        assert torch.equal(bits(C), bits(ref_na))
    assert capi.noalloc_status(True) == 0
    capi.set_dynamic(0)
    ref = torch.zeros(M, N, dtype=torch.bfloat16, device="cuda")
    call(capi.gemm_bf16, A, Bt, ref)
    capi.set_dynamic(1)
    # two streams at once: each has its own counters
    s1, s2 = torch.cuda.Stream(), torch.cuda.Stream()
    outs = [torch.zeros_like(ref) for _ in range(4)]
    torch.cuda.synchronize()
    for i, C in enumerate(outs):
        call(capi.gemm_bf16, A, Bt, C, s1 if i % 2 == 0 else s2)
    torch.cuda.synchronize()
    for C in outs:
        assert torch.equal(bits(C), bits(ref))
    assert capi.device_status(True) == 0


def test_dynamic_under_graph_capture():
    M, N, K = 4096, 4096, 1024
    A, Bt = workloads.make_operands(M, N, K, seed=4)
    ref = torch.zeros(M, N, dtype=torch.bfloat16, device="cuda")
    call(capi.gemm_bf16, A, Bt, ref)
    capi.set_dynamic(1)
    C = torch.zeros_like(ref)
    s = torch.cuda.Stream()
    call(capi.gemm_bf16, A, Bt, C, s)        # set-up outside the capture
    torch.cuda.synchronize()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g, stream=s):
        call(capi.gemm_bf16, A, Bt, C, s)
    for _ in range(3):
        C.zero_()
        g.replay()
        torch.cuda.synchronize()
        assert torch.equal(bits(C), bits(ref))
    del g
    assert capi.device_status(True) == 0


def test_dynamic_fused_k_split_one_rank():
    M, N, K = 2048, 2048, 2048
    A, Bt = workloads.make_operands(M, N, K, seed=6)
    comm, handle = capi.ksplit_create(0, 1, M, N)
    try:
        capi.ksplit_connect(comm, handle)
        outs = []
        for mode in (0, 1, 1):
            capi.set_dynamic(mode)
            C = torch.zeros(M, N, dtype=torch.bfloat16, device="cuda")
            st = capi.ksplit_gemm_bf16(comm, A.data_ptr(), Bt.data_ptr(), C.data_ptr(), M, N, K,
                                       K, K, N, torch.cuda.current_stream().cuda_stream)
            assert st == capi.OK
            torch.cuda.synchronize()
            outs.append(C)
        assert torch.equal(bits(outs[1]), bits(outs[0]))
        assert torch.equal(bits(outs[2]), bits(outs[0]))
    finally:
        capi.ksplit_destroy(comm)
    assert capi.device_status(True) == 0
