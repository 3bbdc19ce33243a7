"""b200_gemm_bf16_noalloc: the GEMM for callers that cannot let a library
allocate device memory (processes that reserve GPU memory up front through
their own allocator, loops where a cudaMalloc/cudaFree would synchronize the
device).  Called through the C ABI and compared with b200_gemm_bf16 on the
same inputs, on two calls in a row, within the parity tolerance the other
tests use; free device memory is read after the entry point's one-time
set-up and must not move across the two calls.  Its error word is read
through b200_gemm_noalloc_status: a wait self-test that runs out is recorded
there, stays until read, and a following call still succeeds.  The file name
makes pytest collect it last.
"""
import pytest
import torch

from blackwell_gemm_b200 import capi, parity, workloads

pytestmark = pytest.mark.gpu

SHAPES = [(512, 1024, 8192),     # pair-kernel split-K: fp32 accumulator in the array
          (16, 28672, 4096),     # skinny stream-K: slots and flags in the array
          (150, 20480, 2048),    # skinny split-K: fp32 accumulator in the array
          (16, 8192, 8192),      # skinny cluster kernel (DSMEM reduction): no workspace
          (8, 4096, 4096),       # skinny cluster kernel, 4-CTA clusters
          (256, 8192, 8192),     # skinny cluster kernel on 2-CTA pairs: no workspace
          (128, 32768, 2048),    # skinny stream-K, slots too large for the array: cluster kernel
          (1024, 1024, 1024),    # not split: only the error word is used
          (300, 520, 4096),      # ragged
          (4096, 4096, 4096)]    # the allocating path adds a stream-K tail, this one not    # the allocating path adds a stream-K tail, this one not


def run(fn, A, Bt, C):
    M, K = A.shape
    N = Bt.shape[0]
    st = fn(A.data_ptr(), Bt.data_ptr(), C.data_ptr(), M, N, K, K, K, C.stride(0),
            torch.cuda.current_stream().cuda_stream)
    assert st == capi.OK, capi.status_string(st)


@pytest.mark.parametrize("M,N,K", SHAPES)
def test_noalloc_matches_allocating_entry_point_twice(M, N, K):
    capi.set_splits(0)
    A, Bt = workloads.make_operands(M, N, K, seed=M + N, weight_std=0.02)
    ldc = (N + 7) // 8 * 8
    ref = torch.zeros(M, ldc, dtype=torch.bfloat16, device="cuda")
    run(capi.gemm_bf16, A, Bt, ref)
    outs = [torch.zeros_like(ref) for _ in range(2)]
    # one-time set-up of the entry point on this device (a no-op after the
    # first time), then free memory before the first call and after each
    assert capi.noalloc_status(True) == 0
    torch.cuda.synchronize()
    free = [torch.cuda.mem_get_info()[0]]
    for C in outs:
        run(capi.gemm_bf16_noalloc, A, Bt, C)
        torch.cuda.synchronize()
        free.append(torch.cuda.mem_get_info()[0])
    assert free[1] == free[0] and free[2] == free[0], free   # neither call took memory
    assert capi.noalloc_status(True) == 0
    for C in outs:
        m = parity.metrics(C[:, :N], ref[:, :N].float(), A, Bt)
        assert m["max_scaled"] <= parity.MAX_SCALED_TOL and m["rel_fro"] <= parity.REL_FRO_TOL, m
        m = parity.metrics(C[:, :N], A.float() @ Bt.float().T, A, Bt)
        assert parity.passes(m), m


def test_noalloc_timeout_is_recorded_and_read():
    # A wait that nothing releases, bounded at 50 ms, recording into the
    # array's error word: the word holds the probe's code until it is read
    # and cleared; the allocating path's word is not touched; a GEMM after it
    # succeeds and leaves the word at zero.
    assert capi.noalloc_status(True) == 0
    assert capi.device_status(True) == 0
    assert capi.noalloc_wait_probe(50_000_000) == capi.OK
    torch.cuda.synchronize()
    assert capi.noalloc_status(False) == 0x1006          # read, kept
    assert capi.noalloc_status(True) == 0x1006           # read, cleared
    assert capi.noalloc_status(True) == 0
    assert capi.device_status(True) == 0
    M, N, K = 512, 512, 512
    A, Bt = workloads.make_operands(M, N, K, seed=9)
    C = torch.zeros(M, N, dtype=torch.bfloat16, device="cuda")
    run(capi.gemm_bf16_noalloc, A, Bt, C)
    torch.cuda.synchronize()
    assert capi.noalloc_status(True) == 0
    assert parity.passes(parity.metrics(C, A.float() @ Bt.float().T, A, Bt))


def test_noalloc_rejects_workspace_beyond_its_fixed_size():
    # forcing split-K on a 4096 x 4096 output needs 64 MiB of workspace
    M = N = 4096
    A, Bt = workloads.make_operands(M, N, 512, seed=1)
    C = torch.empty(M, N, dtype=torch.bfloat16, device="cuda")
    capi.set_splits(4)
    try:
        st = capi.gemm_bf16_noalloc(A.data_ptr(), Bt.data_ptr(), C.data_ptr(), M, N, 512, 512,
                                    512, N, 0)
    finally:
        capi.set_splits(0)
    assert st == capi.ERR_TOO_LARGE
    assert "exceeds" in capi.status_string(st)
