"""b200_gemm_bf16_host / matmul_b200_host: operands in host memory, A and B
uploaded in alternating blocks of rows, the GEMM of each C block issued once
its two blocks are up, uploads, GEMMs and downloads overlapped on three
streams.

Exact-arithmetic inputs must match the oracle bit for bit for every block
size (ragged last blocks included); random inputs meet the parity bar and,
with whole-tile unsplit kernels forced on both sides, equal the
device-resident GEMM bit for bit.
"""
import numpy as np
import pytest
import torch

import oracle
import blackwell_gemm_b200 as bg
from blackwell_gemm_b200 import capi, parity, workloads

pytestmark = pytest.mark.gpu


def host_gemm(A, Bt, block_rows=0, pinned=True):
    M, K = A.shape
    N = Bt.shape[0]
    C = torch.zeros(M, N, dtype=torch.bfloat16)
    if pinned:
        A, Bt, C = A.pin_memory(), Bt.pin_memory(), C.pin_memory()
    s = torch.cuda.current_stream()
    st = capi.gemm_bf16_host(A.data_ptr(), Bt.data_ptr(), C.data_ptr(), M, N, K, K, K, N,
                             block_rows, s.cuda_stream)
    assert st == capi.OK, capi.status_string(st)
    s.synchronize()
    return C


def u16(x):
    return torch.from_numpy(np.ascontiguousarray(x).view(np.int16)).view(torch.bfloat16)


@pytest.mark.parametrize("M,N,K", [(1000, 520, 700), (256, 64, 64), (7, 24, 40), (2048, 1536, 1024)])
@pytest.mark.parametrize("block_rows", [0, 256, 300, 10000])
def test_exact_inputs_bit_exact(M, N, K, block_rows):
    a, b = oracle.exact_inputs(M, N, K, seed=M + block_rows)
    C = host_gemm(u16(a), u16(b), block_rows)
    assert np.array_equal(C.view(torch.int16).numpy().view(np.uint16), oracle.gemm_bf16(a, b))


@pytest.mark.parametrize("pinned", [True, False])
def test_random_matches_device_gemm(pinned):
    M, N, K = 3000, 2048, 2048
    A, Bt = workloads.make_operands(M, N, K, seed=5)
    # whole-tile, unsplit kernels on both sides: every element then sums its
    # K blocks in the same order, whatever the block shapes
    capi.set_stream_k(0)
    capi.set_splits(1)
    try:
        C = host_gemm(A.cpu(), Bt.cpu(), 512, pinned)
    finally:
        capi.set_stream_k(1)
        capi.set_splits(0)
    ref = torch.empty(M, N, dtype=torch.bfloat16, device="cuda")
    capi.set_stream_k(0)
    capi.set_splits(1)
    try:
        assert capi.gemm_bf16(A.data_ptr(), Bt.data_ptr(), ref.data_ptr(), M, N, K, K, K, N,
                              0) == capi.OK
        torch.cuda.synchronize()
    finally:
        capi.set_stream_k(1)
        capi.set_splits(0)
    assert torch.equal(C.view(torch.int16), ref.cpu().view(torch.int16))
    assert parity.passes(parity.metrics(C.cuda(), A.float() @ Bt.float().T, A, Bt))


def test_python_entry_point_and_errors():
    A, Bt = workloads.make_operands(512, 768, 1024, seed=9)
    C = bg.matmul_b200_host(A.cpu(), Bt.cpu().T)
    assert C.is_pinned() and C.shape == (512, 768)
    assert parity.passes(parity.metrics(C.cuda(), A.float() @ Bt.float().T, A, Bt))
    with pytest.raises(RuntimeError):
        bg.matmul_b200_host(A, Bt.T)                  # device tensors
    assert capi.gemm_bf16_host(0, 0, 0, -1, 8, 8, 8, 8, 8, 0, 0) == capi.ERR_INVALID_ARGUMENT
    assert capi.device_status(True) == 0
