"""Fused K-split over NVLink (b200_ksplit_* / distributed.FusedKSplit).

* One rank (any single GPU): the communicator's kernel with P = 1 owns every
  tile, so it must reproduce b200_gemm_bf16 bit for bit (same pair tiles, 256
  or 512 wide, same MMA order) and the oracle exactly on exact-arithmetic
  inputs.
* Two, four and eight ranks (one GPU and one process each, NVLS off): at two
  ranks rows must equal the NCCL reduce-scatter path bit for bit (same fp32
  partials, and a two-term fp32 sum does not depend on order); at more ranks
  the kernel sums in rank order and NCCL's ring in its own order, so rows
  must be within one bf16 ulp of NCCL's for all but a few elements.  At every
  rank count rows must match the oracle exactly on exact inputs (exact sums
  do not depend on order) and meet the parity bar on random ones, across several calls (both receive
  parities, both tile widths) and a change of shape inside the capacity.  Then one rank calls
  alone: its wait for the peer's pieces must run out (bound 5 x 0.2 s), set
  the device error word to 0x1007 and return.
"""
import os
import socket

import numpy as np
import pytest
import torch

import oracle
from blackwell_gemm_b200 import capi, parity, workloads

pytestmark = pytest.mark.gpu


def _dev(x: np.ndarray, device) -> torch.Tensor:
    return torch.from_numpy(np.ascontiguousarray(x).view(np.int16)).to(device).view(torch.bfloat16)


def _bits(t: torch.Tensor) -> np.ndarray:
    return t.contiguous().view(torch.int16).cpu().numpy().view(np.uint16)


def _one_rank_call(comm, A, Bt, M, N, K):
    C = torch.zeros(M, N, dtype=torch.bfloat16, device="cuda")
    st = capi.ksplit_gemm_bf16(comm, A.data_ptr(), Bt.data_ptr(), C.data_ptr(), M, N, K, K, K, N,
                               torch.cuda.current_stream().cuda_stream)
    assert st == capi.OK, capi.status_string(st)
    torch.cuda.synchronize()
    return C


@pytest.mark.parametrize("tile_n", [256, 512])
def test_single_rank_matches_gemm_and_oracle(tile_n):
    comm, handle = capi.ksplit_create(0, 1, 1024, 1024)
    capi.set_tuning(tile_n, 1, 0)
    try:
        capi.ksplit_connect(comm, handle)
        for M, N, K in [(1024, 1024, 1024), (512, 760, 1000), (256, 64, 64)]:
            A, Bt = workloads.make_operands(M, N, K, seed=M + N + K, device="cuda")
            C = _one_rank_call(comm, A, Bt, M, N, K)
            ref = torch.zeros(M, N, dtype=torch.bfloat16, device="cuda")
            capi.set_splits(1)
            try:
                assert capi.gemm_bf16(A.data_ptr(), Bt.data_ptr(), ref.data_ptr(), M, N, K, K, K,
                                      N, 0) == capi.OK
            finally:
                capi.set_splits(0)
            torch.cuda.synchronize()
            assert torch.equal(C.view(torch.int16), ref.view(torch.int16)), (M, N, K)
            a, b = oracle.exact_inputs(M, N, K, seed=3)
            C = _one_rank_call(comm, _dev(a, "cuda"), _dev(b, "cuda"), M, N, K)
            assert np.array_equal(_bits(C), oracle.gemm_bf16(a, b)), (M, N, K)
        assert capi.ksplit_epoch(comm) == 6
    finally:
        capi.set_tuning(-1, 0, 0)
        capi.ksplit_destroy(comm)
    assert capi.device_status(True) == 0


def test_argument_checks():
    with pytest.raises(capi.GemmError):
        capi.ksplit_create(0, 2, 300, 256)       # M not a multiple of 256 * P
    with pytest.raises(capi.GemmError):
        capi.ksplit_create(2, 2, 512, 256)       # rank out of range
    comm, handle = capi.ksplit_create(0, 1, 512, 512)
    try:
        x = torch.zeros(1024, 1024, dtype=torch.bfloat16, device="cuda")
        # not connected yet
        assert capi.ksplit_gemm_bf16(comm, x.data_ptr(), x.data_ptr(), x.data_ptr(), 256, 256,
                                     64, 64, 64, 256, 0) == capi.ERR_INVALID_ARGUMENT
        bad = bytearray(handle)
        bad[0] ^= 1
        with pytest.raises(capi.GemmError):
            capi.ksplit_connect(comm, bytes(bad))
        capi.ksplit_connect(comm, handle)
        # beyond the capacity
        assert capi.ksplit_gemm_bf16(comm, x.data_ptr(), x.data_ptr(), x.data_ptr(), 1024, 512,
                                     64, 64, 64, 512, 0) == capi.ERR_TOO_LARGE
        # K = 0 and ragged M are refused
        assert capi.ksplit_gemm_bf16(comm, x.data_ptr(), x.data_ptr(), x.data_ptr(), 256, 256,
                                     0, 64, 64, 256, 0) == capi.ERR_INVALID_ARGUMENT
        assert capi.ksplit_gemm_bf16(comm, x.data_ptr(), x.data_ptr(), x.data_ptr(), 200, 256,
                                     64, 64, 64, 256, 0) == capi.ERR_INVALID_ARGUMENT
        assert capi.ksplit_epoch(comm) == 0
    finally:
        capi.ksplit_destroy(comm)


# -------------------------------------------------------- several GPUs
def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, q):
    import traceback
    try:
        os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
        from datetime import timedelta
        import torch.distributed as dist
        from blackwell_gemm_b200 import distributed as bdist
        torch.cuda.set_device(rank)
        dev = torch.device("cuda", rank)
        dist.init_process_group("nccl", rank=rank, world_size=world,
                                timeout=timedelta(seconds=60), device_id=dev)
        report = []
        ok = True
        fk = bdist.FusedKSplit(2048, 1536)
        # random operands, several calls (256- then 512-wide pair tiles): bits
        # equal to the NCCL path, parity against fp32
        calls = [(2048, 1536, 4096), (2048, 1536, 4096), (1024, 1000, 2048), (2048, 1536, 1024)]
        # (each rank owns whole 256-row pair-tile rows of C)
        calls = [c for c in calls if c[0] % (world * 256) == 0]
        for call, (M, N, K) in enumerate(calls + calls):
            capi.set_tuning(256 if call < len(calls) else 512, 1, 0)
            A, Bt = workloads.make_operands(M, N, K, seed=100 + call, device=dev)
            ks = bdist.k_slice(K, world, rank)
            Ak, Bk = A[:, ks].contiguous(), Bt[:, ks].contiguous()
            rows = fk(Ak, Bk)
            nccl_rows = bdist.k_split_gemm(Ak, Bk)
            rs = slice(rank * M // world, (rank + 1) * M // world)
            R = A[rs].float() @ Bt.float().T
            m = parity.metrics(rows, R, A[rs], Bt)
            if world == 2:
                same = torch.equal(rows.view(torch.int16), nccl_rows.view(torch.int16))
            else:
                a16 = rows.view(torch.int16).int()
                b16 = nccl_rows.view(torch.int16).int()
                near = ((a16 - b16).abs() <= 1) & ((a16 < 0) == (b16 < 0))
                same = float(near.float().mean()) > 0.999
            ok &= parity.passes(m) and same
            report.append((call, M, N, K, same, m))
        capi.set_tuning(-1, 0, 0)
        # exact inputs: bit-exact against the oracle (unique bf16 result)
        M, N, K = 2048, 1536, 2048
        a, b = oracle.exact_inputs(M, N, K, seed=7)
        ks = bdist.k_slice(K, world, rank)
        rows = fk(_dev(a[:, ks], dev), _dev(b[:, ks], dev))
        want = oracle.gemm_bf16(a[rank * M // world:(rank + 1) * M // world], b)
        exact = np.array_equal(_bits(rows), want)
        ok &= exact
        report.append(("exact", exact))
        torch.cuda.synchronize()
        st = capi.device_status(True)
        ok &= st == 0
        report.append(("status", st))
        fk.close()

        # A peer that never joins a call: rank 0 calls alone, its own-tile waits
        # run out (5 x 0.2 s) and the kernel returns with the error word set.
        fk = bdist.FusedKSplit(256 * world, 256)  # one pair-tile row per rank
        capi.set_wait_timeout_ns(200_000_000)
        if rank == 0:
            A, Bt = workloads.make_operands(256 * world, 256, 128, seed=1, device=dev)
            fk(A, Bt)
            torch.cuda.synchronize()
            st = capi.device_status(True)
            ok &= st == 0x1007
            report.append(("lonely call status", hex(st)))
        capi.set_wait_timeout_ns(2_000_000_000)
        fk.close()
        dist.barrier()
        dist.destroy_process_group()
        q.put((rank, bool(ok), str(report)))
    except Exception:
        q.put((rank, False, traceback.format_exc()))


@pytest.mark.parametrize("world", [2, 4, 8])
def test_fused_k_split_on_several_gpus(world):
    if torch.cuda.device_count() < world:
        pytest.skip(f"needs {world} GPUs")
    import torch.multiprocessing as mp
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    ps = [ctx.Process(target=_worker, args=(r, world, port, q)) for r in range(world)]
    for p in ps:
        p.start()
    res = [q.get(timeout=300) for _ in ps]
    for p in ps:
        p.join(timeout=60)
    assert all(ok for _, ok, _ in res), res
