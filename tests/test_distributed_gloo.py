"""Host logic of the multi-GPU configurations on CPU ranks (gloo, 2 processes):
row sharding and the K-split reduce-scatter, with a plain fp32 GEMM standing
in for the kernel (the GPU runs use the package's kernels).  Also checks that
a rank that fails makes its peers' next collective end with an error instead
of waiting for ever."""
import os
import socket
import traceback

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from blackwell_gemm_b200 import distributed as bdist


def free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def cpu_gemm_f32(A, Bt):
    return A.float() @ Bt.float().T


def cpu_cast(W):
    return W.to(torch.bfloat16)


def operands(M, N, K, seed=0):
    g = torch.Generator().manual_seed(seed)
    A = torch.randn(M, K, generator=g).to(torch.bfloat16)
    Bt = torch.randn(N, K, generator=g).to(torch.bfloat16)
    return A, Bt


def _worker(rank, world, port, case, errq):
    try:
        os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
        from datetime import timedelta
        dist.init_process_group("gloo", rank=rank, world_size=world,
                                timeout=timedelta(seconds=10))
        M, N, K = 64, 48, 96
        A, Bt = operands(M, N, K)
        full = (A.float() @ Bt.float().T)
        if case == "k_split":
            ks = bdist.k_slice(K, world, rank)
            rows = bdist.k_split_gemm(A[:, ks].contiguous(), Bt[:, ks].contiguous(),
                                      gemm_f32=cpu_gemm_f32, cast=cpu_cast)
            mine = full[rank * M // world:(rank + 1) * M // world]
            assert rows.dtype == torch.bfloat16 and rows.shape == mine.shape
            # summed in fp32 across ranks, rounded once
            assert torch.allclose(rows.float(), mine.to(torch.bfloat16).float(), rtol=1e-2,
                                  atol=1e-2)
            err = (rows.float() - mine).norm() / mine.norm()
            assert err < 5e-3, float(err)
        elif case == "row_shard":
            rs = slice(rank * M // world, (rank + 1) * M // world)
            rows = bdist.row_shard_gemm(A[rs], Bt, gemm=lambda a, b: cpu_cast(cpu_gemm_f32(a, b)))
            assert torch.equal(rows, full[rs].to(torch.bfloat16))
        elif case == "sampled_parity":
            # K-split parity on sampled rows without any rank holding all of K:
            # the right rows pass on every rank, a planted error in rank 1's
            # block fails on every rank.
            ks = bdist.k_slice(K, world, rank)
            rs = slice(rank * M // world, (rank + 1) * M // world)
            rows = full[rs].to(torch.bfloat16)
            got = bdist.k_split_sampled_parity(rows, A[:, ks].contiguous(), Bt[:, ks].contiguous(),
                                               per_owner=M // world)
            assert got["pass"] and got["rows_checked"] == M, got
            assert got["max_scaled"] < 1e-2 and got["rel_fro"] < 5e-3, got
            bad = rows.clone()
            if rank == 1:
                bad[3, 5] += 4.0
            got = bdist.k_split_sampled_parity(bad, A[:, ks].contiguous(), Bt[:, ks].contiguous(),
                                               per_owner=M // world)
            assert not got["pass"], got
        elif case == "rank_fails":
            if rank == 1:
                raise SystemExit(0)          # leaves before the collective
            ks = bdist.k_slice(K, world, rank)
            try:
                bdist.k_split_gemm(A[:, ks].contiguous(), Bt[:, ks].contiguous(),
                                   gemm_f32=cpu_gemm_f32, cast=cpu_cast)
            except Exception:
                errq.put((rank, "timed-out-as-expected"))
                return
            raise AssertionError("collective completed although a rank had left")
        dist.destroy_process_group()
        errq.put((rank, "ok"))
    except SystemExit:
        errq.put((rank, "left"))
    except Exception:
        errq.put((rank, traceback.format_exc()))


def run(case, world=2):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, case, q)) for r in range(world)]
    for p in procs:
        p.start()
    out = dict(q.get(timeout=120) for _ in procs)
    for p in procs:
        p.join(timeout=60)
        if p.is_alive():
            p.kill()
    return out


def test_k_split_reduce_scatter_gloo():
    out = run("k_split")
    assert all(v == "ok" for v in out.values()), out


def test_row_shard_gloo():
    out = run("row_shard")
    assert all(v == "ok" for v in out.values()), out


def test_k_split_sampled_parity_gloo():
    out = run("sampled_parity")
    assert all(v == "ok" for v in out.values()), out


def test_failed_rank_ends_peer_collective_with_error():
    out = run("rank_fails")
    assert out[1] == "left"
    assert out[0] == "timed-out-as-expected", out


def test_slicing_rules():
    assert bdist.k_slice(8, 2, 1) == slice(4, 8)
    with pytest.raises(ValueError):
        bdist.k_slice(9, 2, 0)


def test_fused_k_split_checks_operands_and_out_before_any_call():
    # The checks run before the C ABI is reached, so an instance whose
    # construction (a device collective) is skipped can exercise them.
    from blackwell_gemm_b200.distributed import FusedKSplit

    fk = object.__new__(FusedKSplit)
    fk.world = 2
    fk.device = torch.device("cuda", 0)
    A = torch.zeros(512, 64, dtype=torch.bfloat16)
    B = torch.zeros(256, 64, dtype=torch.bfloat16)
    with pytest.raises(ValueError):                 # CPU tensors are not on a GPU
        fk._check_operands(A, B)
    with pytest.raises(TypeError):
        fk._check_operands(A.float(), B)
    with pytest.raises(ValueError):
        fk._check_operands(A, B[:, :32])
    dev = torch.device("cpu")
    fk._check_out(torch.empty(256, 256, dtype=torch.bfloat16), 512, 256, dev)
    with pytest.raises(ValueError):                 # too few rows for M / P
        fk._check_out(torch.empty(128, 256, dtype=torch.bfloat16), 512, 256, dev)
    with pytest.raises(ValueError):                 # columns not contiguous
        fk._check_out(torch.empty(256, 512, dtype=torch.bfloat16)[:, ::2], 512, 256, dev)
    with pytest.raises(TypeError):
        fk._check_out(torch.empty(256, 256, dtype=torch.float32), 512, 256, dev)


class _FakeCudaTensor:
    """Just enough of a tensor on another GPU for FusedKSplit's checks."""

    def __init__(self, shape, device):
        self.shape, self.device, self.dtype = torch.Size(shape), torch.device(device), torch.bfloat16

    def dim(self):
        return len(self.shape)

    def is_contiguous(self):
        return True


def test_fused_k_split_refuses_operands_on_another_gpu():
    # The communicator lives on cuda:0; operands on cuda:1 must be refused in
    # Python, before any pointer reaches b200_ksplit_gemm_bf16.
    from blackwell_gemm_b200.distributed import FusedKSplit

    fk = object.__new__(FusedKSplit)
    fk.world = 2
    fk.device = torch.device("cuda", 0)
    fk._check_operands(_FakeCudaTensor((512, 64), "cuda:0"), _FakeCudaTensor((256, 64), "cuda:0"))
    with pytest.raises(ValueError, match="this rank's GPU"):
        fk._check_operands(_FakeCudaTensor((512, 64), "cuda:1"),
                           _FakeCudaTensor((256, 64), "cuda:1"))
    with pytest.raises(ValueError, match="one CUDA device"):
        fk._check_operands(_FakeCudaTensor((512, 64), "cuda:0"),
                           _FakeCudaTensor((256, 64), "cuda:1"))
