"""The reference's own kernels, built unmodified from its sources into
oracle/_ref (oracle/build.py), on one GPU: every version its binding exports
must compute the GEMM correctly before the bench times it as the "reference
best version" baseline.  (Outside test_gemm_gpu.py, whose fixture repeats
every test on each of our kernel configurations.)"""
import numpy as np
import pytest
import torch

import oracle

pytestmark = pytest.mark.gpu


def test_every_reference_version_on_exact_inputs():
    """Each launcher of the reference binding (src/matmul.cpp:4-13), built from
    its sources, returns the unique exact-arithmetic result at a shape every
    version supports: the bench's "reference best version" baseline times only
    versions that compute the GEMM correctly.  2048^3 is the smallest shape the
    reference's own harness runs (src/main.py:107)."""
    try:
        oracle.ref_lib()
    except ImportError:
        pytest.skip("reference build (oracle/_ref) not present")
    M, N, K = 2048, 2048, 2048
    a, b = oracle.exact_inputs(M, N, K, seed=11)
    want = oracle.gemm_bf16(a, b)
    A = torch.from_numpy(a.view(np.int16)).cuda().view(torch.bfloat16)
    Bt = torch.from_numpy(b.view(np.int16)).cuda().view(torch.bfloat16)
    for v in ["v1_2d", "v1_3d", "v2", "v3", "v4", "v5", "v6", "v7", "v8"]:
        assert oracle.ref_supports(v, M, N, K), v
        C = torch.zeros(M, N, dtype=torch.bfloat16, device="cuda")
        oracle.ref_gemm(v, A.data_ptr(), Bt.data_ptr(), C.data_ptr(), M, N, K)
        torch.cuda.synchronize()
        got = C.view(torch.int16).cpu().numpy().view(np.uint16)
        assert np.array_equal(got, want), v
