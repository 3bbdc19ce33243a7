"""Generates the golden vectors in tests/golden/*.npz by running the
reference's own v8 kernel (matmul_v8, src/kernels/kernel_v8.cu:830-833,
compiled from its sources into oracle/_ref/libref_gemm.so by oracle/build.py)
on the seeded inputs of tests/golden/cases.py.

Run once on a B200:  python tests/golden/make_golden.py [--out DIR]
Also records the v6 kernel's output and checks v6 == v8 on the exact cases,
as a sanity check of the reference build itself.
"""
from __future__ import annotations

import sys
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parents[2]
sys.path.insert(0, str(ROOT))
sys.path.insert(0, str(Path(__file__).resolve().parent))

import torch  # noqa: E402

import cases  # noqa: E402
import oracle  # noqa: E402


def run_ref(version, A, Bt):
    M, K = A.shape
    N = Bt.shape[0]
    a = torch.from_numpy(A.view(np.int16)).cuda()
    b = torch.from_numpy(Bt.view(np.int16)).cuda()
    c = torch.zeros(M, N, dtype=torch.int16, device="cuda")
    oracle.ref_gemm(version, a.data_ptr(), b.data_ptr(), c.data_ptr(), M, N, K)
    torch.cuda.synchronize()
    return c.cpu().numpy().view(np.uint16)


def main():
    out_dir = Path(sys.argv[sys.argv.index("--out") + 1]) if "--out" in sys.argv else cases.HERE
    out_dir.mkdir(parents=True, exist_ok=True)
    for case in cases.CASES:
        A, Bt = cases.inputs(case)
        C8 = run_ref("v8", A, Bt)
        C6 = run_ref("v6", A, Bt)
        if case["kind"] == "exact":
            assert np.array_equal(C8, C6), f"{case['name']}: reference v6 != v8 on exact inputs"
        np.savez_compressed(out_dir / cases.path(case).name, C=C8, kind=case["kind"], version="v8",
                            input_sha256=cases.input_digest(A, Bt),
                            M=case["M"], N=case["N"], K=case["K"], seed=case["seed"],
                            std=case["std"])
        print(f"{case['name']}: wrote {out_dir / cases.path(case).name} "
              f"(v6==v8 on {np.mean(C6 == C8) * 100:.2f}% of elements)")


if __name__ == "__main__":
    main()
