"""Minimal launcher for Nsight Compute captures and counter summaries.

    python -m blackwell_gemm_b200.ncu_driver {ours|cublas} M N K [launches]

builds seeded N(0, 1) bf16 operands (``workloads.make_operands``) and runs
the GEMM ``launches`` times (default 2) on cuda:0, so a capture such as

    ncu --set full --clock-control none -k regex:gemm_bf16_pair -s 1 -c 1 \
        -o prof python -m blackwell_gemm_b200.ncu_driver ours 8192 8192 8192

records one warm launch of a realistically sized problem and nothing else.
(The reference's kernels are captured through ``bench.py --impl reference``.)

    python -m blackwell_gemm_b200.ncu_driver summarize prof.csv

prints the counters the profiles in this repository quote, from the CSV of
``ncu -i prof.ncu-rep --page raw --csv`` (the role of the reference's
CSV-exporting profile runner, src/bench_core.py:303-384).
"""
from __future__ import annotations

import csv
import sys

KEY_METRICS = [
    "gpu__time_duration.sum",
    "gpc__cycles_elapsed.max.per_second",
    "sm__pipe_tensor_cycles_active.avg.pct_of_peak_sustained_elapsed",
    "sm__throughput.avg.pct_of_peak_sustained_elapsed",
    "dram__bytes_read.sum",
    "dram__bytes_write.sum",
    "gpu__dram_throughput.avg.pct_of_peak_sustained_elapsed",
    "lts__t_sector_hit_rate.pct",
    "lts__throughput.avg.pct_of_peak_sustained_elapsed",
    "l1tex__m_xbar2l1tex_read_bytes_mem_global_op_tma_ld.sum",
    "lts__t_sectors_srcunit_ltcfabric.sum",
    "smsp__inst_executed.sum",
    "launch__registers_per_thread",
    "launch__grid_size",
    "launch__block_size",
    "launch__shared_mem_per_block_dynamic",
]


def run(impl: str, M: int, N: int, K: int, launches: int) -> None:
    import torch

    from . import matmul_b200
    from .workloads import make_operands

    A, Bt = make_operands(M, N, K)
    fn = (lambda: matmul_b200(A, Bt.T)) if impl == "ours" else (lambda: torch.matmul(A, Bt.T))
    for _ in range(launches):
        fn()
    torch.cuda.synchronize()
    print(f"ran {impl} {M}x{N}x{K} x{launches}")


def summarize(path: str) -> None:
    rows = list(csv.reader(open(path)))
    hdr, units = rows[0], rows[1]
    for vals in rows[2:]:
        d = dict(zip(hdr, zip(units, vals)))
        print(d.get("Kernel Name", ("", "?"))[1][:100])
        for k in KEY_METRICS:
            if k in d:
                print(f"  {k} = {d[k][1]} {d[k][0]}")
        stalls = [(k, float(v[1])) for k, v in d.items()
                  if k.startswith("smsp__average_warps_issue_stalled")
                  and k.endswith("per_issue_active.ratio") and v[1]]
        for k, v in sorted(stalls, key=lambda x: -x[1])[:6]:
            name = k.replace("smsp__average_warps_issue_stalled_", "").replace(
                "_per_issue_active.ratio", "")
            print(f"  stall {name} = {v:.3f}")


def main(argv) -> None:
    if len(argv) >= 2 and argv[0] == "summarize":
        summarize(argv[1])
        return
    if len(argv) < 4 or argv[0] not in ("ours", "cublas"):
        raise SystemExit(__doc__)
    run(argv[0], int(argv[1]), int(argv[2]), int(argv[3]), int(argv[4]) if len(argv) > 4 else 2)


if __name__ == "__main__":
    main(sys.argv[1:])
