"""Intra-kernel profiler: buffer sizing, decoding and Chrome-trace export.

``profile_matmul_b200(A, B, profiler, num_entries)`` makes every warp of the
GEMM record up to ``num_entries`` intervals into its own row of ``profiler``:

    row = [count, (smid, tag, start_ns, duration_ns) * num_entries]

with ``row = block * warps_per_cta + warp`` (6 warps per CTA for 256-wide
pair tiles, 10 for 512-wide ones: producer, MMA, then epilogue warps).  Row format and tag numbering are the
reference's (src/profiler.h:4-50, decoded in src/bench_core.py:474-527); the
buffer size comes from the real launch grid (``profile_rows``), which the
reference gets wrong for v8 (src/bench_core.py:459-461 vs
src/kernels/kernel_v8.cu:416).
"""
from __future__ import annotations

import json
from collections import defaultdict

import torch

TAGS = ["Setup", "IssueTMA", "IssueMMA", "WaitTMA", "WaitMMA", "WaitMainloop", "WaitEpilogue",
        "Epilogue"]


def role(warp: int) -> str:
    return "producer" if warp == 0 else "mma" if warp == 1 else "epilogue"


def warps_per_cta(M: int, N: int, K: int) -> int:
    """Warps per CTA of the kernel the current tuning launches for M x N x K."""
    from . import capi
    return capi.launch_shape(M, N, K)["threads"] // 32


def alloc(M: int, N: int, K: int, num_entries: int, device="cuda") -> torch.Tensor:
    from . import profile_rows

    rows = profile_rows(M, N, K)
    return torch.zeros(rows, 1 + 4 * num_entries, dtype=torch.int64, device=device)


def decode(buf: torch.Tensor, warps: int):
    """Yields dicts {block, warp, role, smid, tag, start_ns, dur_ns};
    ``warps`` = warps per CTA of the launch (``warps_per_cta``)."""
    data = buf.detach().cpu()
    width = data.shape[1]
    for r in range(data.shape[0]):
        cnt = int(data[r, 0])
        cnt = min(cnt, (width - 1) // 4)
        if cnt <= 0:
            continue
        ent = data[r, 1:1 + 4 * cnt].view(cnt, 4)
        block, warp = divmod(r, warps)
        for smid, tag, start, dur in ent.tolist():
            yield {"block": block, "warp": warp, "role": role(warp), "smid": smid,
                   "tag": TAGS[tag] if 0 <= tag < len(TAGS) else str(tag),
                   "start_ns": start, "dur_ns": dur}


def summary(buf: torch.Tensor, warps: int) -> dict:
    """Total recorded ns per (role, tag), and the kernel's wall span."""
    tot = defaultdict(int)
    lo, hi = None, None
    for e in decode(buf, warps):
        tot[(e["role"], e["tag"])] += e["dur_ns"]
        lo = e["start_ns"] if lo is None else min(lo, e["start_ns"])
        end = e["start_ns"] + e["dur_ns"]
        hi = end if hi is None else max(hi, end)
    return {"span_ns": (hi - lo) if lo is not None else 0,
            "by_role_tag": {f"{r}/{t}": v for (r, t), v in sorted(tot.items())}}


def chrome_trace(buf: torch.Tensor, warps: int) -> str:
    """Chrome/Perfetto trace JSON: one process per SM, one thread per
    (block, warp)."""
    events = list(decode(buf, warps))
    t0 = min((e["start_ns"] for e in events), default=0)
    out = [{"name": e["tag"], "ph": "X", "pid": e["smid"], "tid": e["block"] * 16 + e["warp"],
            "ts": (e["start_ns"] - t0) / 1000.0, "dur": e["dur_ns"] / 1000.0,
            "args": {"block": e["block"], "warp": e["warp"], "role": e["role"]}}
           for e in events]
    return json.dumps({"traceEvents": out, "displayTimeUnit": "ns"})
