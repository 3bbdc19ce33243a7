"""Intra-kernel profiler buffers decoded on the CPU.

Rows follow the reference's format (src/profiler.h:22-50): row r = block *
warps_per_cta + warp holds [count, (smid, tag, start_ns, duration_ns) x
entries].  Hand-built buffers check the decoder, the per-role totals and the
Chrome trace without a GPU.
"""
import json

import torch

from blackwell_gemm_b200 import profiler


def make_buffer(rows, entries):
    """rows: {row_index: [(smid, tag, start, dur), ...]}"""
    n = max(rows) + 1
    buf = torch.zeros(n, 1 + 4 * entries, dtype=torch.int64)
    for r, evs in rows.items():
        buf[r, 0] = len(evs)
        for i, e in enumerate(evs[:entries]):
            buf[r, 1 + 4 * i:5 + 4 * i] = torch.tensor(e)
    return buf


def test_decode_roles_tags_and_positions():
    warps = 6
    rows = {
        0: [(3, 0, 1000, 50)],                       # block 0 producer: Setup
        1: [(3, 2, 1100, 20), (3, 3, 1120, 30)],     # block 0 MMA: IssueMMA, WaitTMA
        8: [(7, 7, 2000, 400)],                      # block 1 warp 2 (epilogue): Epilogue
    }
    ev = list(profiler.decode(make_buffer(rows, 4), warps))
    assert len(ev) == 4
    by = {(e["block"], e["warp"], e["tag"]): e for e in ev}
    assert by[(0, 0, "Setup")]["role"] == "producer"
    assert by[(0, 1, "IssueMMA")]["role"] == "mma" and by[(0, 1, "WaitTMA")]["dur_ns"] == 30
    e = by[(1, 2, "Epilogue")]
    assert e["role"] == "epilogue" and e["smid"] == 7 and e["start_ns"] == 2000


def test_count_beyond_capacity_is_clipped_and_empty_rows_skipped():
    entries = 2
    buf = make_buffer({0: [(0, 1, 10, 1), (0, 1, 20, 1)], 3: []}, entries)
    buf[0, 0] = 99                                   # the kernel stops at capacity
    ev = list(profiler.decode(buf, 6))
    assert len(ev) == entries


def test_summary_and_chrome_trace():
    rows = {0: [(1, 0, 100, 10)], 1: [(1, 2, 120, 30), (1, 2, 160, 5)],
            2: [(1, 7, 130, 100)]}
    buf = make_buffer(rows, 4)
    s = profiler.summary(buf, 6)
    assert s["span_ns"] == 230 - 100
    assert s["by_role_tag"] == {"epilogue/Epilogue": 100, "mma/IssueMMA": 35,
                                "producer/Setup": 10}
    trace = json.loads(profiler.chrome_trace(buf, 6))
    evs = trace["traceEvents"]
    assert len(evs) == 4 and all(e["ph"] == "X" for e in evs)
    assert min(e["ts"] for e in evs) == 0.0
    assert {e["name"] for e in evs} == {"Setup", "IssueMMA", "Epilogue"}
