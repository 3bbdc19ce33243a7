"""Benchmark of the B200 BF16 GEMM: cold-L2 TFLOP/s at 8192^3 per GPU.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
    torchrun --nproc-per-node N bench.py --gpus N ...      (N > 1)

One step = one C = A * B^T of the hot path on one batch of synthetic input.
Each rank owns an 8192-row block of A and a replicated 8192 x 8192 B (the
row-sharded configuration: M = 8192 * N in total, no collective), so per-GPU
work is fixed as N grows ("scaling": "weak").  At N = 1 this is the 8192^3
headline shape.  Operands are seeded N(0, 1) bf16, generated on the device.

Timing follows the reference harness (src/bench_core.py:47-69): a 256 MB
buffer is written before every step so L2 is cold, and each GEMM is bracketed
by CUDA events on the launching stream; the K timed steps sit between a
barrier + synchronize on both sides, and the per-rank GEMM time is maxed over
ranks.  Rank 0 prints one JSON line.

Extra measurements in the same line: e2e (the same GEMM through the C ABI
with pinned host buffers, copies inside the timed region), the roofline of
the kernel against the measured bf16 peak, SM clocks sampled during the timed
region, same-process baselines (cuBLAS and the reference's own v8 kernel) and
the CPU oracle timed on the host's cores on a bounded sample.
"""
from __future__ import annotations

import argparse
import json
import os
import re
import statistics
import sys
import threading
import time
from pathlib import Path

import torch

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

M_PER_GPU, N_DIM, K_DIM = 8192, 8192, 8192
FLUSH_BYTES = 256 * 1024 * 1024
FALLBACK_BF16_TFLOPS = 1590.0      # earlier measurement on this pool (burst)
# Every timed arm (ours, cuBLAS, the reference) starts after the GPU has
# idled this long, so each sees the same power-limiter state; the reference
# harness gets the same by running each (shape, version) in a fresh
# container (src/main.py:85-100,158).
IDLE_BEFORE_ARM_S = 1.0


# --------------------------------------------------------------- utilities
def dist_env():
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    return world, rank, local


def measured_peaks():
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        try:
            d = json.loads(p.read_text())
            return d, "measured"
        except Exception:
            pass
    return {"bf16_tflops": FALLBACK_BF16_TFLOPS, "hbm_gbs": 6650.0}, "fallback"


def profiled_traffic():
    """DRAM bytes per launch of the kernel at the bench shape, from the
    committed ncu summary (profiles/*.md, line 'traffic_bytes_per_launch: N')."""
    for p in sorted((ROOT / "profiles").glob("gemm_bf16_pair*8192*.md")):
        m = re.search(r"traffic_bytes_per_launch:\s*([0-9]+)", p.read_text())
        if m:
            return int(m.group(1)), p.name
    return None, None


def pci_bus_string(device: int) -> str:
    """NVML bus id "DDDDDDDD:BB:DD.0" of a CUDA device (torch reports the
    domain, bus and device numbers as integers; NVML's device order differs
    from CUDA's under CUDA_VISIBLE_DEVICES, so the handle is looked up by bus)."""
    p = torch.cuda.get_device_properties(device)
    dom, bus, dev = p.pci_domain_id, p.pci_bus_id, p.pci_device_id
    if not all(isinstance(v, int) for v in (dom, bus, dev)):
        raise TypeError("unexpected PCI id types from torch")
    return f"{dom:08X}:{bus:02X}:{dev:02X}.0"


class ClockSampler:
    """Samples SM clock and clock-event reasons of one GPU through NVML every
    `period_s`, from a thread, between start() and stop().  The NVML calls are
    made once in the constructor so the first timed sample is not slowed by
    library set-up."""
    REASONS = {0x1: "gpu_idle", 0x2: "applications_clocks_setting", 0x4: "sw_power_cap",
               0x8: "hw_slowdown", 0x10: "sync_boost", 0x20: "sw_thermal_slowdown",
               0x40: "hw_thermal_slowdown", 0x80: "hw_power_brake_slowdown",
               0x100: "display_clock_setting"}

    def __init__(self, device: int, period_s: float = 0.002):
        self.samples, self.reasons, self.max_mhz = [], 0, None
        self.period, self._stop, self._th, self.err = period_s, threading.Event(), None, None
        try:
            import pynvml
            pynvml.nvmlInit()
            self.h = pynvml.nvmlDeviceGetHandleByPciBusId(pci_bus_string(device).encode())
            self.nv = pynvml
            self.max_mhz = pynvml.nvmlDeviceGetMaxClockInfo(self.h, pynvml.NVML_CLOCK_SM)
            pynvml.nvmlDeviceGetClockInfo(self.h, pynvml.NVML_CLOCK_SM)
            pynvml.nvmlDeviceGetCurrentClocksEventReasons(self.h)
        except Exception as e:  # NVML missing: report it, do not fail the bench
            self.nv, self.err = None, repr(e)

    def _sample(self):
        self.samples.append(self.nv.nvmlDeviceGetClockInfo(self.h, self.nv.NVML_CLOCK_SM))
        self.reasons |= int(self.nv.nvmlDeviceGetCurrentClocksEventReasons(self.h))

    def _run(self):
        while not self._stop.is_set():
            try:
                self._sample()
            except Exception as e:
                self.err = repr(e)
                return
            self._stop.wait(self.period)

    def start(self):
        if self.nv:
            self._th = threading.Thread(target=self._run, daemon=True)
            self._th.start()

    def stop(self):
        if self._th:
            self._stop.set()
            self._th.join()
            if not self.samples:
                try:  # the region ended before the thread ran: one sample now
                    self._sample()
                except Exception as e:
                    self.err = repr(e)

    def report(self):
        names = [n for b, n in self.REASONS.items() if self.reasons & b]
        out = {"sm_mhz": statistics.median(self.samples) if self.samples else None,
               "sm_max_mhz": self.max_mhz, "reasons": names, "samples": len(self.samples)}
        if self.err:
            out["error"] = self.err
        return out


def step_stats(ms):
    """Distribution of the per-step GEMM times of one rank (ms)."""
    k = max(1, len(ms) // 10)
    return {"min": min(ms), "median": statistics.median(ms), "mean": statistics.mean(ms),
            "max": max(ms), "first_tenth_mean": statistics.mean(ms[:k]),
            "last_tenth_mean": statistics.mean(ms[-k:])}


def cold_l2_loop(fn, steps, stream, flush):
    """Per step: write the flush buffer, then time fn() with events."""
    starts = [torch.cuda.Event(enable_timing=True) for _ in range(steps)]
    ends = [torch.cuda.Event(enable_timing=True) for _ in range(steps)]
    for i in range(steps):
        flush.zero_()
        starts[i].record(stream)
        fn()
        ends[i].record(stream)
    return starts, ends


def wait_event(ev):
    """Block until `ev` completes while sleeping in short naps, so the clock
    sampling thread gets the interpreter during the timed region."""
    while not ev.query():
        time.sleep(0.0005)
    torch.cuda.synchronize()


def time_cold(fn, steps, warmup, stream, flush):
    torch.cuda.synchronize()
    time.sleep(IDLE_BEFORE_ARM_S)
    for _ in range(warmup):
        flush.zero_()
        fn()
    torch.cuda.synchronize()
    s, e = cold_l2_loop(fn, steps, stream, flush)
    torch.cuda.synchronize()
    return [a.elapsed_time(b) for a, b in zip(s, e)]


def time_clean(fn, steps, warmup, stream, flush, clean):
    """As time_cold, but the zero-write of the flush buffer is followed by a
    read of a second buffer larger than L2, so the timed call starts with an
    L2 that holds neither its operands nor dirty lines.  (After the write
    alone, up to the whole L2 is dirty and the timed call pays for writing it
    back: at the HBM-bound shapes that halves the apparent read rate.)"""
    def clean_flush():
        flush.zero_()
        clean.sum()
    torch.cuda.synchronize()
    time.sleep(IDLE_BEFORE_ARM_S)
    for _ in range(warmup):
        clean_flush()
        fn()
    torch.cuda.synchronize()
    starts = [torch.cuda.Event(enable_timing=True) for _ in range(steps)]
    ends = [torch.cuda.Event(enable_timing=True) for _ in range(steps)]
    for i in range(steps):
        clean_flush()
        starts[i].record(stream)
        fn()
        ends[i].record(stream)
    torch.cuda.synchronize()
    return [a.elapsed_time(b) for a, b in zip(starts, ends)]


# ------------------------------------------------------------------- arms
def gemm_ours(A, Bt, C, stream):
    """The product call the bench times: the C ABI on device pointers."""
    from blackwell_gemm_b200 import capi
    M, K = A.shape
    N = Bt.shape[0]
    st = capi.gemm_bf16(A.data_ptr(), Bt.data_ptr(), C.data_ptr(), M, N, K, K, K, N,
                        stream.cuda_stream)
    if st != 0:
        raise RuntimeError(f"b200_gemm_bf16 failed: {capi.status_string(st)}")


def gemm_reference(A, Bt, C, stream, version="v8"):
    """The reference's own matmul_<version> (v8 by default), through its
    launcher (legacy stream)."""
    import oracle
    M, K = A.shape
    N = Bt.shape[0]
    oracle.ref_gemm(version, A.data_ptr(), Bt.data_ptr(), C.data_ptr(), M, N, K)


# Versions of the reference timed as its "best version" baseline: every
# launcher its binding exports (src/matmul.cpp:4-13), where the shape allows.
REFERENCE_VERSIONS = ["v1_2d", "v1_3d", "v2", "v3", "v4", "v5", "v6", "v7", "v8"]


def reference_versions(M, N, K):
    import oracle
    return [v for v in REFERENCE_VERSIONS if oracle.ref_supports(v, M, N, K)]


def parity_sample(C, A, Bt, nrows=256, seed=1):
    from blackwell_gemm_b200 import parity
    g = torch.Generator(device="cpu").manual_seed(seed)
    rows = torch.randperm(A.shape[0], generator=g)[:nrows].to(A.device)
    prev = torch.backends.cuda.matmul.allow_tf32
    torch.backends.cuda.matmul.allow_tf32 = False
    try:
        R = A.index_select(0, rows).float() @ Bt.float().T
    finally:
        torch.backends.cuda.matmul.allow_tf32 = prev
    m = parity.metrics(C, R, A, Bt, rows=rows)
    return {"max_scaled": m["max_scaled"], "rel_fro": m["rel_fro"], "pass": parity.passes(m),
            "rows_checked": nrows, "against": "fp32 GEMM of the same bf16 inputs (GPU, no TF32)"}


def e2e_measure(gemm, A, Bt, stream, steps=8, warmup=2):
    """Same GEMM with host buffers: H2D of A and B from pinned memory, the
    call, D2H of C, all inside the timed region, one stream."""
    M, K = A.shape
    N = Bt.shape[0]
    hA = A.cpu().pin_memory()
    hB = Bt.cpu().pin_memory()
    hC = torch.empty(M, N, dtype=torch.bfloat16).pin_memory()
    dA = torch.empty_like(A)
    dB = torch.empty_like(Bt)
    dC = torch.empty(M, N, dtype=torch.bfloat16, device=A.device)

    def step():
        dA.copy_(hA, non_blocking=True)
        dB.copy_(hB, non_blocking=True)
        gemm(dA, dB, dC, stream)
        hC.copy_(dC, non_blocking=True)

    with torch.cuda.stream(stream):
        for _ in range(warmup):
            step()
        torch.cuda.synchronize()
        s = torch.cuda.Event(enable_timing=True)
        e = torch.cuda.Event(enable_timing=True)
        s.record(stream)
        for _ in range(steps):
            step()
        e.record(stream)
        torch.cuda.synchronize()
    ms = s.elapsed_time(e) / steps
    return ms, 2 * (M * K + N * K), 2 * M * N


def e2e_measure_host(A, Bt, stream, steps=8, warmup=2):
    """Our public host-memory entry point, b200_gemm_bf16_host: pinned host A,
    B and C; inside each call A and B go up in alternating blocks whose
    uploads, GEMMs and C downloads overlap.  CUDA events on the caller's
    stream bracket the calls (the call orders itself after, and releases,
    that stream)."""
    from blackwell_gemm_b200 import capi
    M, K = A.shape
    N = Bt.shape[0]
    hA = A.cpu().pin_memory()
    hB = Bt.cpu().pin_memory()
    hC = torch.empty(M, N, dtype=torch.bfloat16).pin_memory()

    def step():
        st = capi.gemm_bf16_host(hA.data_ptr(), hB.data_ptr(), hC.data_ptr(), M, N, K, K, K, N,
                                 0, stream.cuda_stream)
        capi.check(st, "b200_gemm_bf16_host")

    for _ in range(warmup):
        step()
    torch.cuda.synchronize()
    s = torch.cuda.Event(enable_timing=True)
    e = torch.cuda.Event(enable_timing=True)
    s.record(stream)
    for _ in range(steps):
        step()
    e.record(stream)
    torch.cuda.synchronize()
    ms = s.elapsed_time(e) / steps
    # the result that came back, checked like the device result
    par = parity_sample(hC.to(A.device), A, Bt)
    return ms, 2 * (M * K + N * K), 2 * M * N, par


def link_floor_ms(h2d_bytes, d2h_bytes, dev, reps=3):
    """The PCIe floor of one e2e step: its host->device and device->host bytes
    copied at the same time on two streams, pinned host memory, CUDA events on
    the caller's stream around both (best of `reps` after one warm-up).  The
    link is not full duplex at full rate, so this is below max(up, down)
    at the one-way rates."""
    hu = torch.empty(h2d_bytes, dtype=torch.uint8).pin_memory()
    hd = torch.empty(d2h_bytes, dtype=torch.uint8).pin_memory()
    du = torch.empty(h2d_bytes, dtype=torch.uint8, device=dev)
    dd = torch.empty(d2h_bytes, dtype=torch.uint8, device=dev)
    main = torch.cuda.current_stream(dev)
    s_up, s_down = torch.cuda.Stream(dev), torch.cuda.Stream(dev)
    best = None
    for r in range(reps + 1):
        e0 = torch.cuda.Event(enable_timing=True)
        e1 = torch.cuda.Event(enable_timing=True)
        e0.record(main)
        s_up.wait_stream(main)
        s_down.wait_stream(main)
        with torch.cuda.stream(s_up):
            du.copy_(hu, non_blocking=True)
        with torch.cuda.stream(s_down):
            hd.copy_(dd, non_blocking=True)
        main.wait_stream(s_up)
        main.wait_stream(s_down)
        e1.record(main)
        torch.cuda.synchronize(dev)
        if r:
            ms = e0.elapsed_time(e1)
            best = ms if best is None else min(best, ms)
    return best


def cpu_baseline(Bt, rows=256):
    """CPU oracle (C restatement, all host threads) on `rows` rows of A against
    the full B; TFLOP/s extrapolates linearly in M."""
    import numpy as np
    import oracle
    B_u16 = Bt.cpu().view(torch.int16).numpy().view(np.uint16)
    rng = np.random.default_rng(0)
    A_u16 = oracle.round_bf16(rng.standard_normal((rows, Bt.shape[1]), dtype=np.float32))
    threads = oracle.default_threads()
    t0 = time.perf_counter()
    oracle.gemm_f32(A_u16, B_u16, nthreads=threads)
    dt = time.perf_counter() - t0
    flops = 2 * rows * Bt.shape[0] * Bt.shape[1]
    out = {"value": flops / dt / 1e12, "unit": "TFLOP/s", "cores": threads, "kind": "port",
           "sample": f"{rows} x {Bt.shape[0]} x {Bt.shape[1]} (rows of A against the full B); "
                     f"{dt:.2f} s; rate scales linearly in M",
           "seconds": dt}
    # torch's CPU bf16 matmul on the same sample (the configuration's third baseline)
    a = torch.from_numpy(A_u16.view(np.int16)).view(torch.bfloat16)
    b = Bt.cpu()
    t0 = time.perf_counter()
    torch.matmul(a, b.T)
    dt2 = time.perf_counter() - t0
    out["torch_cpu_bf16"] = {"value": flops / dt2 / 1e12, "unit": "TFLOP/s",
                             "threads": torch.get_num_threads(), "seconds": dt2}
    return out


# ------------------------------------------------------------------- main
def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=100)
    ap.add_argument("--warmup", type=int, default=20)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--no-extras", action="store_true",
                    help="skip e2e, baselines and the CPU sample (timing only)")
    ap.add_argument("--mode", choices=["rows", "ksplit", "sweep"], default="rows",
                    help="rows: 8192^3 per GPU, rows of A sharded (default, the headline); "
                         "ksplit: 8192 x 8192 x 131072 with K split across the GPUs, "
                         "reduced inside the GEMM kernel over NVLink; "
                         "sweep: every single-GPU configuration shape, one line each")
    ap.add_argument("--ref-versions", choices=["all", "v8", "none"], default="all",
                    help="with --mode sweep: reference versions timed per shape (all that "
                         "support it -- the best is reported --, v8 only, or none)")
    ap.add_argument("--shapes", default="",
                    help="with --mode sweep: comma-separated MxNxK shapes to time instead "
                         "of the configuration shapes (weights N(0, 0.02) for M <= 256, "
                         "the skinny rule, else N(0, 1))")
    args = ap.parse_args()
    if args.warmup < 3:
        ap.error("--warmup must be >= 3")

    world, rank, local = dist_env()
    if world != args.gpus:
        print(f"warning: --gpus {args.gpus} but WORLD_SIZE={world}; using {world}",
              file=sys.stderr)
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)

    if args.impl == "reference":
        return run_reference(args, world, rank, dev)
    if args.mode == "ksplit":
        return run_ksplit(args, world, rank, dev)
    if args.mode == "sweep":
        return run_sweep(args, world, rank, dev)

    import torch.distributed as dist
    if world > 1:
        from datetime import timedelta
        dist.init_process_group("nccl", timeout=timedelta(seconds=120), device_id=dev)

    import blackwell_gemm_b200  # noqa: F401  (loads the native library; fails loudly)
    from blackwell_gemm_b200 import capi
    from blackwell_gemm_b200.workloads import make_operands

    M, N, K = M_PER_GPU, N_DIM, K_DIM
    A, _ = make_operands(M, 8, K, seed=1000 + rank, device=dev)        # this rank's rows
    _, Bt = make_operands(8, N, K, seed=0, device=dev)                 # replicated B
    C = torch.empty(M, N, dtype=torch.bfloat16, device=dev)
    flush = torch.empty(FLUSH_BYTES // 4, dtype=torch.int32, device=dev)
    stream = torch.cuda.current_stream()

    gemm_ours(A, Bt, C, stream)
    torch.cuda.synchronize()
    par = parity_sample(C, A, Bt)
    tuning = capi.get_tuning()
    shape = capi.launch_shape(M, N, K)

    torch.cuda.synchronize()
    time.sleep(IDLE_BEFORE_ARM_S)
    for _ in range(args.warmup):
        flush.zero_()
        gemm_ours(A, Bt, C, stream)
    clocks = ClockSampler(local)
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    clocks.start()
    region_s = torch.cuda.Event(enable_timing=True)
    region_e = torch.cuda.Event(enable_timing=True)
    region_s.record(stream)
    starts, ends = cold_l2_loop(lambda: gemm_ours(A, Bt, C, stream), args.steps, stream, flush)
    region_e.record(stream)
    wait_event(region_e)
    if world > 1:
        dist.barrier()
    clocks.stop()
    launch_ms = [a.elapsed_time(b) for a, b in zip(starts, ends)]
    gemm_ms_total = sum(launch_ms)
    region_ms = region_s.elapsed_time(region_e)
    t = torch.tensor([gemm_ms_total, region_ms], dtype=torch.float64, device=dev)
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    gemm_ms_max, region_ms_max = float(t[0]), float(t[1])

    flops_step = 2 * M * N * K
    value = flops_step * world * args.steps / (gemm_ms_max * 1e-3) / 1e12
    ms_per_step = gemm_ms_max / args.steps

    # e2e through the C ABI with host buffers, every rank
    e2e = None
    if not args.no_extras:
        e_ms, h2d, d2h, same = e2e_measure_host(A, Bt, stream)
        s_ms, _, _ = e2e_measure(gemm_ours, A, Bt, stream)
        f_ms = link_floor_ms(h2d, d2h, dev)
        et = torch.tensor([e_ms, s_ms, f_ms], dtype=torch.float64, device=dev)
        if world > 1:
            dist.all_reduce(et, op=dist.ReduceOp.MAX)
        e2e = {"value": flops_step * world / (float(et[0]) * 1e-3) / 1e12, "unit": "TFLOP/s",
               "h2d_bytes_per_step": h2d * world, "d2h_bytes_per_step": d2h * world,
               "ms_per_step": float(et[0]),
               "path": "capi.gemm_bf16_host (b200_gemm_bf16_host) with pinned host A, B and C: "
                       "A and B uploaded in alternating blocks, each block of C computed once "
                       "its two blocks are up and downloaded once done, uploads / GEMMs / "
                       "downloads overlapped on three streams",
               "link_floor": {"ms_per_step": float(et[2]),
                              "value": flops_step * world / (float(et[2]) * 1e-3) / 1e12,
                              "frac": float(et[2]) / float(et[0]),
                              "what": "the step's upload and download bytes copied at once on "
                                      "two streams (pinned memory), no GEMM: the PCIe floor"},
               "parity": same,
               "serial_copies": {"value": flops_step * world / (float(et[1]) * 1e-3) / 1e12,
                                 "ms_per_step": float(et[1]),
                                 "path": "H2D A, B; b200_gemm_bf16; D2H C on one stream"}}

    peaks, peak_src = measured_peaks()
    traffic, traffic_src = profiled_traffic()
    mean_launch_ms = statistics.mean(launch_ms)
    achieved = flops_step / (mean_launch_ms * 1e-3) / 1e12
    roofline = {"bound": "tensor", "achieved": achieved, "peak": peaks["bf16_tflops"],
                "unit": "TFLOP/s", "frac": achieved / peaks["bf16_tflops"],
                "traffic": traffic,
                "peak_source": f"{peak_src} (bf16 burst: kernel timed alone)",
                "algorithmic_flops_per_launch": flops_step,
                "algorithmic_bytes_per_launch": 2 * (M * K + N * K + M * N),
                "traffic_source": traffic_src}

    extras = {}
    if rank == 0 and world == 1 and not args.no_extras:
        ref_ms = {}
        try:
            Cr = torch.empty_like(C)
            for v in reference_versions(M, N, K):
                ref_ms[v] = statistics.median(time_cold(
                    lambda: gemm_reference(A, Bt, Cr, stream, v), 50, 10, stream, flush))
        except Exception as e:  # the reference build may be absent
            extras["reference_error"] = repr(e)
        cub_ms = statistics.median(time_cold(lambda: torch.matmul(A, Bt.T), 50, 10, stream, flush))
        ours_med = statistics.median(time_cold(lambda: gemm_ours(A, Bt, C, stream), 50, 10, stream,
                                               flush))
        tf = lambda ms: flops_step / (ms * 1e-3) / 1e12
        best = min(ref_ms, key=ref_ms.get) if ref_ms else None
        extras["baselines"] = {
            "ours_median_tflops": tf(ours_med),
            "cublas_median_tflops": tf(cub_ms),
            "reference_v8_median_tflops": tf(ref_ms["v8"]) if "v8" in ref_ms else None,
            "reference_versions_median_tflops": {v: tf(t) for v, t in ref_ms.items()},
            "reference_best": {"version": best, "median_tflops": tf(ref_ms[best])} if best else None,
            "ours_vs_cublas": cub_ms / ours_med,
            "ours_vs_reference_best": (ref_ms[best] / ours_med) if best else None,
            "method": "median of 50 cold-L2 launches each after 1 s idle and 10 warm-up "
                      "launches, same process and inputs (src/bench_core.py:47-69 method); "
                      "every reference version that supports the shape "
                      "(src/main.py:154-158 times each)"}
        extras["cpu_baseline"] = cpu_baseline(Bt)

    if rank == 0:
        line = {
            "metric": "BF16 GEMM TFLOP/s (cold-L2) at 8192^3 per GPU",
            "value": value, "unit": "TFLOP/s", "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": ms_per_step, "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": "bf16", "data": "synthetic",
            "config": {"workload": "bf16 GEMM C = A B^T, 8192 x 8192 x 8192 per GPU "
                                   "(rows of A sharded, B replicated, no collective)",
                       "M": M * world, "N": N, "K": K, "m_per_gpu": M,
                       "inputs": "A, B iid N(0,1) bf16, seeded, resident in HBM",
                       "l2": "flushed: 256 MB written before every step, outside the GEMM events",
                       "parallelism": f"m-shard{world}"},
            "timed_region_ms": region_ms_max,
            "step_ms": step_stats(launch_ms),
            "gpu_launches": args.steps,
            "roofline": roofline,
            "e2e": e2e,
            "clocks": clocks.report(),
            "parity": par,
            "impl": "ours",
            "kernel": {"pair_tile": "256x512" if shape["threads"] // 32 > 6 else "256x256",
                       "threads": shape["threads"], "grid": shape["grid"],
                       "smem_bytes": shape["smem_bytes"], "tuning": tuning},
        }
        line.update(extras)
    # Per-rank spread of the headline: each rank's median step time and
    # median SM clock name the slowest rank that sets the max over ranks.
    mine = {"rank": rank, "median_ms": statistics.median(launch_ms),
            "sm_mhz": clocks.report()["sm_mhz"]}
    per_rank = [mine]
    if world > 1:
        per_rank = [None] * world
        dist.all_gather_object(per_rank, mine)
    # The two large multi-GPU configurations, measured at every N (N = 1
    # included, so the lines of a scaling run give their curves).
    more = {}
    if not args.no_extras:
        del C
        torch.cuda.empty_cache()
        more["m_shard_131072"] = extra_m_shard(args, world, rank, dev, Bt, flush, stream)
        torch.cuda.empty_cache()
        more["ksplit"] = extra_ksplit(args, world, rank, dev, flush, stream)
    if rank == 0:
        line["per_rank"] = per_rank
        line.update(more)
        print(json.dumps(line), flush=True)
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()


def extra_steps(args) -> int:
    """Timed steps of the side measurements: at most 20, at least 5."""
    return max(5, min(args.steps, 20))


def max_over_ranks(values, world, dev):
    """Element-wise max over ranks of a list of floats."""
    t = torch.tensor(values, dtype=torch.float64, device=dev)
    if world > 1:
        import torch.distributed as dist
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return [float(v) for v in t]


def timed_cold_steps(step, steps, warmup, stream, flush, world):
    """Cold-L2 steps between barriers: warm-up, then `steps` steps each
    bracketed by CUDA events on `stream`.  Returns this rank's per-step ms."""
    import torch.distributed as dist
    step()
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    time.sleep(IDLE_BEFORE_ARM_S)
    for _ in range(warmup):
        flush.zero_()
        step()
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    starts, ends = cold_l2_loop(step, steps, stream, flush)
    wait_event(ends[-1])
    if world > 1:
        dist.barrier()
    return [a.elapsed_time(b) for a, b in zip(starts, ends)]


def extra_m_shard(args, world, rank, dev, Bt, flush, stream):
    """Configuration 5a as stated: M = 131072 rows in total, split over the N
    ranks (strong scaling: rank r owns 131072 / N rows of A, B replicated, no
    collective).  Value = all ranks' FLOPs / the slowest rank's summed GEMM
    time.  At N > 1 rank 0 also times the whole 131072-row problem alone in
    the same job (the 1-GPU point of the curve), and the line gives the
    strong-scaling efficiency against it.  Parity on sampled rows of every
    rank (max of the metrics over ranks)."""
    from blackwell_gemm_b200 import parity as par_mod
    from blackwell_gemm_b200.workloads import M_SHARD, make_operands
    M, N, K = M_SHARD
    rows = M // world
    steps = extra_steps(args)
    A, _ = make_operands(rows, 8, K, seed=5000 + rank, device=dev)
    C = torch.empty(rows, N, dtype=torch.bfloat16, device=dev)
    ms = timed_cold_steps(lambda: gemm_ours(A, Bt, C, stream), steps, 3, stream, flush, world)
    par = parity_sample(C, A, Bt)
    total, mx_scaled, mx_fro, fail = max_over_ranks(
        [sum(ms), par["max_scaled"], par["rel_fro"], 0.0 if par["pass"] else 1.0], world, dev)
    flops = 2 * M * N * K
    out = {"value": flops * steps / (total * 1e-3) / 1e12, "unit": "TFLOP/s",
           "ms_per_step": total / steps, "steps": steps, "scaling": "strong",
           "config": {"M": M, "N": N, "K": K, "rows_per_gpu": rows,
                      "inputs": "A (each rank's rows), B iid N(0,1) bf16, seeded, resident in HBM",
                      "l2": "flushed: 256 MB written before every step"},
           "parity": {"max_scaled": mx_scaled, "rel_fro": mx_fro, "pass": fail == 0.0,
                      "rows_checked": 256 * world, "combined": "max over ranks"}}
    del A, C
    if world > 1:
        import torch.distributed as dist
        one = torch.zeros(1, dtype=torch.float64, device=dev)
        if rank == 0:
            # the whole problem on one GPU, in the same job (others wait)
            torch.cuda.empty_cache()
            Af, _ = make_operands(M, 8, K, seed=5000, device=dev)
            Cf = torch.empty(M, N, dtype=torch.bfloat16, device=dev)
            s1 = max(3, steps // 4)
            ms1 = timed_cold_steps(lambda: gemm_ours(Af, Bt, Cf, stream), s1, 3, stream, flush, 1)
            one[0] = flops * s1 / (sum(ms1) * 1e-3) / 1e12
            del Af, Cf
        dist.barrier()
        dist.broadcast(one, 0)
        out["one_gpu_same_job"] = {"value": float(one[0]), "unit": "TFLOP/s",
                                   "what": "rank 0 alone on all 131072 rows, same job"}
        out["strong_scaling_efficiency"] = out["value"] / (world * float(one[0]))
    return out


def extra_ksplit(args, world, rank, dev, flush, stream):
    """Configuration 5b: C = A B^T with M = N = 8192 and K = 131072 split over
    the N ranks (strong scaling).  The fused kernel (b200_ksplit_gemm_bf16:
    the other owners' fp32 tiles written into their memory over NVLink while
    the GEMM runs, own rows summed and rounded in the epilogue) is timed
    beside the unfused sequence (b200_gemm_bf16_f32out, NCCL
    reduce_scatter_tensor(sum), b200_cast_f32_bf16), same inputs, cold L2,
    max over ranks.  Parity of the fused output on sampled rows of every
    owner against an fp32 GEMM over the whole K (distributed.
    k_split_sampled_parity), and the device error word after the calls."""
    import torch.distributed as dist
    from blackwell_gemm_b200 import capi
    from blackwell_gemm_b200 import distributed as bdist
    from blackwell_gemm_b200.workloads import K_SPLIT, make_operands
    M, N, K = K_SPLIT
    Kr = K // world
    steps = extra_steps(args)
    group = dist.group.WORLD if world > 1 else None
    A, _ = make_operands(M, 8, Kr, seed=2000 + rank, device=dev)
    _, Bk = make_operands(8, N, Kr, seed=3000 + rank, device=dev)
    fused = bdist.FusedKSplit(M, N, group)
    out = torch.empty(M // world, N, dtype=torch.bfloat16, device=dev)
    try:
        def step_fused():
            fused(A, Bk, out)

        def step_unfused():
            partial = bdist.gemm_f32_cuda(A, Bk)
            if world > 1:
                rs = torch.empty(M // world, N, dtype=torch.float32, device=dev)
                dist.reduce_scatter_tensor(rs, partial, op=dist.ReduceOp.SUM, group=group)
            else:
                rs = partial
            return bdist.cast_bf16_cuda(rs)

        ms_unf = timed_cold_steps(step_unfused, steps, 3, stream, flush, world)
        ms_fused = timed_cold_steps(step_fused, steps, 3, stream, flush, world)
        torch.cuda.synchronize()
        status = capi.device_status(True)
        fused(A, Bk, out)        # a fresh result for the parity check
        torch.cuda.synchronize()
        par = bdist.k_split_sampled_parity(out, A, Bk, group)
        status2 = capi.device_status(True)
    finally:
        torch.cuda.synchronize()
        fused.close()
    t_fused, t_unf, st = max_over_ranks([sum(ms_fused), sum(ms_unf), float(max(status, status2))],
                                        world, dev)
    flops = 2 * M * N * K
    tf = lambda t: flops * steps / (t * 1e-3) / 1e12
    return {"value": tf(t_fused), "unit": "TFLOP/s", "ms_per_step": t_fused / steps,
            "steps": steps, "scaling": "strong",
            "config": {"M": M, "N": N, "K": K, "k_per_gpu": Kr,
                       "inputs": "each rank's K-slices of A and B, iid N(0,1) bf16, seeded",
                       "l2": "flushed: 256 MB written before every step"},
            "path": "b200_ksplit_gemm_bf16: one kernel per rank, peers' fp32 tiles over "
                    "NVLink (CUDA IPC, plain stores), own rows summed and rounded once",
            "unfused_nccl": {"value": tf(t_unf), "ms_per_step": t_unf / steps,
                             "what": "b200_gemm_bf16_f32out + NCCL reduce_scatter_tensor(sum) "
                                     "+ b200_cast_f32_bf16" if world > 1 else
                                     "b200_gemm_bf16_f32out + b200_cast_f32_bf16 (one rank)"},
            "fused_vs_unfused": t_unf / t_fused,
            "nvlink_bytes_per_rank_per_step": (world - 1) * (M // world) * N * 4,
            "device_status": int(st), "parity": par}


def run_ksplit(args, world, rank, dev):
    """Configuration 5b: C = A B^T with M = N = 8192 and K = 131072 split
    across the ranks (strong scaling).  One step of the headline arm = one
    fused kernel per rank (b200_ksplit_gemm_bf16: this rank's K-slice, the
    other owners' fp32 tiles written into their memory over NVLink while it
    computes, its own rows summed and rounded in the epilogue).  The unfused
    sequence -- fp32 partial (b200_gemm_bf16_f32out), NCCL reduce-scatter
    (sum), bf16 cast -- is timed the same way beside it.  CUDA events around
    each step, max over ranks."""
    import torch.distributed as dist
    from datetime import timedelta
    if world > 1:
        dist.init_process_group("nccl", timeout=timedelta(seconds=120), device_id=dev)
    from blackwell_gemm_b200 import distributed as bdist
    from blackwell_gemm_b200.workloads import K_SPLIT, make_operands
    M, N, K = K_SPLIT
    Kr = K // world
    A, _ = make_operands(M, 8, Kr, seed=2000 + rank, device=dev)
    _, Bt = make_operands(8, N, Kr, seed=3000 + rank, device=dev)
    flush = torch.empty(FLUSH_BYTES // 4, dtype=torch.int32, device=dev)
    stream = torch.cuda.current_stream()
    group = dist.group.WORLD if world > 1 else None
    fused = bdist.FusedKSplit(M, N, group)
    out = torch.empty(M // world, N, dtype=torch.bfloat16, device=dev)

    def step_fused():
        return fused(A, Bt, out)

    def step_nccl():
        partial = bdist.gemm_f32_cuda(A, Bt)
        if world > 1:
            rs = torch.empty(M // world, N, dtype=torch.float32, device=dev)
            dist.reduce_scatter_tensor(rs, partial, op=dist.ReduceOp.SUM, group=group)
        else:
            rs = partial
        return bdist.cast_bf16_cuda(rs)

    def timed(step):
        step()
        torch.cuda.synchronize()
        if world > 1:
            dist.barrier()
        time.sleep(IDLE_BEFORE_ARM_S)
        for _ in range(args.warmup):
            flush.zero_()
            step()
        torch.cuda.synchronize()
        if world > 1:
            dist.barrier()
        starts, ends = cold_l2_loop(step, args.steps, stream, flush)
        wait_event(ends[-1])
        if world > 1:
            dist.barrier()
        ms = [a.elapsed_time(b) for a, b in zip(starts, ends)]
        t = torch.tensor([sum(ms)], dtype=torch.float64, device=dev)
        if world > 1:
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t[0]), ms

    # The unfused sequence first, then the fused kernel (headline).
    nccl_ms, _ = timed(step_nccl)
    clocks = ClockSampler(dev.index)
    clocks.start()
    total_ms, ms = timed(step_fused)
    clocks.stop()
    clk = clocks.report()
    from blackwell_gemm_b200 import capi
    status = capi.device_status(True)
    fused.close()
    flops = 2 * M * N * K
    tf = flops * args.steps / (total_ms * 1e-3) / 1e12
    peaks, src = measured_peaks()
    peak = float(peaks.get("bf16_tflops", FALLBACK_BF16_TFLOPS))
    # fp32 bytes each rank sends over NVLink per step: (P-1)/P of its M x N partial
    link_bytes = (world - 1) * (M // world) * N * 4
    if rank == 0:
        print(json.dumps({
            "metric": "BF16 GEMM TFLOP/s (cold-L2), K-split 8192 x 8192 x 131072",
            "value": tf, "unit": "TFLOP/s",
            "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": total_ms / args.steps, "higher_is_better": True, "scaling": "strong",
            "vs_baseline": None, "dtype": "bf16", "data": "synthetic",
            "config": {"workload": "K-split GEMM, fused: per-rank K-slice GEMM whose epilogue "
                                   "sends other owners' fp32 tiles over NVLink and sums + "
                                   "rounds its own rows (one kernel per rank)",
                       "M": M, "N": N, "K": K, "k_per_gpu": Kr,
                       "l2": "flushed: 256 MB written before every step",
                       "parallelism": f"k-split{world}"},
            "roofline": {"bound": "tensor", "achieved": tf / world, "peak": peak,
                         "unit": "TFLOP/s", "frac": tf / world / peak,
                         "peak_source": src, "per": "GPU",
                         "nvlink_bytes_per_rank_per_step": link_bytes},
            "unfused_nccl": {"value": flops * args.steps / (nccl_ms * 1e-3) / 1e12,
                             "ms_per_step": nccl_ms / args.steps,
                             "what": "b200_gemm_bf16_f32out + NCCL reduce_scatter_tensor(sum) "
                                     "+ b200_cast_f32_bf16"},
            "clocks": clk, "device_status": status,
            "step_ms": step_stats(ms), "impl": "ours", "gpu_launches": args.steps,
            "parity": "tests/test_ksplit_fused_gpu.py",
        }), flush=True)
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()


def run_sweep(args, world, rank, dev):
    """Every single-GPU configuration shape (workloads.CONFIGS: 1024^3, the
    square sweep, the transformer projections, the skinny decode shapes), one
    JSON line each on rank 0: cold-L2 medians of ours, cuBLAS and the
    reference's v8 (where it supports the shape) in the same process, the
    roofline fraction (tensor peak, or HBM for the skinny shapes) and parity on
    sampled rows.  Not the driver's bench line; the evidence for the configs."""
    if rank != 0:
        return
    import oracle
    from blackwell_gemm_b200 import workloads
    from blackwell_gemm_b200.workloads import CONFIGS, WEIGHT_STD, make_operands
    peaks, src = measured_peaks()
    peak_tf = float(peaks.get("bf16_tflops", FALLBACK_BF16_TFLOPS))
    peak_gbs = float(peaks.get("hbm_gbs", 6650.0))
    flush = torch.empty(FLUSH_BYTES // 4, dtype=torch.int32, device=dev)
    clean = torch.ones(FLUSH_BYTES // 4, dtype=torch.int32, device=dev)
    stream = torch.cuda.current_stream()
    steps = max(10, min(args.steps, 50))
    if args.shapes:
        custom = [tuple(int(v) for v in sh.lower().split("x")) for sh in args.shapes.split(",")]
        groups = [("skinny" if M <= 256 else "shape", [(M, N, K)]) for M, N, K in custom]
    else:
        groups = [(name, CONFIGS[name]) for name in ("square_1024", "square", "projection", "skinny")]
    # What any kernel costs under this protocol: a one-block add after the
    # flush (launch and completion), reported beside the small shapes.
    tiny = torch.zeros(16, device=dev)
    floor_us = statistics.median(time_cold(lambda: tiny.add_(1), steps, args.warmup, stream,
                                           flush)) * 1e3
    for name, shapes in groups:
        for (M, N, K) in shapes:
            std = WEIGHT_STD.get(name, WEIGHT_STD["skinny"] if M <= 256 else WEIGHT_STD["square"])
            A, Bt = make_operands(M, N, K, seed=M + N + K, weight_std=std, device=dev)
            C = torch.empty(M, N, dtype=torch.bfloat16, device=dev)
            gemm_ours(A, Bt, C, stream)
            torch.cuda.synchronize()
            par = parity_sample(C, A, Bt)
            med = lambda fn: statistics.median(time_cold(fn, steps, args.warmup, stream, flush))
            ours = med(lambda: gemm_ours(A, Bt, C, stream))
            cub = med(lambda: torch.matmul(A, Bt.T))
            refs = {}
            if args.ref_versions != "none":
                want = reference_versions(M, N, K)
                if args.ref_versions == "v8":
                    want = [v for v in want if v == "v8"]
                Cr = torch.empty_like(C)
                for v in want:
                    try:
                        refs[v] = med(lambda: gemm_reference(A, Bt, Cr, stream, v))
                    except Exception:
                        pass
            best = min(refs, key=refs.get) if refs else None
            ref = refs.get(best)
            fl = workloads.flops(M, N, K)
            by = workloads.min_bytes(M, N, K)
            tf = lambda ms: fl / (ms * 1e-3) / 1e12
            hbm = name == "skinny"
            achieved = by / (ours * 1e-3) / 1e9 if hbm else tf(ours)
            probe = clean_l2 = None
            if hbm:
                # A plain read of B's N x K bf16 (torch's sum, fp32 accumulation)
                # under the same protocol: the HBM rate a library kernel gets for
                # these bytes after the flush, launch and completion included.
                pr = med(lambda: Bt.sum(dtype=torch.float32))
                probe = {"what": "torch sum over B (N x K bf16), same protocol",
                         "us": pr * 1e3, "gbs": 2 * N * K / (pr * 1e-3) / 1e9,
                         "ours_vs_probe": pr / ours}
                # The same three calls after a flush that leaves L2 clean.
                cmed = lambda fn: statistics.median(
                    time_clean(fn, steps, args.warmup, stream, flush, clean))
                c_ours = cmed(lambda: gemm_ours(A, Bt, C, stream))
                c_cub = cmed(lambda: torch.matmul(A, Bt.T))
                c_pr = cmed(lambda: Bt.sum(dtype=torch.float32))
                clean_l2 = {"flush": "256 MB written, then another 256 MB read",
                            "ours_us": c_ours * 1e3, "cublas_us": c_cub * 1e3,
                            "sum_b_us": c_pr * 1e3, "ours_vs_cublas": c_cub / c_ours,
                            "ours_gbs": by / (c_ours * 1e-3) / 1e9,
                            "ours_frac": by / (c_ours * 1e-3) / 1e9 / peak_gbs}
            print(json.dumps({
                "config": name, "M": M, "N": N, "K": K, "ours_us": ours * 1e3,
                "ours_tflops": tf(ours), "cublas_tflops": tf(cub),
                "reference_v8_tflops": tf(refs["v8"]) if "v8" in refs else None,
                "reference_best": {"version": best, "tflops": tf(ref)} if ref else None,
                "reference_versions_tflops": {v: tf(t) for v, t in refs.items()},
                "ours_vs_cublas": cub / ours,
                "ours_vs_reference_v8": (refs["v8"] / ours) if "v8" in refs else None,
                "ours_vs_reference_best": (ref / ours) if ref else None,
                "roofline": {"bound": "hbm" if hbm else "tensor", "achieved": achieved,
                             "peak": peak_gbs if hbm else peak_tf,
                             "unit": "GB/s" if hbm else "TFLOP/s",
                             "frac": achieved / (peak_gbs if hbm else peak_tf),
                             "peak_source": src},
                "hbm_read_probe": probe,
                "clean_l2": clean_l2,
                "launch_floor_us": floor_us,
                "parity": par, "timing": f"median of {steps} cold-L2 launches (256 MB flush "
                                          "between), same process, 1 s idle before each arm",
            }), flush=True)


def run_reference(args, world, rank, dev):
    """The reference's own implementation of the path: its matmul_v8 kernel
    (src/kernels/kernel_v8.cu:830-833), built from its sources into
    oracle/_ref by oracle/build.py and called through its launcher.  The
    reference has no CPU implementation; this GPU kernel is it.  It is
    single-GPU, so it runs one process per GPU (its tile-table cache is
    device-blind, kernel_v8.cu:796-820): under torchrun every rank runs it on
    its own 8192-row block of A with the replicated B -- the same row-sharded
    workload and seeds as our arm -- and the per-rank summed GEMM time is
    maxed over ranks, as for our arm, so the two lines compare like for like
    at every N.  Rank 0 prints the line."""
    import torch.distributed as dist
    if world > 1:
        from datetime import timedelta
        dist.init_process_group("nccl", timeout=timedelta(seconds=120), device_id=dev)
    try:
        import oracle
        oracle.ref_lib()
        missing = None
    except Exception as e:
        missing = f"reference build oracle/_ref missing: {e}"
    flag = torch.tensor([1.0 if missing else 0.0], device=dev)
    if world > 1:
        dist.all_reduce(flag, op=dist.ReduceOp.MAX)
    if float(flag[0]) > 0:
        if rank == 0:
            print(json.dumps({"impl": "reference", "unavailable": missing or
                              "reference build missing on another rank"}), flush=True)
        if world > 1:
            dist.destroy_process_group()
        return
    from blackwell_gemm_b200.workloads import make_operands
    M, N, K = M_PER_GPU, N_DIM, K_DIM
    A, _ = make_operands(M, 8, K, seed=1000 + rank, device=dev)
    _, Bt = make_operands(8, N, K, seed=0, device=dev)
    C = torch.empty(M, N, dtype=torch.bfloat16, device=dev)
    flush = torch.empty(FLUSH_BYTES // 4, dtype=torch.int32, device=dev)
    stream = torch.cuda.current_stream()
    gemm_reference(A, Bt, C, stream)
    torch.cuda.synchronize()
    par = parity_sample(C, A, Bt)
    torch.cuda.synchronize()
    time.sleep(IDLE_BEFORE_ARM_S)
    for _ in range(args.warmup):
        flush.zero_()
        gemm_reference(A, Bt, C, stream)
    clocks = ClockSampler(dev.index)
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    clocks.start()
    starts, ends = cold_l2_loop(lambda: gemm_reference(A, Bt, C, stream), args.steps, stream,
                                flush)
    wait_event(ends[-1])
    if world > 1:
        dist.barrier()
    clocks.stop()
    launch_ms = [a.elapsed_time(b) for a, b in zip(starts, ends)]
    flops_step = 2 * M * N * K
    e_ms, h2d, d2h = e2e_measure(gemm_reference, A, Bt, stream)
    total, e_max, mx_scaled, mx_fro, fail = max_over_ranks(
        [sum(launch_ms), e_ms, par["max_scaled"], par["rel_fro"], 0.0 if par["pass"] else 1.0],
        world, dev)
    mine = {"rank": rank, "median_ms": statistics.median(launch_ms),
            "sm_mhz": clocks.report()["sm_mhz"]}
    per_rank = [mine]
    if world > 1:
        per_rank = [None] * world
        dist.all_gather_object(per_rank, mine)
    value = flops_step * world * args.steps / (total * 1e-3) / 1e12
    if rank == 0:
        line = {
            "metric": "BF16 GEMM TFLOP/s (cold-L2) at 8192^3 per GPU",
            "value": value, "unit": "TFLOP/s", "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": total / args.steps, "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": "bf16", "data": "synthetic",
            "config": {"workload": "bf16 GEMM C = A B^T, 8192 x 8192 x 8192 per GPU "
                                   "(rows of A sharded, B replicated, no collective; the "
                                   "reference's v8 in one process per GPU)",
                       "M": M * world, "N": N, "K": K, "m_per_gpu": M,
                       "inputs": "A, B iid N(0,1) bf16, seeded, resident in HBM",
                       "l2": "flushed: 256 MB written before every step, outside the GEMM events",
                       "parallelism": f"m-shard{world}"},
            "impl": "reference",
            "cpu_baseline": {"value": value, "unit": "TFLOP/s", "cores": 0, "kind": "reference",
                             "sample": "the reference's matmul_v8 GPU kernel on the full "
                                       "workload (the reference has no CPU implementation of "
                                       "the path)"},
            "e2e": {"value": flops_step * world / (e_max * 1e-3) / 1e12, "unit": "TFLOP/s",
                    "h2d_bytes_per_step": h2d * world, "d2h_bytes_per_step": d2h * world,
                    "ms_per_step": e_max,
                    "path": "reference matmul_v8 launcher with pinned host A, B and C, serial "
                            "copies, every rank (max over ranks)"},
            "gpu_launches": 0,
            "step_ms": step_stats(launch_ms),
            "per_rank": per_rank,
            "clocks": clocks.report(),
            "parity": {"max_scaled": mx_scaled, "rel_fro": mx_fro, "pass": fail == 0.0,
                       "rows_checked": 256 * world, "combined": "max over ranks"},
        }
        print(json.dumps(line), flush=True)
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
