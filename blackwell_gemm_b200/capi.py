"""ctypes binding of the C ABI in ``include/b200_gemm.h`` (libb200gemm.so).

This is the boundary the parity tests and the end-to-end bench call: plain
pointers, sizes and a stream handle, a status code back.  Loading fails
loudly when the library has not been built -- there is no fallback.
"""
from __future__ import annotations

import ctypes
from pathlib import Path

LIB_PATH = Path(__file__).resolve().parent / "libb200gemm.so"

# Status codes (include/b200_gemm.h).
OK = 0
ERR_INVALID_ARGUMENT = 1
ERR_ALIGNMENT = 2
ERR_UNSUPPORTED_DEVICE = 3
ERR_TENSOR_MAP = 4
ERR_LAUNCH = 5
ERR_DEVICE_TIMEOUT = 6
ERR_TOO_LARGE = 7

# Device error-word values written by a pipeline wait that ran out.
DEVICE_WAIT_CODES = {
    0x1001: "producer wait on a ring slot",
    0x1002: "MMA wait on TMA data",
    0x1003: "MMA wait on the epilogue",
    0x1004: "epilogue wait on the MMA",
    0x1005: "final MMA drain",
    0x1006: "wait probe",
    0x1007: "K-split: a peer's piece of an own tile never arrived",
    0x1008: "stream-K: an earlier CTA's partial tile never arrived",
    0x1009: "dynamic dealing: a slot of the pair's unit ring",
}

KSPLIT_HANDLE_BYTES = 128

# Every symbol the header declares, with (restype, argtypes).
_vp, _i, _u32, _u64, _ull = ctypes.c_void_p, ctypes.c_int, ctypes.c_uint32, ctypes.c_uint64, \
    ctypes.c_ulonglong
_ip = ctypes.POINTER(ctypes.c_int)
SIGNATURES = {
    "b200_gemm_bf16": (_i, [_vp, _vp, _vp, _i, _i, _i, _i, _i, _i, _vp]),
    "b200_gemm_bf16_profile": (_i, [_vp, _vp, _vp, _i, _i, _i, _i, _i, _i, _vp, _i, _vp]),
    "b200_gemm_bf16_f32out": (_i, [_vp, _vp, _vp, _i, _i, _i, _i, _i, _i, _vp]),
    "b200_gemm_bf16_noalloc": (_i, [_vp, _vp, _vp, _i, _i, _i, _i, _i, _i, _vp]),
    "b200_gemm_noalloc_status": (_i, [_i, _ip]),
    "b200_gemm_noalloc_wait_probe": (_i, [_ull, _vp]),
    "b200_cast_f32_bf16": (_i, [_vp, _i, _vp, _i, _i, _i, _vp]),
    "b200_gemm_bf16_host": (_i, [_vp, _vp, _vp, _i, _i, _i, _i, _i, _i, _i, _vp]),
    "b200_gemm_bf16_epilogue": (_i, [_vp, _vp, _vp, _i, _i, _i, _i, _i, _i, ctypes.c_float, _vp,
                                     ctypes.c_float, _vp, _i, _vp]),
    "b200_gemm_set_splits": (_i, [_i]),
    "b200_gemm_set_skinny_mode": (_i, [_i]),
    "b200_gemm_set_skinny_tiles": (_i, [_i]),
    "b200_gemm_set_stream_k": (_i, [_i]),
    "b200_gemm_set_dynamic": (_i, [_i]),
    "b200_gemm_get_splits": (_i, [_i, _i, _i, _ip]),
    "b200_gemm_profile_rows": (_i, [_i, _i, _i, _ip]),
    "b200_gemm_device_status": (_i, [_i, _ip]),
    "b200_gemm_set_wait_timeout_ns": (_i, [_ull]),
    "b200_gemm_set_tuning": (_i, [_i, _i, _i]),
    "b200_gemm_get_tuning": (_i, [_ip, _ip, _ip]),
    "b200_gemm_wait_probe": (_i, [_ull, _vp]),
    "b200_gemm_status_string": (ctypes.c_char_p, [_i]),
    "b200_gemm_tile_coord": (None, [_i, _i, _i, _i, _ip, _ip]),
    "b200_gemm_idesc": (_u32, [_i, _i]),
    "b200_gemm_sk_range_pairs": (_i, [ctypes.c_longlong, _i]),
    "b200_gemm_sk_range": (None, [_i, ctypes.c_longlong, _i, ctypes.POINTER(ctypes.c_longlong),
                                  ctypes.POINTER(ctypes.c_longlong)]),
    "b200_gemm_sk_owner": (_i, [ctypes.c_longlong, ctypes.c_longlong, _i]),
    "b200_gemm_sk_next_segment": (None, [ctypes.c_longlong, ctypes.POINTER(ctypes.c_longlong), _i,
                                         _ip, _ip, _ip]),
    "b200_gemm_smem_desc": (_u64, [_u32]),
    "b200_gemm_launch_shape": (_i, [_i, _i, _i, _ip, _ip, _ip, _ip]),
    "b200_ksplit_create": (_i, [_i, _i, _i, _i, ctypes.POINTER(_vp), _vp]),
    "b200_ksplit_connect": (_i, [_vp, _vp]),
    "b200_ksplit_gemm_bf16": (_i, [_vp, _vp, _vp, _vp, _i, _i, _i, _i, _i, _i, _vp]),
    "b200_ksplit_epoch": (_i, [_vp, ctypes.POINTER(ctypes.c_uint)]),
    "b200_ksplit_destroy": (_i, [_vp]),
}

_lib = None


class GemmError(RuntimeError):
    def __init__(self, status: int, what: str = "b200_gemm"):
        self.status = status
        super().__init__(f"{what}: {status_string(status)} (status {status})")


def lib() -> ctypes.CDLL:
    global _lib
    if _lib is None:
        if not LIB_PATH.exists():
            raise ImportError(f"{LIB_PATH.name} is not built; run `python -m blackwell_gemm_b200.build`")
        handle = ctypes.CDLL(str(LIB_PATH))
        for name, (res, args) in SIGNATURES.items():
            fn = getattr(handle, name)
            fn.restype = res
            fn.argtypes = args
        _lib = handle
    return _lib


def status_string(status: int) -> str:
    return lib().b200_gemm_status_string(int(status)).decode()


def check(status: int, what: str = "b200_gemm") -> None:
    if status != OK:
        raise GemmError(status, what)


def gemm_bf16(a_ptr: int, b_ptr: int, c_ptr: int, M: int, N: int, K: int, lda: int, ldb: int,
              ldc: int, stream: int = 0) -> int:
    """Raw C-ABI call: returns the status code (does not raise)."""
    return lib().b200_gemm_bf16(a_ptr, b_ptr, c_ptr, M, N, K, lda, ldb, ldc, stream)


def gemm_bf16_f32out(a_ptr: int, b_ptr: int, c_ptr: int, M: int, N: int, K: int, lda: int,
                     ldb: int, ldc: int, stream: int = 0) -> int:
    """fp32 C = A * B^T (no rounding); ldc in floats.  Returns the status."""
    return lib().b200_gemm_bf16_f32out(a_ptr, b_ptr, c_ptr, M, N, K, lda, ldb, ldc, stream)


def gemm_bf16_epilogue(a_ptr, b_ptr, c_ptr, M, N, K, lda, ldb, ldc, alpha, bias_ptr, beta,
                       resid_ptr, ldr, stream=0) -> int:
    """C = round(alpha A B^T + bias + beta R); bias_ptr / resid_ptr may be 0."""
    return lib().b200_gemm_bf16_epilogue(a_ptr, b_ptr, c_ptr, M, N, K, lda, ldb, ldc,
                                         float(alpha), bias_ptr or None, float(beta),
                                         resid_ptr or None, ldr, stream)


def gemm_bf16_host(a_ptr: int, b_ptr: int, c_ptr: int, M: int, N: int, K: int, lda: int,
                   ldb: int, ldc: int, block_rows: int = 0, stream: int = 0) -> int:
    """b200_gemm_bf16_host: host pointers (pinned for overlap), asynchronous on
    `stream`."""
    return lib().b200_gemm_bf16_host(a_ptr, b_ptr, c_ptr, M, N, K, lda, ldb, ldc, block_rows,
                                     stream)


def cast_f32_bf16(w_ptr: int, ldw: int, c_ptr: int, ldc: int, M: int, N: int,
                  stream: int = 0) -> int:
    return lib().b200_cast_f32_bf16(w_ptr, ldw, c_ptr, ldc, M, N, stream)


def gemm_bf16_noalloc(a_ptr: int, b_ptr: int, c_ptr: int, M: int, N: int, K: int, lda: int,
                      ldb: int, ldc: int, stream: int = 0) -> int:
    """b200_gemm_bf16 without any device allocation (fixed 16 MiB scratch in
    the library; overlapping calls race; timeouts are read with
    noalloc_status).  Returns the status."""
    return lib().b200_gemm_bf16_noalloc(a_ptr, b_ptr, c_ptr, M, N, K, lda, ldb, ldc, stream)


def noalloc_status(clear: bool = True) -> int:
    """Error word of the allocation-free entry point's array (sticky until
    cleared); synchronises the device."""
    v = ctypes.c_int(0)
    check(lib().b200_gemm_noalloc_status(1 if clear else 0, ctypes.byref(v)), "noalloc_status")
    return v.value


def noalloc_wait_probe(timeout_ns: int, stream: int = 0) -> int:
    """The wait self-test, recording into the allocation-free array's word."""
    return lib().b200_gemm_noalloc_wait_probe(int(timeout_ns), stream)


def set_splits(splits: int) -> None:
    check(lib().b200_gemm_set_splits(int(splits)), "set_splits")


def set_stream_k(mode: int) -> None:
    """0 off, 1 when the last wave is short (default), 2 whenever it is partial."""
    check(lib().b200_gemm_set_stream_k(mode), "b200_gemm_set_stream_k")


def set_skinny_tiles(tiles: int) -> None:
    """Blocks of B per skinny stream-K tile: 1, 2, or 0 (chosen)."""
    check(lib().b200_gemm_set_skinny_tiles(tiles), "b200_gemm_set_skinny_tiles")


def set_dynamic(mode: int) -> None:
    """1 dynamic dealing of whole tiles (default), 0 static."""
    check(lib().b200_gemm_set_dynamic(mode), "b200_gemm_set_dynamic")


def set_skinny_mode(mode: int) -> None:
    """0 off, 1 per shape (default), 2 cluster kernel, 3 stream-K kernel."""
    check(lib().b200_gemm_set_skinny_mode(mode), "b200_gemm_set_skinny_mode")


def get_splits(M: int, N: int, K: int) -> int:
    v = ctypes.c_int(0)
    check(lib().b200_gemm_get_splits(M, N, K, ctypes.byref(v)), "get_splits")
    return v.value


def gemm_bf16_profile(a_ptr, b_ptr, c_ptr, M, N, K, lda, ldb, ldc, prof_ptr, entries,
                      stream=0) -> int:
    return lib().b200_gemm_bf16_profile(a_ptr, b_ptr, c_ptr, M, N, K, lda, ldb, ldc, prof_ptr,
                                        entries, stream)


def profile_rows(M: int, N: int, K: int) -> int:
    rows = ctypes.c_int(0)
    check(lib().b200_gemm_profile_rows(M, N, K, ctypes.byref(rows)), "profile_rows")
    return rows.value


def device_status(clear: bool = True) -> int:
    v = ctypes.c_int(0)
    check(lib().b200_gemm_device_status(1 if clear else 0, ctypes.byref(v)), "device_status")
    return v.value


def set_wait_timeout_ns(ns: int) -> None:
    check(lib().b200_gemm_set_wait_timeout_ns(int(ns)), "set_wait_timeout_ns")


def set_tuning(tile_n: int = 0, stage_slabs: int = 0, raster_group: int = 0) -> None:
    """tile_n: 256, 512, -1 (per shape) or 0 (keep); stage_slabs: 1, 2 or 0;
    raster_group: band width in tiles (negative: column bands) or 0."""
    check(lib().b200_gemm_set_tuning(int(tile_n), int(stage_slabs), int(raster_group)),
          "set_tuning")


def get_tuning() -> dict:
    t, s, g = ctypes.c_int(0), ctypes.c_int(0), ctypes.c_int(0)
    check(lib().b200_gemm_get_tuning(ctypes.byref(t), ctypes.byref(s), ctypes.byref(g)),
          "get_tuning")
    return {"tile_n": t.value, "stage_slabs": s.value, "raster_group": g.value}


def wait_probe(timeout_ns: int, stream: int = 0) -> int:
    return lib().b200_gemm_wait_probe(int(timeout_ns), stream)


def tile_coord(t: int, tiles_m: int, tiles_n: int, group: int):
    tm, tn = ctypes.c_int(0), ctypes.c_int(0)
    lib().b200_gemm_tile_coord(t, tiles_m, tiles_n, group, ctypes.byref(tm), ctypes.byref(tn))
    return tm.value, tn.value


def idesc(mma_m: int, mma_n: int) -> int:
    return lib().b200_gemm_idesc(mma_m, mma_n)


def sk_range_pairs(items: int, pairs: int) -> int:
    return lib().b200_gemm_sk_range_pairs(items, pairs)


def sk_range(pair: int, items: int, range_pairs: int):
    lo, hi = ctypes.c_longlong(0), ctypes.c_longlong(0)
    lib().b200_gemm_sk_range(pair, items, range_pairs, ctypes.byref(lo), ctypes.byref(hi))
    return lo.value, hi.value


def sk_owner(x: int, items: int, range_pairs: int) -> int:
    return lib().b200_gemm_sk_owner(x, items, range_pairs)


def sk_segments(lo: int, hi: int, k_blocks: int):
    """A pair's stream-K segments in the kernel's order: [(tile, kb0, kb1), ...]."""
    pos = ctypes.c_longlong(hi)
    t, kb0, kb1 = ctypes.c_int(0), ctypes.c_int(0), ctypes.c_int(0)
    out = []
    while pos.value > lo:
        lib().b200_gemm_sk_next_segment(lo, ctypes.byref(pos), k_blocks, ctypes.byref(t),
                                        ctypes.byref(kb0), ctypes.byref(kb1))
        out.append((t.value, kb0.value, kb1.value))
    return out


def smem_desc(addr: int) -> int:
    return lib().b200_gemm_smem_desc(addr)


def launch_shape(M: int, N: int, K: int) -> dict:
    t, g, s, th = (ctypes.c_int(0) for _ in range(4))
    check(lib().b200_gemm_launch_shape(M, N, K, ctypes.byref(t), ctypes.byref(g), ctypes.byref(s),
                                       ctypes.byref(th)), "launch_shape")
    return {"tiles": t.value, "grid": g.value, "smem_bytes": s.value, "threads": th.value}


# ------------------------------------------------- fused K-split over NVLink
def ksplit_create(rank: int, nranks: int, max_m: int, max_n: int):
    """(communicator handle, exchange bytes) for this rank on the current
    device; raises GemmError on failure."""
    comm = _vp()
    buf = ctypes.create_string_buffer(KSPLIT_HANDLE_BYTES)
    check(lib().b200_ksplit_create(rank, nranks, max_m, max_n, ctypes.byref(comm), buf),
          "b200_ksplit_create")
    return comm.value, buf.raw


def ksplit_connect(comm: int, handles: bytes) -> None:
    buf = ctypes.create_string_buffer(bytes(handles), len(handles))
    check(lib().b200_ksplit_connect(comm, buf), "b200_ksplit_connect")


def ksplit_gemm_bf16(comm: int, a_ptr: int, b_ptr: int, c_ptr: int, M: int, N: int, K: int,
                     lda: int, ldb: int, ldc: int, stream: int = 0) -> int:
    return lib().b200_ksplit_gemm_bf16(comm, a_ptr, b_ptr, c_ptr, M, N, K, lda, ldb, ldc, stream)


def ksplit_epoch(comm: int) -> int:
    e = ctypes.c_uint(0)
    check(lib().b200_ksplit_epoch(comm, ctypes.byref(e)), "b200_ksplit_epoch")
    return e.value


def ksplit_destroy(comm: int) -> None:
    check(lib().b200_ksplit_destroy(comm), "b200_ksplit_destroy")
