"""The C-ABI library loads, exports every function include/*.h declares, and
rejects bad arguments before touching a device (so this runs without a GPU)."""
import ctypes
import re
from pathlib import Path

import pytest

from blackwell_gemm_b200 import capi

ROOT = Path(__file__).resolve().parents[1]


def declared_functions():
    names = []
    for h in sorted((ROOT / "include").glob("*.h")):
        text = re.sub(r"/\*.*?\*/", "", h.read_text(), flags=re.S)
        names += re.findall(r"^[A-Za-z_][\w\s\*]*?\b(b200_\w+)\s*\(", text, flags=re.M)
    return names


def test_header_declares_the_entry_points():
    names = declared_functions()
    for n in ("b200_gemm_bf16", "b200_gemm_bf16_profile", "b200_gemm_profile_rows",
              "b200_gemm_device_status", "b200_gemm_status_string"):
        assert n in names


def test_library_exports_every_declared_symbol():
    lib = capi.lib()
    for n in declared_functions():
        assert hasattr(lib, n), f"{n} declared in include/ but not exported"
        assert n in capi.SIGNATURES or n.startswith("b200_gemm"), n


def test_every_declared_symbol_has_a_python_signature():
    for n in declared_functions():
        assert n in capi.SIGNATURES, f"{n} has no ctypes signature in capi.SIGNATURES"


def test_status_strings():
    for code in range(0, 8):
        assert capi.status_string(code)
    assert "unknown" in capi.status_string(999)


FAKE = 0x7F0000000000  # never dereferenced: validation fails or returns first


@pytest.mark.parametrize("args,expect", [
    ((FAKE, FAKE, FAKE, -1, 8, 8, 8, 8, 8), capi.ERR_INVALID_ARGUMENT),
    ((FAKE, FAKE, FAKE, 8, -1, 8, 8, 8, 8), capi.ERR_INVALID_ARGUMENT),
    ((FAKE, FAKE, FAKE, 8, 8, -1, 8, 8, 8), capi.ERR_INVALID_ARGUMENT),
    ((0, FAKE, FAKE, 8, 8, 8, 8, 8, 8), capi.ERR_INVALID_ARGUMENT),
    ((FAKE, 0, FAKE, 8, 8, 8, 8, 8, 8), capi.ERR_INVALID_ARGUMENT),
    ((FAKE, FAKE, 0, 8, 8, 8, 8, 8, 8), capi.ERR_INVALID_ARGUMENT),
    ((FAKE, FAKE, FAKE, 8, 8, 16, 8, 16, 8), capi.ERR_INVALID_ARGUMENT),   # lda < K
    ((FAKE, FAKE, FAKE, 8, 16, 8, 8, 8, 8), capi.ERR_INVALID_ARGUMENT),    # ldc < N
    ((FAKE + 2, FAKE, FAKE, 8, 8, 8, 8, 8, 8), capi.ERR_ALIGNMENT),
    ((FAKE, FAKE, FAKE + 8, 8, 8, 8, 8, 8, 8), capi.ERR_ALIGNMENT),
    ((FAKE, FAKE, FAKE, 8, 8, 12, 12, 16, 8), capi.ERR_ALIGNMENT),         # lda % 8
    ((FAKE, FAKE, FAKE, 8, 12, 8, 8, 8, 12), capi.ERR_ALIGNMENT),          # ldc % 8
    ((0, 0, 0, 0, 8, 8, 8, 8, 8), capi.OK),                                # M == 0: no-op
    ((0, 0, 0, 8, 0, 8, 8, 8, 8), capi.OK),                                # N == 0: no-op
])
def test_argument_validation(args, expect):
    assert capi.gemm_bf16(*args, 0) == expect


def test_profile_requires_buffer():
    st = capi.gemm_bf16_profile(FAKE, FAKE, FAKE, 8, 8, 8, 8, 8, 8, 0, 4, 0)
    # validation passes, then a null profiler buffer is rejected before launch
    assert st == capi.ERR_INVALID_ARGUMENT


def test_tuning_roundtrip_and_validation():
    before = capi.get_tuning()
    capi.set_tuning(512, 2, -4)
    assert capi.get_tuning() == {"tile_n": 512, "stage_slabs": 2, "raster_group": -4}
    capi.set_tuning(-1, 1, -8)
    assert capi.get_tuning()["tile_n"] == 0
    for bad in ((300, 0, 0), (0, 3, 0), (0, -1, 0)):
        with pytest.raises(capi.GemmError):
            capi.set_tuning(*bad)
    capi.set_tuning(before["tile_n"] or -1, before["stage_slabs"], before["raster_group"])


def test_timeout_setter_rejects_zero():
    with pytest.raises(capi.GemmError):
        capi.set_wait_timeout_ns(0)
    capi.set_wait_timeout_ns(2_000_000_000)


def test_wait_probe_rejects_unbounded():
    assert capi.wait_probe(0) == capi.ERR_INVALID_ARGUMENT
    assert capi.wait_probe(60_000_000_000) == capi.ERR_INVALID_ARGUMENT


def test_torch_extension_builds_and_checks_inputs():
    import torch
    import blackwell_gemm_b200 as bg

    ext = bg.load()
    assert hasattr(ext, "matmul_b200") and hasattr(ext, "profile_matmul_b200")
    a = torch.zeros(4, 8, dtype=torch.bfloat16)
    with pytest.raises(RuntimeError, match="CUDA"):
        bg.matmul_b200(a, a.T)
    with pytest.raises(RuntimeError, match="2-D"):
        bg.matmul_b200(a[0], a.T)


def test_ksplit_rejects_bad_arguments_without_a_device():
    for args in [(2, 2, 512, 256), (-1, 2, 512, 256), (0, 9, 4608, 256), (0, 2, 300, 256),
                 (0, 1, 256, 0)]:
        with pytest.raises(capi.GemmError) as e:
            capi.ksplit_create(*args)
        assert e.value.status == capi.ERR_INVALID_ARGUMENT, args
    lib = capi.lib()
    assert lib.b200_ksplit_gemm_bf16(None, FAKE, FAKE, FAKE, 512, 256, 64, 64, 64, 256,
                                     None) == capi.ERR_INVALID_ARGUMENT
    assert lib.b200_ksplit_connect(None, None) == capi.ERR_INVALID_ARGUMENT
    assert lib.b200_ksplit_destroy(None) == capi.OK
    assert capi.KSPLIT_HANDLE_BYTES == 128


def test_mode_setters_accept_their_range_and_reject_the_rest():
    lib = capi.lib()
    for mode in range(6):                       # 4, 5: stream-K / cluster on 2-CTA pairs
        assert lib.b200_gemm_set_skinny_mode(mode) == capi.OK
    assert lib.b200_gemm_set_skinny_mode(6) == capi.ERR_INVALID_ARGUMENT
    assert lib.b200_gemm_set_skinny_mode(-1) == capi.ERR_INVALID_ARGUMENT
    capi.set_skinny_mode(1)
    for tiles in (0, 1, 2):
        assert lib.b200_gemm_set_skinny_tiles(tiles) == capi.OK
    assert lib.b200_gemm_set_skinny_tiles(3) == capi.ERR_INVALID_ARGUMENT
    capi.set_skinny_tiles(0)
    for mode in (0, 1):
        assert lib.b200_gemm_set_dynamic(mode) == capi.OK
    assert lib.b200_gemm_set_dynamic(2) == capi.ERR_INVALID_ARGUMENT
    capi.set_dynamic(0)


def test_skinny_slice_reports_follow_the_kernel_choice():
    # Without a device the launcher assumes 148 SMs; the per-shape choice is
    # plain integer arithmetic: one-CTA stream-K up to M = 128, the pair
    # stream-K kernel above it where the split-K workspace reaches 16 MB.
    capi.set_skinny_mode(1)
    capi.set_splits(0)
    wide = capi.get_splits(256, 28672, 4096)           # pair stream-K: contributors per tile
    narrow = capi.get_splits(256, 8192, 8192)          # split-K kernel: K slices
    assert wide >= 1 and narrow >= 1
    capi.set_skinny_mode(4)
    assert capi.get_splits(256, 28672, 4096) == wide   # forcing the pair kernel changes nothing
    capi.set_skinny_mode(1)


def test_noalloc_status_needs_a_device():
    v = ctypes.c_int(7)
    assert capi.lib().b200_gemm_noalloc_status(1, None) == capi.ERR_INVALID_ARGUMENT
    st = capi.lib().b200_gemm_noalloc_status(1, ctypes.byref(v))
    assert st in (capi.OK, capi.ERR_UNSUPPORTED_DEVICE)   # no GPU here: refused, not crashed
    assert capi.noalloc_wait_probe(0) == capi.ERR_INVALID_ARGUMENT
