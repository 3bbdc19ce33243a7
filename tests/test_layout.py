"""Host-side layout rules of the kernel, checked through the C ABI (no GPU).

Descriptor fields are checked against the bit positions of the PTX ISA
tables for tcgen05 (instruction descriptor of kind::f16, shared-memory matrix
descriptor); the rasteriser is checked to visit every tile exactly once.
"""
import pytest

from blackwell_gemm_b200 import capi


def bits(x, lo, hi):
    """Field [lo, hi) of x."""
    return (x >> lo) & ((1 << (hi - lo)) - 1)


@pytest.mark.parametrize("m,n", [(256, 256), (128, 256), (256, 128), (128, 64), (64, 8)])
def test_instruction_descriptor_fields(m, n):
    d = capi.idesc(m, n)
    assert bits(d, 0, 4) == 0          # dense, no saturate
    assert bits(d, 4, 6) == 1          # D = f32
    assert bits(d, 7, 10) == 1         # A = bf16
    assert bits(d, 10, 13) == 1        # B = bf16
    assert bits(d, 13, 15) == 0        # no negation
    assert bits(d, 15, 17) == 0        # A and B K-major
    assert bits(d, 17, 23) == n >> 3
    assert bits(d, 23, 24) == 0
    assert bits(d, 24, 29) == m >> 4
    assert bits(d, 29, 32) == 0


def test_instruction_descriptor_matches_reference_packing():
    # kernel_v8.cu:450-455 packs (1<<4)|(1<<7)|(1<<10)|(BN>>3<<17)|((2*BM)>>4<<24)
    ref = (1 << 4) | (1 << 7) | (1 << 10) | ((256 >> 3) << 17) | ((2 * 128) >> 4 << 24)
    assert capi.idesc(256, 256) == ref


@pytest.mark.parametrize("addr", [0, 1024, 0x8000, 0x30000, 0x37C00, 1024 + 32, 1024 + 96])
def test_smem_descriptor_fields(addr):
    d = capi.smem_desc(addr)
    assert bits(d, 0, 14) == (addr & 0x3FFFF) >> 4    # start address >> 4
    assert bits(d, 16, 30) == 0                       # LBO unused (swizzled K-major)
    assert bits(d, 32, 46) == 1024 >> 4               # SBO: 8 rows x 128 B
    assert bits(d, 46, 48) == 1                       # sm_100 descriptor version
    assert bits(d, 49, 52) == 0                       # base offset
    assert bits(d, 52, 53) == 0                       # LBO mode
    assert bits(d, 61, 64) == 2                       # 128 B swizzle


def test_smem_descriptor_k_advance_is_plus_two():
    # The kernel adds 2 (= 32 B >> 4) per K16 step to the descriptor itself.
    for base in (0, 1024, 0x20000):
        for k in range(4):
            assert capi.smem_desc(base + 32 * k) == capi.smem_desc(base) + 2 * k


@pytest.mark.parametrize("tm,tn,group", [(32, 32, 8), (1, 1, 8), (4, 64, 8), (33, 7, 8),
                                          (5, 5, 16), (112, 24, 8), (32, 32, 1), (3, 9, 2),
                                          (32, 32, -8), (7, 33, -8), (24, 112, -4), (9, 3, -2)])
def test_raster_is_a_permutation(tm, tn, group):
    seen = set()
    for t in range(tm * tn):
        m, n = capi.tile_coord(t, tm, tn, group)
        assert 0 <= m < tm and 0 <= n < tn
        seen.add((m, n))
    assert len(seen) == tm * tn


def test_raster_bands_keep_wave_working_set_small():
    # 74 consecutive tiles (one wave of pairs on 148 SMs) at 8192^3 touch at
    # most ~group + 74/group distinct A row blocks + B column blocks.
    tm = tn = 32
    for start in range(0, tm * tn - 74, 37):
        ms, ns = set(), set()
        for t in range(start, start + 74):
            m, n = capi.tile_coord(t, tm, tn, 8)
            ms.add(m)
            ns.add(n)
        assert len(ms) + len(ns) <= 8 + 8 + 11


def test_raster_serpentine_band_transition_reuses_blocks():
    # the last tile of band 0 and the first of band 1 share a column block
    tm, tn, g = 32, 32, 8
    last = capi.tile_coord(g * tn - 1, tm, tn, g)
    first = capi.tile_coord(g * tn, tm, tn, g)
    assert last[1] == first[1]
    last = capi.tile_coord(g * tm - 1, tm, tn, -g)
    first = capi.tile_coord(g * tm, tm, tn, -g)
    assert last[0] == first[0]


def test_persistent_assignment_covers_all_tiles_once():
    tiles, pairs = 1024, 74
    owner = {}
    for p in range(pairs):
        for t in range(p, tiles, pairs):
            assert t not in owner
            owner[t] = p
    assert len(owner) == tiles
    loads = [len(range(p, tiles, pairs)) for p in range(pairs)]
    assert max(loads) - min(loads) <= 1


def test_launch_shape_without_gpu():
    before = capi.get_tuning()
    try:
        capi.set_tuning(256, 1, 0)
        s = capi.launch_shape(8192, 8192, 8192)
        assert s["tiles"] == 32 * 32 and s["threads"] == 192
        assert s["smem_bytes"] <= 227 * 1024
        assert capi.launch_shape(16, 8192, 8192)["tiles"] == 32
        assert capi.launch_shape(300, 520, 200)["tiles"] == 2 * 3
        capi.set_tuning(512, 1, 0)
        s = capi.launch_shape(8192, 8192, 8192)
        assert s["tiles"] == 32 * 16 and s["threads"] == 320
        assert s["smem_bytes"] <= 227 * 1024
        capi.set_tuning(-1, 1, 0)
        # per-shape choice: wide tiles on a big grid, 256-wide on a small one
        assert capi.launch_shape(8192, 8192, 8192)["threads"] == 320
        assert capi.launch_shape(2048, 2048, 2048)["threads"] == 192
        assert capi.launch_shape(16, 8192, 8192)["threads"] == 192
        # grids under one wave of 256-wide tiles: the width minimising
        # waves x width (no device: 74 pairs assumed)
        assert capi.launch_shape(1024, 1024, 1024)["tiles"] == 4 * 16      # 64 wide
        assert capi.launch_shape(768, 1024, 1024)["tiles"] == 3 * 16       # 64 wide
        assert capi.launch_shape(1024, 2048, 1024)["tiles"] == 4 * 16      # 128 wide
        assert capi.launch_shape(2048, 2048, 2048)["tiles"] == 8 * 8       # ties keep 256
        for width, tiles in ((128, 32 * 64), (64, 32 * 128)):
            capi.set_tuning(width, 1, 0)
            s = capi.launch_shape(8192, 8192, 8192)
            assert s["tiles"] == tiles and s["threads"] == 192
            assert s["smem_bytes"] <= 227 * 1024
    finally:
        capi.set_tuning(before["tile_n"] or -1, before["stage_slabs"], before["raster_group"])


def _check_stream_k_split(sk_tiles, k_blocks, pairs):
    items = sk_tiles * k_blocks
    G = capi.sk_range_pairs(items, pairs)
    assert G == min(items, pairs)
    covered = {}
    nonfinishing = {}          # pair -> tile of its one unfinished piece
    finisher = {}              # tile -> pair holding its last K block
    prev_hi = 0
    for p in range(G):
        lo, hi = capi.sk_range(p, items, G)
        assert lo == prev_hi and hi > lo      # contiguous, non-empty
        prev_hi = hi
        segs = capi.sk_segments(lo, hi, k_blocks)
        pos = hi
        for i, (t, kb0, kb1) in enumerate(segs):
            # walked from the end, one tile per segment, exactly covering the range
            assert 0 <= kb0 < kb1 <= k_blocks
            assert t * k_blocks + kb1 == pos
            pos = t * k_blocks + kb0
            for kb in range(kb0, kb1):
                assert (t, kb) not in covered
                covered[(t, kb)] = p
            if kb1 < k_blocks:
                # a piece left for another pair: at most one per pair (one slot),
                # and it is the pair's first segment
                assert p not in nonfinishing and i == 0
                nonfinishing[p] = t
            else:
                finisher[t] = p
        assert pos == lo
    assert prev_hi == items and len(covered) == items
    for t in range(sk_tiles):
        f = finisher[t]
        c0 = capi.sk_owner(t * k_blocks, items, G)
        assert covered[(t, 0)] == c0
        # the finisher adds the pieces of pairs c0 .. f-1, each holding this tile's piece
        for c in range(c0, f):
            assert nonfinishing.get(c) == t
    # every unfinished piece is added by the finisher of its tile
    for c, t in nonfinishing.items():
        assert capi.sk_owner(t * k_blocks, items, G) <= c < finisher[t]


@pytest.mark.parametrize("sk_tiles,k_blocks,pairs", [
    (34, 64, 74),      # 4096^3 on 256 x 256 tiles: 222 whole tiles + 34 in the tail
    (22, 64, 74),      # 8192 x 6144 x 4096
    (73, 128, 74), (1, 128, 74), (1, 1, 74), (3, 2, 74), (5, 30, 8), (7, 3, 8),
    (2, 1000, 3), (9, 17, 74), (60, 5, 74),
])
def test_stream_k_split_covers_every_item_once_with_one_piece_per_pair(sk_tiles, k_blocks, pairs):
    _check_stream_k_split(sk_tiles, k_blocks, pairs)


def test_stream_k_split_random_shapes():
    import random
    rng = random.Random(7)
    for _ in range(300):
        pairs = rng.choice([74, 70, 37, 8, 2])
        _check_stream_k_split(rng.randint(1, pairs), rng.randint(1, 300), pairs)
