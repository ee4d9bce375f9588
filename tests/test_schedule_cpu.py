"""The persistent kernels' schedule arithmetic, run on the host (the same __host__
__device__ functions the kernels call): every (tile, K block) unit of the problem is
computed by exactly one slot, stream-K partial pieces name consistent contributor ranges,
and each partial tile's contributors are exactly the slots that hold a piece of it."""
import ctypes
import itertools

import pytest

import hipgemm_b200 as hg


def schedule(tiles, slots, kblocks, mode):
    out = (ctypes.c_int * 3)()
    assert hg.lib().hgemm_debug_schedule(tiles, slots, kblocks, mode, out) == 0
    return tuple(out)


def items(kblocks, nslots, dp, sk, sk_slots, slot):
    buf = (ctypes.c_int * (6 * 4096))()
    n = hg.lib().hgemm_debug_work_items(kblocks, nslots, dp, sk, sk_slots, slot, buf, 4096)
    assert n >= 0
    return [tuple(buf[6 * i:6 * i + 6]) for i in range(n)]


CASES = [  # (tiles, slots, kblocks)
    (1024, 74, 64), (128, 74, 64), (32, 148, 64), (112, 74, 16), (320, 74, 56), (256, 74, 32), (7168, 74, 64),
    (1, 148, 1), (3, 148, 2), (5, 7, 3), (148, 148, 64), (149, 148, 64), (2048, 148, 64), (64, 148, 64),
]


@pytest.mark.parametrize("tiles,slots,kblocks", CASES)
@pytest.mark.parametrize("mode", [hg.HGEMM_SCHEDULE_AUTO, hg.HGEMM_SCHEDULE_DATA_PARALLEL, hg.HGEMM_SCHEDULE_STREAM_K])
def test_every_unit_exactly_once(tiles, slots, kblocks, mode):
    dp, sk, sk_slots = schedule(tiles, slots, kblocks, mode)
    assert dp + sk == tiles and 0 <= sk_slots <= slots
    if mode == hg.HGEMM_SCHEDULE_DATA_PARALLEL:
        assert sk == 0
    if sk:
        assert sk * kblocks >= sk_slots >= 1  # no slot gets an empty stream-K range
    covered = {}
    pieces = {}  # tile -> list of (slot, piece)
    for s in range(slots):
        for (t, k0, k1, piece, c_lo, c_hi) in items(kblocks, slots, dp, sk, sk_slots, s):
            assert 0 <= t < tiles and 0 <= k0 < k1 <= kblocks
            for k in range(k0, k1):
                assert (t, k) not in covered, (t, k)
                covered[(t, k)] = s
            if piece < 0:
                assert (k0, k1) == (0, kblocks)
            else:
                assert t >= dp and c_lo <= s <= c_hi and c_lo < c_hi
                pieces.setdefault(t, []).append((s, piece, c_lo, c_hi))
    assert len(covered) == tiles * kblocks
    for t, lst in pieces.items():
        slots_of_t = sorted(s for s, _, _, _ in lst)
        c_lo, c_hi = lst[0][2], lst[0][3]
        assert all((a, b) == (c_lo, c_hi) for _, _, a, b in lst)
        assert slots_of_t == list(range(c_lo, c_hi + 1))  # contributors == slots holding a piece
    # Each slot holds at most one piece 0 (its first stream-K tile) and one piece 1 (its
    # last): two workspace partials per slot suffice, and piece 0 precedes piece 1.
    for s in range(slots):
        ps = [(t, p) for (t, _, _, p, _, _) in items(kblocks, slots, dp, sk, sk_slots, s) if p >= 0]
        assert [p for _, p in ps] in ([], [0], [1], [0, 1])
        if len(ps) == 2:
            assert ps[0][0] < ps[1][0]


def test_schedule_choices():
    for tiles, slots in [(1024, 74), (128, 74), (32, 148), (7168, 74)]:
        assert schedule(tiles, slots, 64, hg.HGEMM_SCHEDULE_AUTO) == (tiles, 0, 0)  # automatic = data-parallel
    dp, sk, sks = schedule(128, 74, 64, hg.HGEMM_SCHEDULE_STREAM_K)  # 8192^3 / 8 GPUs: 1.73 waves
    assert (dp, sk) == (74, 54) and sks == 74                       # stream-K over the partial wave
    dp, sk, sks = schedule(32, 148, 64, hg.HGEMM_SCHEDULE_STREAM_K)  # 128 x 8192 x 8192 on 128 x 256 tiles
    assert (dp, sk) == (0, 32) and sks == 148
    dp, sk, sks = schedule(148, 148, 64, hg.HGEMM_SCHEDULE_STREAM_K)  # balanced: each slot gets one tile
    assert (dp, sk, sks) == (0, 148, 148)


def test_debug_entry_points_reject_bad_input():
    out = (ctypes.c_int * 6)()
    assert hg.lib().hgemm_debug_schedule(0, 74, 64, 0, out) == hg.HGEMM_ERR_INVALID_VALUE
    assert hg.lib().hgemm_debug_work_items(64, 74, 0, 10, 0, 0, out, 1) == hg.HGEMM_ERR_INVALID_VALUE
    assert hg.lib().hgemm_debug_work_items(64, 74, 0, 0, 0, 74, out, 1) == hg.HGEMM_ERR_INVALID_VALUE


@pytest.mark.parametrize("split", [2, 4])
@pytest.mark.parametrize("tiles,kblocks", [(37, 64), (74, 64), (1, 1), (3, 3), (5, 4), (2, 7), (37, 16), (9, 130)])
def test_split_k_clusters_cover_every_unit_once(split, tiles, kblocks):
    """The split-K configurations: CTA r of cluster t gets exactly K part r of tile t (one
    item), the parts of a tile are contiguous, disjoint and cover all its K blocks in rank
    order, and CTAs past the last cluster get nothing."""
    L = hg.lib()
    out = (ctypes.c_int * 3)()
    for t in range(tiles):
        parts = []
        for r in range(split):
            assert L.hgemm_debug_split_work(kblocks, split, tiles, t * split + r, out) == 1
            assert out[0] == t
            parts.append((out[1], out[2]))
        assert parts[0][0] == 0 and parts[-1][1] == kblocks
        for (b0, e0), (b1, e1) in zip(parts, parts[1:]):
            assert e0 == b1 and b0 <= e0
        # Balanced: part sizes differ by at most one K block.
        sizes = [e - b for b, e in parts]
        assert max(sizes) - min(sizes) <= 1
    assert L.hgemm_debug_split_work(kblocks, split, tiles, tiles * split, out) == 0
    assert L.hgemm_debug_split_work(kblocks, 1, tiles, 0, out) == hg.HGEMM_ERR_INVALID_VALUE


def _b200_resident():
    """CTAs resident at once per configuration on B200, as the library measures them at set-up
    (cudaOccupancy*): 148 for every configuration except 4-CTA clusters (33 clusters fit)."""
    names = hg.config_names()
    res = (ctypes.c_int * len(names))(*([0] + [148] * (len(names) - 1)))
    res[names.index("bn128_s5_k4")] = 132
    return names, res


@pytest.mark.parametrize("shape,auto,data_parallel", [
    ((8192, 8192, 8192), "pair256_s6", "pair256_s6"),        # the headline: 256 x 256 CTA-pair tiles
    ((16384, 28672, 8192), "pair256_s6", "pair256_s6"),
    ((128, 8192, 8192), "bn128_s5_k2", "bn128_s6"),          # skinny, long K: split-K only under AUTO
    ((64, 8192, 8192), "bn128_s5_k2", "bn128_s6"),
    ((128, 4096, 8192), "bn128_s5_k4", "bn128_s6"),          # fewer tiles: four K parts
    ((128, 7168, 2048), "bn128_s6", "bn128_s6"),             # K too short for split-K to pay
    ((256, 8192, 8192), "bn128_s6", "bn128_s6"),             # 128 tiles: clusters would not fit at once
    ((1024, 8192, 8192), "pair256_s6", "pair256_s6"),        # the 8-GPU shard: 2 waves either way
    ((1024, 7168, 2048), "pair256_s6", "pair256_s6"),        # 2 waves either way: the wider tile
    ((4000, 5120, 7168), "pair256_s6", "pair256_s6"),        # 5 waves either way
])
def test_automatic_choice(shape, auto, data_parallel):
    """The configuration choice (host-only entry point, same code as the launch path) under the
    automatic and the explicit data-parallel schedule, with B200's resident CTA counts."""
    names, res = _b200_resident()
    L = hg.lib()
    assert names[L.hgemm_debug_choose(*shape, hg.HGEMM_SCHEDULE_AUTO, res, len(names))] == auto
    assert names[L.hgemm_debug_choose(*shape, hg.HGEMM_SCHEDULE_DATA_PARALLEL, res, len(names))] == data_parallel
    sk = names[L.hgemm_debug_choose(*shape, hg.HGEMM_SCHEDULE_STREAM_K, res, len(names))]
    assert "_k" not in sk  # an explicit stream-K schedule never gets a split-K cluster configuration


def test_automatic_choice_respects_cluster_residency():
    """With fewer 4-CTA clusters resident than tiles, the four-way split gives way."""
    names, res = _b200_resident()
    res[names.index("bn128_s5_k4")] = 120  # 30 clusters < 32 tiles of 128 x 4096
    L = hg.lib()
    assert names[L.hgemm_debug_choose(128, 4096, 8192, hg.HGEMM_SCHEDULE_AUTO, res, len(names))] == "bn128_s5_k2"
    assert L.hgemm_debug_choose(128, 4096, 8192, 0, res, len(names) - 1) == hg.HGEMM_ERR_INVALID_VALUE
    assert L.hgemm_debug_choose(0, 4096, 8192, 0, res, len(names)) == hg.HGEMM_ERR_INVALID_VALUE
    res[1] = 0
    assert L.hgemm_debug_choose(128, 4096, 8192, 0, res, len(names)) == hg.HGEMM_ERR_INVALID_VALUE


def test_automatic_choice_never_takes_the_224_wide_tile():
    """Measured on B200, a 256x224 pair tile takes as long as a 256x256 one, and a narrower tile
    never needs fewer waves: the automatic choice keeps the 224-wide tile for explicit requests."""
    names, res = _b200_resident()
    L = hg.lib()
    for M in (256, 512, 1024, 2048, 4000, 4096, 8192):
        for N in (1568, 4096, 5120, 7168, 8192, 9472, 28672):
            for K in (2048, 8192):
                for sched in (hg.HGEMM_SCHEDULE_AUTO, hg.HGEMM_SCHEDULE_DATA_PARALLEL):
                    assert names[L.hgemm_debug_choose(M, N, K, sched, res, len(names))] != "pair224_s6", (M, N, K)
