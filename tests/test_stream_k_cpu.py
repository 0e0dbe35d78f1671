"""The CTA-pair kernel's work split, walked on the CPU.

The kernel's three roles (TMA producer, MMA issuer, epilogue) each enumerate
the same work units of their pair: whole tiles t = pair, pair + P, ... below
dp_tiles, then the pair's stream-K range.  This test restates that walk
around the library's own split (st_stream_k_split) and checks, for many
shapes, that every K block of every tile is computed exactly once, that all
units of a split tile agree on its slots (the kernel's split_tile), that the
units' own output boxes partition the tile for both box widths, that a pair
holds at most two split accumulators, and that workspace slots stay in
range."""
import itertools

import pytest

from sptiles_b200.runtime import stream_k_split

WHOLE, SPLIT = 0, 1


def units_of(pair, pairs, tiles, kb, split):
    dp_tiles, sk_pairs, sk_iters = split
    t = pair
    while t < dp_tiles:
        yield (t, 0, kb, WHOLE)
        t += pairs
    q = pairs - 1 - pair
    if q >= sk_pairs:
        return
    a, b = q * sk_iters // sk_pairs, (q + 1) * sk_iters // sk_pairs
    assert 0 < b - a <= kb  # a range is at most one tile long: one unit or two

    def unit(rel, lo, hi):
        k0, k1 = lo - rel * kb, hi - rel * kb
        return (dp_tiles + rel, k0, k1, SPLIT if (k0 > 0 or k1 < kb) else WHOLE)
    sa, sb = a // kb, (b - 1) // kb
    if sa == sb:
        yield unit(sa, a, b)
    else:  # the start of the next tile first, then the end of this one
        assert sb == sa + 1
        yield unit(sb, sb * kb, b)
        yield unit(sa, a, sb * kb)


def split_tile(pair, pairs, unit, kb, split, nb):
    """(q0, n, j, own boxes) as the kernel's split_tile computes them."""
    dp_tiles, sk_pairs, sk_iters = split
    begin = lambda q: q * sk_iters // sk_pairs
    q = pairs - 1 - pair
    start = (unit[0] - dp_tiles) * kb
    q0 = q
    while q0 > 0 and begin(q0) > start:
        q0 -= 1
    q1 = q + 1
    while q1 < sk_pairs and begin(q1) < start + kb:
        q1 += 1
    n, j = q1 - q0, q - q0
    return q0, n, j, range(nb * j // n, nb * (j + 1) // n)


SHAPES = [(t, p, kb) for t, p, kb in itertools.product(
    [1, 2, 7, 8, 16, 54, 73, 74, 75, 128, 147, 148, 256, 1024, 2048, 2049],
    [1, 2, 37, 73, 74],
    [1, 7, 8, 16, 64, 128, 1000])]


@pytest.mark.parametrize("mode", ["1", "2"], ids=["fewer_tiles", "tails_too"])
@pytest.mark.parametrize("tiles,pairs,kb", SHAPES)
def test_every_k_block_once_and_split_tiles_reduce_scatter(monkeypatch, mode, tiles, pairs, kb):
    monkeypatch.setenv("SPTILES_B200_STREAM_K", mode)
    split = stream_k_split(tiles, pairs, kb)
    dp_tiles, sk_pairs, sk_iters = split
    assert 0 <= sk_pairs <= pairs
    if sk_pairs:
        if mode == "1":
            assert tiles < pairs and dp_tiles == 0
        assert dp_tiles == tiles - tiles % pairs and sk_iters == (tiles - dp_tiles) * kb
        assert sk_pairs > tiles - dp_tiles  # better than one whole tile per pair
        assert sk_iters // sk_pairs >= 1   # no empty range: every listed piece arrives
    else:
        assert dp_tiles == tiles
    covered = {}
    slots = {}
    split_units = {}  # tile -> [(stream-K index, (q0, n), own boxes of 8, own boxes of 4)]
    for pair in range(pairs):
        n_split = 0
        for unit in units_of(pair, pairs, tiles, kb, split):
            t, k0, k1, kind = unit
            assert 0 <= t < tiles and 0 <= k0 < k1 <= kb
            for k in range(k0, k1):
                assert (t, k) not in covered
                covered[(t, k)] = pair
            if kind == SPLIT:
                n_split += 1
                q = pairs - 1 - pair
                assert 0 <= q < sk_pairs
                q0, n, j, own8 = split_tile(pair, pairs, unit, kb, split, 8)
                own4 = split_tile(pair, pairs, unit, kb, split, 4)[3]
                assert q == q0 + j
                # workspace slot (the kernel's sk_slot): 2q for the tile q's range starts in, 2q + 1 after
                rel = t - dp_tiles
                slot = 2 * q + (0 if rel == (q * sk_iters // sk_pairs) // kb else 1)
                assert slot not in slots, f"slot {slot} of tile {t} already used by tile {slots.get(slot)}"
                slots[slot] = t
                split_units.setdefault(t, []).append((q, (q0, n), own8, own4))
        assert n_split <= 2  # at most two accumulators held across the publish step
    assert len(covered) == tiles * kb
    for t, us in split_units.items():
        geo = {u[1] for u in us}
        assert len(geo) == 1, f"tile {t}: units disagree on the slots {geo}"
        q0, n = geo.pop()
        assert 2 <= n <= 6
        assert sorted(u[0] for u in us) == list(range(q0, q0 + n))  # one unit per slot, all present
        for col, nb in ((2, 8), (3, 4)):  # own boxes partition the tile: fp32 and 16-bit outputs
            assert sorted(b for u in us for b in u[col]) == list(range(nb))
        # the other units' boxes of one unit's own columns land in 48 KB per warp (12 boxes)
        for u in us:
            assert max(len(u[2]), 2 * len(u[3])) * (n - 1) <= 12


def test_split_only_with_fewer_tiles_than_pairs():
    """8192 x 8192 x 8192 f16 on 1/2/4/8 GPUs (M rows per GPU, >= 128 tiles)
    runs whole tiles; the fp32 1024^3 configuration (16 tiles of 96 K blocks
    of the packed 3xTF32 operands) splits over 64 pairs."""
    for m in (8192, 4096, 2048, 1024):
        tiles = (m // 256) * (8192 // 256)
        assert stream_k_split(tiles, 74, 8192 // 64) == (tiles, 0, 0)
    assert stream_k_split(16, 74, 96) == (0, 64, 16 * 96)
