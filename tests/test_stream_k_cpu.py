"""The CTA-pair kernel's work split, walked on the CPU.

The kernel's three roles (TMA producer, MMA issuer, epilogue) each enumerate
the same work units of their pair: whole tiles t = pair, pair + P, ... below
dp_tiles, then the pair's stream-K range.  This test restates that walk
around the library's own split (st_stream_k_split) and checks, for many
shapes, that every K block of every tile is computed exactly once, that each
split tile has one owner (the unit holding its K block 0), that the pieces
the owner folds are exactly the other units of the tile, that every piece
comes from a pair with a lower number than its owner (so nothing waits on a
pair that may not have started), and that workspace slots stay in range."""
import itertools

import pytest

from sptiles_b200.runtime import stream_k_split

WHOLE, OWNER, PIECE = 0, 1, 2


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
        return (dp_tiles + rel, k0, k1, PIECE if k0 > 0 else (OWNER if k1 < kb else WHOLE))
    sa, sb = a // kb, (b - 1) // kb
    if sa == sb:
        yield unit(sa, a, b)
    else:  # the owned start of the next tile first, then the piece of this one
        assert sb == sa + 1
        owned, piece = unit(sb, sb * kb, b), unit(sa, a, sb * kb)
        assert owned[3] == OWNER and piece[3] == PIECE
        yield owned
        yield piece


def owner_pieces(pair, pairs, unit, kb, split):
    """Stream-K slots the owner folds (the kernel's sk_fold_pieces loop)."""
    dp_tiles, sk_pairs, sk_iters = split
    q = pairs - 1 - pair
    tile_end = (unit[0] - dp_tiles + 1) * kb
    out = []
    r = q + 1
    while r < sk_pairs and r * sk_iters // sk_pairs < tile_end:
        out.append(r)
        r += 1
    return out


SHAPES = [(t, p, kb) for t, p, kb in itertools.product(
    [1, 2, 7, 8, 16, 54, 73, 74, 75, 128, 147, 148, 256, 1024, 2048, 2049],
    [1, 2, 37, 73, 74],
    [1, 7, 8, 16, 64, 128, 1000])]


@pytest.mark.parametrize("tiles,pairs,kb", SHAPES)
def test_every_k_block_once_and_owners_fold_their_pieces(tiles, pairs, kb):
    split = stream_k_split(tiles, pairs, kb)
    dp_tiles, sk_pairs, sk_iters = split
    assert 0 <= sk_pairs <= pairs
    if sk_pairs:
        assert tiles < pairs and dp_tiles == 0 and sk_iters == tiles * kb
        assert sk_pairs > tiles - dp_tiles  # better than one whole tile per pair
        assert sk_iters // sk_pairs >= 1   # no empty range: every listed piece arrives
    else:
        assert dp_tiles == tiles
    covered = {}
    pieces = {}   # tile -> [(slot, pair)]
    owners = {}   # tile -> (pair, folded slots)
    for pair in range(pairs):
        n_pieces = 0
        for unit in units_of(pair, pairs, tiles, kb, split):
            t, k0, k1, kind = unit
            assert 0 <= t < tiles and 0 <= k0 < k1 <= kb
            for k in range(k0, k1):
                assert (t, k) not in covered
                covered[(t, k)] = pair
            if kind == PIECE:
                n_pieces += 1
                slot = pairs - 1 - pair
                assert 0 <= slot < sk_pairs
                pieces.setdefault(t, []).append((slot, pair))
            elif kind == OWNER:
                assert t not in owners
                owners[t] = (pair, owner_pieces(pair, pairs, unit, kb, split))
        assert n_pieces <= 1  # one workspace slot per pair suffices
    assert len(covered) == tiles * kb
    for t, plist in pieces.items():
        assert t in owners, f"tile {t} has pieces but no owner"
        opair, folded = owners[t]
        assert sorted(s for s, _ in plist) == folded
        assert all(p < opair for _, p in plist)
        assert len(folded) <= 6
    for t, (_, folded) in owners.items():
        assert folded, f"owner of tile {t} has nothing to fold"


def test_split_only_with_fewer_tiles_than_pairs():
    """8192 x 8192 x 8192 f16 on 1/2/4/8 GPUs (M rows per GPU, >= 128 tiles)
    runs whole tiles; the fp32 1024^3 configuration (16 tiles of 96 K blocks
    of the packed 3xTF32 operands) splits over 64 pairs."""
    for m in (8192, 4096, 2048, 1024):
        tiles = (m // 256) * (8192 // 256)
        assert stream_k_split(tiles, 74, 8192 // 64) == (tiles, 0, 0)
    assert stream_k_split(16, 74, 96) == (0, 64, 16 * 96)
