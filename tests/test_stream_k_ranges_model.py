"""The stream-K split arithmetic the GEMM kernels share, checked on the CPU.

k_gemv_tma (csrc/gemv_tma.cu), k_umma_bs / k_bs_fixup (csrc/umma_bs.cu) and
k_umma_sk (csrc/umma_sk.cu) give CTA b of G the iterations
[floor(b T / G), floor((b + 1) T / G)) of T = tiles x KS, and the CTA that
sums a split tile t finds its contributors as the CTAs owning the tile's
first and last iterations, c(i) = floor(((i + 1) G - 1) / T); a contributor
parks its partial in slot 2 c + (0 if t is its first tile else 1), and the
last arriver is the one whose ticket equals c_hi - c_lo.  This restates those
formulas and checks them against a direct walk of the ranges for every
T <= 240 and every G <= min(T, 160) at several KS: c(i) is the owner of i,
every CTA's range is non-empty, a CTA's split segments are at most its first
and last tile, so the two slots never collide, and a tile's contributors are
exactly c_lo .. c_hi.  No GPU is involved.
"""
import pytest


def _owner(i, G, T):
    return ((i + 1) * G - 1) // T


@pytest.mark.parametrize("KS", [1, 2, 3, 16, 32])
def test_contributor_ranges(KS):
    for tiles in range(1, 240 // KS + 1):
        T = tiles * KS
        for G in range(1, min(T, 160) + 1):
            start = [b * T // G for b in range(G + 1)]
            owner = []
            for b in range(G):
                assert start[b + 1] > start[b]            # every CTA has work
                owner += [b] * (start[b + 1] - start[b])
            assert [_owner(i, G, T) for i in range(T)] == owner
            slots = {}
            for t in range(tiles):
                t0, t1 = t * KS, t * KS + KS - 1
                c_lo, c_hi = _owner(t0, G, T), _owner(t1, G, T)
                assert set(owner[t0:t1 + 1]) == set(range(c_lo, c_hi + 1))
                if c_lo == c_hi:
                    continue                              # whole tile: stored directly
                for c in range(c_lo, c_hi + 1):
                    first_tile = start[c] // KS
                    last_tile = (start[c + 1] - 1) // KS
                    assert t in (first_tile, last_tile)   # split segments sit at a range's ends
                    slot = 2 * c + (0 if t == first_tile else 1)
                    assert slots.setdefault(slot, t) == t, (T, G, c, t)
