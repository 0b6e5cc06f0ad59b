"""The MMA GEMV's work split, restated on the CPU (xdna.cpp_b200/csrc/gemv_mma.cu:
the launcher's grid choice, the kernel's inline unit-mode ranges and struct
Split for tile mode), checked for the invariants its combine relies on:

* every (tile, group) unit belongs to exactly one warp, and the inverse
  (the warp of a unit) agrees with the ranges;
* tile mode: no tile spans two CTAs (no cross-CTA combine is needed);
* the warps that share a tile are consecutive and none of them is empty (the
  shared-memory combine counts every warp from the first to the last);
* a warp shares at most its first and its last tile (two partial slots);
* a CTA touches at most cta_tiles tiles (its shared-memory counters).
"""
from __future__ import annotations

import random

import pytest

KWARPS = 24  # one 24-warp CTA per SM
SMS = 148


def warp_of(u: int, n: int, parts: int) -> int:
    return ((u + 1) * parts + n - 1) // n - 1


class Grid:
    def __init__(self, ntiles: int, ng: int, sms: int = SMS):
        self.T, self.ng, self.U = ntiles, ng, ntiles * ng
        self.tiles = self.U <= 64 * sms
        blocks = sms
        if self.tiles:
            blocks = min(blocks, ntiles)
            per = -(-ntiles // blocks)  # whole tiles per CTA, about the same for all
            blocks = -(-ntiles // per)
            self.NW = blocks * KWARPS
            self.cta_tiles = -(-ntiles // blocks) + 2
        else:
            blocks = max(1, min(blocks, -(-self.U // KWARPS)))
            self.NW = min(blocks * KWARPS, self.U)
            per_warp = -(-self.U // self.NW)
            self.cta_tiles = -(-(KWARPS * per_warp) // ng) + 2
        self.NC = blocks

    def cta_unit0(self, c: int) -> int:
        if self.tiles:
            return (c * self.T // self.NC) * self.ng
        return min(c * KWARPS, self.NW) * self.U // self.NW

    @staticmethod
    def cta_warps(uc: int) -> int:
        return min((uc + 1) // 2, KWARPS)

    def warp_unit0(self, w: int) -> int:
        if not self.tiles:
            return w * self.U // self.NW if w < self.NW else self.U
        c, i = divmod(w, KWARPS)
        if c >= self.NC:
            return self.U
        cs, ce = self.cta_unit0(c), self.cta_unit0(c + 1)
        nw = self.cta_warps(ce - cs)
        return ce if i >= nw else cs + i * (ce - cs) // nw

    def warp_of_unit(self, u: int) -> int:
        if not self.tiles:
            return warp_of(u, self.U, self.NW)
        c = warp_of(u // self.ng, self.T, self.NC)
        cs = self.cta_unit0(c)
        uc = self.cta_unit0(c + 1) - cs
        return c * KWARPS + warp_of(u - cs, uc, self.cta_warps(uc))


CASES = [(688, 8), (128, 43), (256, 16), (512, 32), (640, 32), (1792, 32), (4, 1), (1, 1), (1, 112),
         (64, 32), (3, 43), (147, 8), (149, 8), (600, 16), (16, 1), (2, 256)]
rng = random.Random(7)
CASES += [(rng.randint(1, 4000), rng.choice([1, 2, 4, 8, 16, 20, 32, 43, 112])) for _ in range(120)]


@pytest.mark.parametrize("ntiles,ng", CASES)
def test_split_invariants(ntiles, ng):
    g = Grid(ntiles, ng)
    owner = [-1] * g.U
    for w in range(g.NC * KWARPS):
        a, b = g.warp_unit0(w), g.warp_unit0(w + 1)
        assert a <= b
        tiles_of_w = set()
        for u in range(a, b):
            assert owner[u] == -1
            owner[u] = w
            tiles_of_w.add(u // ng)
        # a warp's tiles are consecutive; only its first and last can be shared
        if tiles_of_w:
            assert max(tiles_of_w) - min(tiles_of_w) + 1 == len(tiles_of_w)
    assert all(o >= 0 for o in owner)
    for u in range(g.U):
        assert g.warp_of_unit(u) == owner[u]
    for t in range(ntiles):
        wa, wb = owner[t * ng], owner[t * ng + ng - 1]
        if g.tiles:
            assert wa // KWARPS == wb // KWARPS
        for w in range(wa + 1, wb):  # the warps between hold only this tile, and something of it
            a, b = g.warp_unit0(w), g.warp_unit0(w + 1)
            assert a < b and a >= t * ng and b <= t * ng + ng
    for c in range(g.NC):
        a, b = g.cta_unit0(c), g.cta_unit0(c + 1)
        if b > a:
            assert (b - 1) // ng - a // ng + 1 <= g.cta_tiles
