"""CPU check of the cost-weighted work split of the grouped GEMMs
(warp-route_b200/csrc/wr_grouped.cu: chunk_cost, tile_cost_of,
make_costsplit, WorkIter, k_combine, the gate/up fixup's partial slots),
restated here in Python.

The device code walks each CTA's range of cost positions tile by tile, and
the combine finds a tile's CTAs from the positions the bucketing stores per
row.  The split is correct when, for every routing: each (tile, K chunk) is
taken by exactly one CTA, a CTA's partial slot stays below jmax, and the
CTAs the combine reads for a tile are exactly those that wrote it.  These
are checked over random skewed routings, including one-expert
(expert-parallel) shards that must still use every SM.
"""
from __future__ import annotations

import random

K_NMAX_B = 64
COST_ONE, COST_WIDE = 5, 6


def chunk_cost(n, nmax_b):
    if nmax_b > K_NMAX_B:
        return COST_WIDE if n > K_NMAX_B else COST_ONE
    return 1


def cost_of(cnt, nt, nmax_b, kc):
    np_ = (cnt + 15) & ~15
    wf = chunk_cost(nmax_b, nmax_b)
    wl = chunk_cost(np_ - (nt - 1) * nmax_b, nmax_b) if nt else 0
    r = kc * ((nt - 1) * wf + wl) if nt else 0
    return wf, wl, r


def split(cnts, nmax_b, kc, mt, grid, jmax):
    """Returns (G, {(tile, k): (cta, slot)}, [(tile, first cta, last cta)])."""
    E = len(cnts)
    ntl = [(((c + 15) & ~15) + nmax_b - 1) // nmax_b for c in cnts]
    cost_b, pre_b, wmax = [0], [0], 1
    for e in range(E):
        wf, wl, r = cost_of(cnts[e], ntl[e], nmax_b, kc)
        cost_b.append(cost_b[-1] + mt * r)
        pre_b.append(pre_b[-1] + mt * ntl[e])
        if ntl[e]:
            wmax = max(wmax, wf if ntl[e] > 1 else wl)
    C = cost_b[E]
    if C == 0:
        return 0, {}, []
    L = (kc + jmax - 2) // (jmax - 1)
    G = min(max(C // (L * wmax), 1), grid)
    lo = lambda c: c * C // G  # noqa: E731
    cta_of = lambda p: ((p + 1) * G - 1) // C  # noqa: E731
    taken = {}
    for c in range(G):
        p, p1 = lo(c), lo(c + 1)
        if p >= p1:
            continue
        e = 0
        while e + 1 < E and cost_b[e + 1] <= p:
            e += 1
        wf, wl, r = cost_of(cnts[e], ntl[e], nmax_b, kc)
        m = (p - cost_b[e]) // r
        tn = min((p - cost_b[e] - m * r) // (kc * wf), ntl[e] - 1)
        while p < p1 and e < E:
            nt = ntl[e]
            wf, wl, r = cost_of(cnts[e], nt, nmax_b, kc)
            wt = wl if tn == nt - 1 else wf
            pos = cost_b[e] + m * r + tn * kc * wf
            k0 = (p - pos + wt - 1) // wt if p > pos else 0
            k1 = min(kc, (p1 - pos + wt - 1) // wt)
            ce, cm, ctn = e, m, tn
            tn += 1
            if tn == nt:
                tn, m = 0, m + 1
                if m == mt:
                    m, e = 0, e + 1
                    while e < E and ntl[e] == 0:
                        e += 1
            if k0 >= kc:
                continue
            if k1 <= k0:
                break
            p = pos + k1 * wt
            tile = pre_b[ce] + cm * nt + ctn
            for k in range(k0, k1):
                assert (tile, k) not in taken
                taken[(tile, k)] = (c, c - cta_of(pos))
    spans = []
    for e in range(E):
        wf, wl, r = cost_of(cnts[e], ntl[e], nmax_b, kc)
        for m in range(mt):
            for tn in range(ntl[e]):
                wt = wl if tn == ntl[e] - 1 else wf
                pos = cost_b[e] + tn * kc * wf + m * r  # row_tile x + m * y
                spans.append((pre_b[e] + m * ntl[e] + tn, cta_of(pos),
                              cta_of(pos + (kc - 1) * wt)))
    return G, taken, spans


def _check(cnts, nmax_b, kc, mt, grid=148):
    jmax = max(4, min(16, (grid + mt - 1) // mt + 1))
    G, taken, spans = split(cnts, nmax_b, kc, mt, grid, jmax)
    ntl = [(((c + 15) & ~15) + nmax_b - 1) // nmax_b for c in cnts]
    assert len(taken) == sum(ntl) * mt * kc
    for tile, c0, c1 in spans:
        ctas = sorted({taken[(tile, k)][0] for k in range(kc)})
        assert ctas == list(range(c0, c1 + 1))
        for k in range(kc):
            cta, slot = taken[(tile, k)]
            assert slot == cta - c0 and 0 <= slot < jmax
    return G


def test_random_skewed_routings():
    rng = random.Random(1)
    for _ in range(400):
        E = rng.choice([1, 2, 3, 8, 16, 64])
        T = rng.choice([2, 16, 33, 64, 65, 100, 128, 256, 300])
        K = min(E, rng.choice([1, 2, 4, 8]))
        wts = [rng.random() ** 3 for _ in range(E)]
        cnts = [0] * E
        for _ in range(T * K):
            cnts[rng.choices(range(E), wts)[0]] += 1
        cnts = [min(c, T) for c in cnts]
        n16 = (T + 15) & ~15
        nmax_b = n16 if n16 <= K_NMAX_B else 128
        _check(cnts, nmax_b, rng.choice([1, 7, 64, 224]), rng.choice([1, 2, 16]))


def test_one_expert_shard_keeps_every_sm():
    # Mixtral down GEMM (16 H tiles x 224 K chunks), expert parallel over 8:
    # one local expert, with and without a tile above 64 tokens.
    for tokens in (40, 70, 129):
        assert _check([tokens], 128, 224, 16) == 148


# ---------------------------------------------------------------------------
# The cost walker both GEMMs share (wr_grouped.cu: chunk_cost, tile_cost_of,
# WorkIter, part_slot_of_piece / part_slot_of_cta), restated with the gate/up
# specifics: wide gate/up tiles (above 128 tokens) cost 7, the gate/up range
# that ends inside a tile walks that piece first, and a cut gate/up tile's
# partials are parked in slot 1 by its first CTA and in slot 0 by the others.

K_TOK_M = 128
COST_WIDE_A = 7


def chunk_cost_g(gu, n, nmax):
    narrow = K_TOK_M if gu else K_NMAX_B
    if nmax > narrow:
        return (COST_WIDE_A if gu else COST_WIDE) if n > narrow else COST_ONE
    return 1


def tile_cost(gu, cnt, nt, nmax, kc):
    np_ = (cnt + 15) & ~15
    wf = chunk_cost_g(gu, nmax, nmax)
    wl = chunk_cost_g(gu, np_ - (nt - 1) * nmax, nmax) if nt else 0
    r = kc * ((nt - 1) * wf + wl) if nt else 0
    return wf, wl, r


class Walker:
    """One CTA's WorkIter: the pieces (tile, k0, k1, pos, wt) in walk order."""

    def __init__(self, gu, cnts, nmax, kc, mt, grid, jmax):
        self.gu, self.cnts, self.nmax, self.kc, self.mt = gu, cnts, nmax, kc, mt
        E = len(cnts)
        self.ntl = [(((c + 15) & ~15) + nmax - 1) // nmax for c in cnts]
        self.cost, self.pre, wmax = [0], [0], 1
        for e in range(E):
            wf, wl, r = tile_cost(gu, cnts[e], self.ntl[e], nmax, kc)
            self.cost.append(self.cost[-1] + mt * r)
            self.pre.append(self.pre[-1] + mt * self.ntl[e])
            if self.ntl[e]:
                wmax = max(wmax, wf if self.ntl[e] > 1 else wl)
        self.C = self.cost[E]
        L = (kc + jmax - 2) // (jmax - 1)
        self.G = min(max(self.C // (L * wmax), 1), grid) if self.C else 0

    def lo(self, c):
        return c * self.C // self.G

    def cta_of(self, p):
        return ((p + 1) * self.G - 1) // self.C

    def seek(self, x):
        E = len(self.cnts)
        e = 0
        while e + 1 < E and self.cost[e + 1] <= x:
            e += 1
        wf, wl, r = tile_cost(self.gu, self.cnts[e], self.ntl[e], self.nmax, self.kc)
        m = (x - self.cost[e]) // r
        tn = min((x - self.cost[e] - m * r) // (self.kc * wf), self.ntl[e] - 1)
        return e, m, tn

    def tile_pos(self, e, m, tn):
        wf, wl, r = tile_cost(self.gu, self.cnts[e], self.ntl[e], self.nmax, self.kc)
        wt = wl if tn == self.ntl[e] - 1 else wf
        return self.cost[e] + m * r + tn * self.kc * wf, wt

    def stretch(self, p, p1, e, m, tn):
        E, kc = len(self.cnts), self.kc
        out = []
        while p < p1 and e < E:
            nt = self.ntl[e]
            pos, wt = self.tile_pos(e, m, tn)
            k0 = (p - pos + wt - 1) // wt if p > pos else 0
            k1 = min(kc, (p1 - pos + wt - 1) // wt)
            ce, cm, ctn = e, m, tn
            tn += 1
            if tn == nt:
                tn, m = 0, m + 1
                if m == self.mt:
                    m, e = 0, e + 1
                    while e < E and self.ntl[e] == 0:
                        e += 1
            if k0 >= kc:
                continue
            if k1 <= k0:
                break
            p = pos + k1 * wt
            out.append((self.pre[ce] + cm * nt + ctn, k0, k1, pos, wt))
        return out

    def pieces(self, c):
        p, p1 = self.lo(c), self.lo(c + 1)
        if p >= p1:
            return []
        if self.gu:
            e, m, tn = self.seek(p1 - 1)
            pos, wt = self.tile_pos(e, m, tn)
            k1 = (p1 - pos + wt - 1) // wt
            if k1 < self.kc and pos > p:
                return (self.stretch(pos, p1, e, m, tn) +
                        self.stretch(p, pos, *self.seek(p)))
        return self.stretch(p, p1, *self.seek(p))


def _check_walk(gu, cnts, nmax, kc, mt, grid=148):
    jmax = 3 if gu else max(4, min(16, (grid + mt - 1) // mt + 1))
    w = Walker(gu, cnts, nmax, kc, mt, grid, jmax)
    taken, slots = {}, {}
    for c in range(w.G):
        ps = w.pieces(c)
        if gu and ps:  # the end-cut piece, when there is one, comes first
            last = max(ps, key=lambda t: (t[3], t[1]))
            if last[2] < kc and len(ps) > 1:
                assert ps[0] == last
        for tile, k0, k1, pos, wt in ps:
            for k in range(k0, k1):
                assert (tile, k) not in taken
                taken[(tile, k)] = c
            cf, cl = w.cta_of(pos), w.cta_of(pos + (kc - 1) * wt)
            assert cf <= c <= cl and cl - cf < jmax
            if (k0, k1) != (0, kc):  # a cut piece: its parking slot
                slot = 1 if k0 == 0 else 0
                assert (c, slot) not in slots, "two cut pieces in one slot"
                slots[(c, slot)] = tile
                assert slot == (1 if c == cf else 0)  # what the fixup reads
    assert len(taken) == sum(w.ntl) * mt * kc
    return w.G


def test_cost_walker_both_gemms():
    rng = random.Random(2)
    for _ in range(400):
        E = rng.choice([1, 2, 3, 8, 16, 64])
        T = rng.choice([2, 16, 33, 64, 65, 100, 128, 129, 200, 256, 300])
        K = min(E, rng.choice([1, 2, 4, 8]))
        wts = [rng.random() ** 3 for _ in range(E)]
        cnts = [0] * E
        for _ in range(T * K):
            cnts[rng.choices(range(E), wts)[0]] += 1
        cnts = [min(c, T) for c in cnts]
        n16 = (T + 15) & ~15
        kc = rng.choice([1, 7, 16, 64, 224])
        mt = rng.choice([1, 2, 11, 16, 112])
        _check_walk(True, cnts, n16 if n16 <= K_TOK_M else 2 * K_TOK_M, kc, mt)
        _check_walk(False, cnts, n16 if n16 <= K_NMAX_B else 128, kc, mt)
        _check_walk(True, cnts, min(n16, 64), kc, mt)  # fp32 tiles: <= 64 tokens


def test_wide_gate_up_tile_on_one_expert():
    # expert-parallel shard with one expert of 129..256 tokens: wide tiles only
    for tokens in (129, 200, 256):
        assert _check_walk(True, [tokens], 256, 64, 112) == 148
