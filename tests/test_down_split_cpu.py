"""CPU check of the cost-weighted work split of the grouped down GEMM
(warp-route_b200/csrc/wr_grouped.cu: down_chunk_cost, down_cost_of,
make_costsplit, WorkIter<false>, k_combine), restated here in Python.

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
