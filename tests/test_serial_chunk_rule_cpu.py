"""CPU check of the chunk rule behind the serial-order Sum kernels (unpopped_b200/csrc/spec.cuh).

A numpy restatement of the row kernel's decisions must give the plain serial f64 fold's bits
(oracle/plan_eval.rs:566-645: s = ((0 + x0) + x1) + ..., one rounding) on data built to stress it. The row kernel
works in segments of 32 chunks of 64 values, with one test per segment from the running sum and a chunk-by-chunk
walk with value-by-value folds where the test fails. Here the segment test uses exact rational arithmetic, the
weakest bound the rule allows (the kernel's upward-rounded sums pass less often). This tests the rule, not the CUDA
code; the GPU tests compare the kernels with the oracle.
"""
import math
from fractions import Fraction

import numpy as np
import pytest

CHUNK = 64
SEGMENT = 32 * CHUNK


def _summary(v):
    """(T, H, L) of one chunk: the f64 prefix sum in fold order, its largest magnitude rounded up to f32 (+inf
    unless it is below L and T is finite), and 2^(q + 53) for q the smallest ulp exponent of the nonzero values."""
    pre = np.cumsum(np.concatenate(([0.0], v.astype(np.float64))))[1:]  # the fold's own partial sums from +0
    t = float(pre[-1])
    hi = float(np.max(np.abs(pre)))
    bits = v.view(np.uint32)
    nz = bits[(bits & 0x7FFFFFFF) != 0]
    if nz.size == 0:
        lim = math.inf
    else:
        e = max(int(((nz >> 23) & 0xFF).min()), 1)
        lim = 2.0 ** (e - 150 + 53)
    if hi < lim and math.isfinite(t):
        h = np.float32(hi)
        if float(h) < hi:
            h = np.nextafter(h, np.float32(np.inf))
        h = float(h)
    else:
        h = math.inf
    return t, h, lim


def _anchor(s):
    """2^(lowbit(s) + 53) for a finite nonzero s, +inf otherwise."""
    if s == 0.0 or not math.isfinite(s):
        return math.inf
    m, e = math.frexp(s)
    mant = int(abs(m) * 2.0 ** 53)
    tz = (mant & -mant).bit_length() - 1
    return 2.0 ** min(e - 53 + tz + 53, 1023)


def _spec_row(v, counts):
    s, lim = 0.0, math.inf
    n = v.size
    for c0 in range(0, n, SEGMENT):
        chunks = [v[c0 + j:min(c0 + j + CHUNK, n)] for j in range(0, SEGMENT, CHUNK) if c0 + j < n]
        summ = [_summary(c) for c in chunks]
        l2 = min([lim] + [x[2] for x in summ])
        ok = math.isfinite(s) and all(math.isfinite(x[1]) for x in summ)
        if ok and math.isfinite(l2):
            ok = Fraction(abs(s)) + sum(Fraction(x[1]) for x in summ) < Fraction(l2)
        if ok:
            ts = float(np.sum(np.array([x[0] for x in summ])))  # pairwise: any order is exact here
            s += ts
            lim = l2
            counts["segments"] += 1
            continue
        for (t, h, lc), c in zip(summ, chunks):
            lim = min(lim, lc)
            if abs(s) + h < lim:
                s += t
            else:
                for x in c:
                    s += float(x)
                lim = _anchor(s)
                counts["folds"] += 1
    return s


def _rows(rng, kind, n):
    if kind == "normal":
        return rng.standard_normal(n)
    if kind == "uniform":
        return rng.random(n)
    if kind == "tiny":
        v = rng.standard_normal(n)
        v[rng.random(n) < 0.01] = rng.choice([2.0 ** -40, -3.0 * 2.0 ** -45, 2.0 ** -30], 1)[0]
        return v
    if kind == "binades":
        return np.where(rng.random(n) < 0.7, 1.0, rng.choice([2.0 ** -28, 2.0 ** -52, 3.0 * 2.0 ** 24], n))
    if kind == "spread":
        return (rng.random(n) - 0.5) * 2.0 ** rng.integers(-20, 20, n)
    if kind == "subnormal":
        return rng.standard_normal(n) * np.where(rng.random(n) < 0.5, 2.0 ** -135, 1.0)
    if kind == "zeros":
        return np.where(rng.random(n) < 0.5, -0.0, 0.0)
    v = rng.standard_normal(n).astype(np.float32)  # specials
    pick = rng.random(n)
    v[pick < 0.02] = 0.0
    v[(pick >= 0.02) & (pick < 0.04)] = -0.0
    v[(pick >= 0.04) & (pick < 0.042)] = np.inf
    v[(pick >= 0.042) & (pick < 0.044)] = -np.inf
    v.view(np.uint32)[pick > 0.998] = np.uint32(0x7FC00001)
    return v


KINDS = ["normal", "uniform", "tiny", "binades", "spread", "subnormal", "zeros", "specials"]


@pytest.mark.parametrize("kind", KINDS)
def test_chunk_rule_gives_the_serial_fold(kind):
    rng = np.random.default_rng(KINDS.index(kind) + 40)
    counts = {"segments": 0, "folds": 0}
    for n in (1, 63, 64, 65, 2047, 2048, 2049, 9000):
        for _ in range(6):
            v = np.ascontiguousarray(_rows(rng, kind, n), dtype=np.float32)
            with np.errstate(invalid="ignore"):  # inf - inf in the specials rows is part of the fold
                want = float(np.cumsum(np.concatenate(([0.0], v.astype(np.float64))))[-1])  # from +0, as the fold
                got = _spec_row(v, counts)
            if math.isnan(want):
                assert math.isnan(got), (kind, n)
            else:
                assert np.float64(got).tobytes() == np.float64(want).tobytes(), (kind, n, got, want)
    # the data reaches the branch it was built for
    if kind in ("normal", "uniform", "zeros"):
        assert counts["segments"] > 0
    if kind in ("tiny", "binades", "spread", "specials"):
        assert counts["folds"] > 0


def _walk(s, lim, chunks, summ, counts):
    """The chain over chunks in order from (s, lim): add T where |s| + H < lim, else fold the chunk's values."""
    for (t, h, lc), c in zip(summ, chunks):
        lim = min(lim, lc)
        if abs(s) + h < lim:
            s += t
        else:
            for x in c:
                s += float(x)
            lim = _anchor(s)
            counts["folds"] += 1
    return s, lim


def _rank_exact(s, lim, part):
    """One test for a whole rank from start s: |s| + MX + HM below min(lim, ML), in exact rationals."""
    sl, ml, mx, hm = part
    if not (math.isfinite(s) and math.isfinite(mx) and math.isfinite(hm)):
        return False
    bound = min(lim, ml)
    return math.isinf(bound) or Fraction(abs(s)) + Fraction(mx) + Fraction(hm) < Fraction(bound)


def _spec_column(v, counts, ranks=4, cap=32):
    """The cluster column kernel's round protocol for one column: each round's chunks split over `ranks`; each
    rank's SL (its T added in order), ML, MX (largest |partial| of SL) and HM (largest H); speculative starts from
    the carry plus SL of earlier ranks; if every rank's one test holds and every SL used is exact, the last rank's
    result carries, else the ranks go in order, keeping a result whose speculative start was the carry."""
    n = v.size
    chunks = [v[i:min(i + CHUNK, n)] for i in range(0, n, CHUNK)]
    summ = [_summary(c) for c in chunks]
    s, lim = 0.0, math.inf
    per_round = ranks * cap
    for g0 in range(0, len(chunks), per_round):
        nch = min(per_round, len(chunks) - g0)
        share = -(-nch // ranks)
        spans = [(g0 + min(nch, k * share), g0 + min(nch, (k + 1) * share)) for k in range(ranks)]
        parts = []
        for a, b in spans:
            sl, ml, mx, hm = 0.0, math.inf, 0.0, 0.0
            for t, h, lc in summ[a:b]:
                ml = min(ml, lc)
                hm = max(hm, h)
                sl += t
                mx = max(mx, abs(sl))  # a NaN partial is dropped, as fmax drops it
            parts.append((sl, ml, mx, hm))
        spec = []  # per rank: start, start lim, result, result lim, walk held, SL exact
        for k, (a, b) in enumerate(spans):
            si, li = s, lim
            for q in range(k):
                si += parts[q][0]
                li = min(li, parts[q][1])
            if _rank_exact(si, li, parts[k]):
                so, lo, wok = si + parts[k][0], min(li, parts[k][1]), True
            else:
                so, lo, wok = si, li, True
                for t, h, lc in summ[a:b]:
                    lo = min(lo, lc)
                    wok &= abs(so) + h < lo
                    so += t
            exact = k == ranks - 1 or parts[k][2] < parts[k][1]
            spec.append((si, li, so, lo, wok, exact))
        if all(w and e for (_, _, _, _, w, e) in spec):
            s, lim = spec[-1][2], spec[-1][3]
            counts["segments"] += 1
            continue
        for k, (a, b) in enumerate(spans):  # rank order from the true carry
            si, li, so, lo, wok, _ = spec[k]
            same = wok and np.float64(s).tobytes() == np.float64(si).tobytes() and lim == li
            if same:
                s, lim = so, lo
            elif _rank_exact(s, lim, parts[k]):
                s, lim = s + parts[k][0], min(lim, parts[k][1])
            else:
                s, lim = _walk(s, lim, chunks[a:b], summ[a:b], counts)
    return s


@pytest.mark.parametrize("kind", KINDS)
def test_cluster_round_protocol_gives_the_serial_fold(kind):
    rng = np.random.default_rng(KINDS.index(kind) + 80)
    counts = {"segments": 0, "folds": 0}
    for n in (1, 64, 65, 1000, 8192, 8193, 20000):
        for _ in range(4):
            v = np.ascontiguousarray(_rows(rng, kind, n), dtype=np.float32)
            with np.errstate(invalid="ignore"):
                want = float(np.cumsum(np.concatenate(([0.0], v.astype(np.float64))))[-1])
                got = _spec_column(v, counts)
            if math.isnan(want):
                assert math.isnan(got), (kind, n)
            else:
                assert np.float64(got).tobytes() == np.float64(want).tobytes(), (kind, n, got, want)
    if kind in ("normal", "uniform", "zeros"):
        assert counts["segments"] > 0
    if kind in ("tiny", "binades", "spread", "specials"):
        assert counts["folds"] > 0
