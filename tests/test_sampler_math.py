"""The arithmetic the device sampler relies on, restated on the CPU (no GPU).

`select.cu` evaluates NumPy's pairwise float32 sum on a complete binary tree of
2^D slots and, when some probability is not a multiple of 2^-52, proves its
integer-scan pick against the float64 running sum by a margin. These tests pin
both arguments against NumPy itself: the slot-tree order gives `np.sum`'s
result bit for bit, and every proven pick equals `searchsorted(cumsum/last, u,
'right')`, the index `np.random.choice` returns (data_selection.py:641-675).
"""
from fractions import Fraction

import numpy as np
import pytest

PW_BLOCK = 128


def _leaf(a):
    """NumPy's pairwise leaf: a running sum below 8, else 8 accumulators then the tail."""
    n = len(a)
    if n < 8:
        r = np.float32(0)
        for x in a:
            r = np.float32(r + x)
        return r
    acc = [a[j] for j in range(8)]
    full = n - n % 8
    for i in range(8, full, 8):
        for j in range(8):
            acc[j] = np.float32(acc[j] + a[i + j])
    res = np.float32(np.float32(np.float32(acc[0] + acc[1]) + np.float32(acc[2] + acc[3]))
                     + np.float32(np.float32(acc[4] + acc[5]) + np.float32(acc[6] + acc[7])))
    for i in range(full, n):
        res = np.float32(res + a[i])
    return res


def _depth(m):
    d, ln = 0, m
    while ln > PW_BLOCK:
        ln -= (ln // 2) & ~7
        d += 1
    return d


def _slot_tree_sum(a):
    """The device order: slot g descends along its bits; pairs of slots combine level by level."""
    m = len(a)
    depth = _depth(m)
    sums = []
    for g in range(1 << depth):
        a0, ln = 0, m
        for d in range(depth - 1, -1, -1):
            right = (g >> d) & 1
            if ln > PW_BLOCK:
                n2 = (ln // 2) & ~7
                if right:
                    a0, ln = a0 + n2, ln - n2
                else:
                    ln = n2
            elif right:
                ln = 0
        sums.append(_leaf(a[a0:a0 + ln]) if ln else np.float32(0))
    v = np.array(sums, np.float32)
    while len(v) > 1:
        v = (v[0::2] + v[1::2]).astype(np.float32)
    return np.float32(np.float32(0) + v[0])


def test_slot_tree_reproduces_numpy_pairwise_sum():
    rng = np.random.default_rng(0)
    ms = list(range(1, 300)) + [1023, 1024, 2047, 2048, 4095, 4096, 7695, 7696, 8191, 8192]
    ms += [int(x) for x in rng.integers(300, 8193, 40)]
    for m in ms:
        a = (rng.random(m) ** 8).astype(np.float32) * np.float32(rng.choice([1e-3, 1.0, 1e3]))
        assert _slot_tree_sum(a) == np.float32(a.sum()), m


def test_split_depth_is_the_right_spine_and_fits_the_slots():
    """The right piece is never shallower, so the depth is a walk down the right spine;
    at most 128 slots (8 lanes each) for up to 8192 candidates."""

    def exact(m):
        if m <= PW_BLOCK:
            return 0
        n2 = (m // 2) & ~7
        return 1 + max(exact(n2), exact(m - n2))

    assert all(exact(m) == _depth(m) for m in range(1, 8193, 7))
    assert max(_depth(m) for m in range(1, 8193)) == 7


def _p52(p):
    return int(Fraction(float(p)) * (1 << 52))


def _threshold(u, total):
    """max{X : RN(X / total) <= u} by bisection on IEEE division."""
    lo, hi = -1, total
    while lo < hi:
        mid = (lo + hi + 1) // 2
        if float(mid) / float(total) <= u:
            lo = mid
        else:
            hi = mid - 1
    return lo


@pytest.mark.parametrize("spread", [3.0, 10.0, 20.0])
def test_margin_proven_pick_matches_searchsorted(spread):
    rng = np.random.default_rng(int(spread))
    proven = 0
    for _ in range(40):
        m = int(rng.integers(2, 700))
        x = (rng.standard_normal(m) * spread).astype(np.float32)
        x -= x.max()
        p = np.exp(x.astype(np.float64)).astype(np.float32)
        p = (p / np.float32(p.sum())).astype(np.float32)
        c = p.astype(np.float64).cumsum()
        cdf = c / c[-1]
        T = np.cumsum(np.array([_p52(v) for v in p], dtype=object))
        total = int(T[-1])
        us = list(rng.random(4))
        for j in rng.integers(0, m - 1, 2):
            us += [float(cdf[j]), float(np.nextafter(cdf[j], 0.0))]
        for u in us:
            if u >= 1.0:  # a cdf entry can round to 1; random_sample never returns it
                continue
            want = int(np.searchsorted(cdf, u, side="right"))
            thr = _threshold(u, total)
            q = next(i for i in range(m) if T[i] > thr)
            e = 2.0 * m + 2.0
            ok = True
            if q != m - 1:
                ok = float(T[q]) - e >= (u * (float(total) + e)) * (1 + 2.0 ** -50)
            if q != 0:
                ok = ok and float(T[q - 1]) + e <= (u * (float(total) - e)) * (1 - 2.0 ** -50)
            if ok:
                proven += 1
                assert q == want, (m, u)
    assert proven >= 160  # every random u is proven; u on a cdf entry may fall back
