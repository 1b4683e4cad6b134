"""CPU: the logic of the block-wide sequential sum that the RMSNorm prologues
use (llmq_spec_sum.cuh), restated with numpy float32 and run on chosen rows.

The kernel cuts the row into 32 segments, estimates each segment's start from
the segments' shifts, runs every segment from 8 candidate starts around its
estimate (consecutive bit patterns), and walks the segments in order using only
runs whose start equals the exact partial sum, summing a segment itself when the
exact start is not a candidate.  Whatever the estimates, the result must be the
plain loop's bit for bit; the rows here include ones that defeat the estimates,
so the fallback path is exercised too."""
from __future__ import annotations

import numpy as np
import pytest

f32 = np.float32
SEG, C = 32, 8


def _loop(v, acc=f32(0)):
    s = f32(acc)
    for t in v:
        s = f32(s + t)
    return s


def _bits(x):
    return int(np.asarray(x, f32).view(np.uint32))


def _float(b):
    return np.asarray(b & 0xFFFFFFFF, np.uint32).view(f32)[()]


def _chains(v, L, starts):
    """Segment j's loop from starts[..., j], for every j at once."""
    s = starts.astype(f32).copy()
    n = len(v)
    for i in range(L):
        idx = np.arange(SEG) * L + i
        live = idx < n
        t = np.where(live, v[np.minimum(idx, n - 1)], f32(-0.0)).astype(f32)  # x + (-0) == x for every x
        with np.errstate(all="ignore"):
            s = (s + t).astype(f32)
    return s


def spec_sum(v, acc=f32(0)):
    """Restatement of spec_seq_sum; returns (sum, fallback segments)."""
    v = np.asarray(v, f32)
    n = len(v)
    L = -(-n // SEG)
    L = (L + 3) & ~3
    if (L >> 2) % 2 == 0:
        L += 4
    segs = [v[min(n, j * L):min(n, j * L + L)] for j in range(SEG)]
    with np.errstate(all="ignore"):
        segsum = np.array([np.sum(s, dtype=f32) for s in segs], f32)       # 1. any order will do
        b = np.concatenate([[f32(acc)], (np.cumsum(segsum, dtype=f32)[:-1] + f32(acc)).astype(f32)]).astype(f32)
        d = (_chains(v, L, b) - b).astype(f32)                               # 2. shift of every segment
    est = np.zeros(SEG + 1, f32)
    S = f32(acc)
    for w in range(SEG):
        est[w] = S
        with np.errstate(all="ignore"):
            S = f32(S + d[w])
    est[SEG] = S
    eb = est.view(np.uint32).astype(np.int64)
    ends = np.zeros((C, SEG), f32)                                           # 3. candidates
    for c in range(C):
        st = ((eb[:SEG] + (c - C // 2)) & 0xFFFFFFFF).astype(np.uint32).view(f32)
        ends[c] = _chains(v, L, st)
    S, w, miss = f32(acc), 0, 0                                              # 4. the walk
    while w < SEG:
        c = _bits(S) - int(eb[w]) + C // 2
        if 0 <= c < C:
            off = c - C // 2
            while True:  # follow the run of segments that keep the offset
                e = ends[c][w]
                w += 1
                if w == SEG or _bits(e) != ((int(eb[w]) + off) & 0xFFFFFFFF):
                    S = e
                    break
        else:
            S = _loop(segs[w], S)
            miss += 1
            w += 1
    return S, miss


def _rows(n, rng):
    x = rng.standard_normal(n).astype(f32)
    drift = np.zeros(n, f32)
    drift[0] = s = f32(1.0)
    for k in range(1, n):
        drift[k] = t = f32(np.spacing(s) * f32(0.75))
        s = f32(s + t)
    out = {
        "gaussian squares": (x * x).astype(f32),
        "scaled squares with outliers": (np.where(rng.uniform(size=n) < 0.003, x * 300, x * 0.01) ** 2).astype(f32),
        "half zeros": np.where(rng.uniform(size=n) < 0.5, f32(0), x * x).astype(f32),
        "rounding always up": drift,
        "signed terms": x,
        "signed, large": (x * 1e4).astype(f32),
        "constant": np.full(n, f32(0.1)),
        "subnormal": np.full(n, f32(1e-42)),
        "overflow": np.full(n, f32(3e37)),
    }
    nan_row = (x * x).astype(f32)
    nan_row[n // 3] = np.nan
    out["nan"] = nan_row
    inf_row = (x * x).astype(f32)
    inf_row[n // 2] = np.inf
    out["inf"] = inf_row
    return out


@pytest.mark.parametrize("n", [1024, 1500, 4096, 8192])
def test_spec_sum_restatement_equals_the_loop(n):
    rng = np.random.default_rng(n)
    fallbacks = {}
    for name, v in _rows(n, rng).items():
        with np.errstate(all="ignore"):
            want = np.add.accumulate(v, dtype=f32)[-1]
        got, miss = spec_sum(v)
        fallbacks[name] = miss
        if np.isnan(want):
            assert np.isnan(got), name
        else:
            assert _bits(got) == _bits(want), name
    assert fallbacks["gaussian squares"] <= 2
    # the estimates fail (partial sums of both signs; a sum that overflows to
    # inf, whose shifts are inf - inf): the walk sums those segments itself
    assert fallbacks["signed, large"] > 0
    assert fallbacks["overflow"] > 0


def test_spec_sum_restatement_with_a_start_value():
    rng = np.random.default_rng(3)
    v = (rng.standard_normal(4096) ** 2).astype(f32)
    for acc in (f32(0), f32(-0.0), f32(123.25), f32(1e30), f32(-5.0)):
        got, _ = spec_sum(v, acc)
        assert _bits(got) == _bits(_loop(v, acc))
