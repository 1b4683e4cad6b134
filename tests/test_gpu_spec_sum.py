"""GPU: the block-wide sequential sum of the RMSNorm prologues (rmsnorm.c:15).

The row's 32 segments run in parallel from candidate starts around estimated
partial sums; one thread links them in order using only runs whose start is the
exact partial sum, summing a segment itself when no candidate matches.  The
result must equal the one-thread loop (and numpy's sequential float32 sum) bit
for bit on every row, whether the candidates match or not.  Signed and
overflowing rows defeat the estimates and force that fallback; drifting,
infinite, NaN and subnormal rows check that nothing but speed depends on the
estimates."""
from __future__ import annotations

import ctypes as C

import numpy as np
import pytest

from helpers import fp

pytestmark = pytest.mark.gpu

f32 = np.float32


def _seq(v: np.ndarray) -> np.float32:
    """The C loop s = 0; for k: s = s + v[k], in float32."""
    return np.add.accumulate(v.astype(f32), dtype=f32)[-1] if len(v) else f32(0)


def _run(lib, rows: np.ndarray, threads: int = 512):
    rows = np.ascontiguousarray(rows, dtype=f32)
    R, n = rows.shape
    sums = np.zeros(2 * R, f32)
    misses = np.zeros(R, np.int32)
    cycles = np.zeros(2 * R, np.int64)
    rc = lib.llmq_spec_sum_check(fp(rows), R, n, threads, fp(sums), misses.ctypes.data_as(C.POINTER(C.c_int)),
                                 cycles.ctypes.data_as(C.POINTER(C.c_longlong)))
    assert rc == 0, lib.q_llama_last_error_message()
    return sums[0::2], sums[1::2], misses, cycles[0::2], cycles[1::2]


def _drifting_row(n: int, start: float = 1.0) -> np.ndarray:
    """Terms of 3/4 ulp of the running float32 sum: every add rounds up by a
    quarter ulp, so the loop drifts n/4 ulps above the exact sum."""
    v = np.zeros(n, f32)
    v[0] = s = f32(start)
    for k in range(1, n):
        v[k] = t = f32(np.spacing(s) * f32(0.75))
        s = f32(s + t)
    return v


def _squares(x):
    x = x.astype(f32)
    return (x * x).astype(f32)


@pytest.mark.parametrize("n", [1000, 1024, 1031, 4096, 5000, 6144, 6145, 8192, 14336])
def test_spec_sum_equals_loop_on_gaussian_squares(lib, n):
    rng = np.random.default_rng(n)
    rows = np.stack([_squares(rng.standard_normal(n) * rng.uniform(0.05, 20)) for _ in range(12)])
    rows[1, rng.integers(0, n, 6)] *= 4000.0  # outlier dimensions
    spec, loop, misses, _, _ = _run(lib, rows)
    want = np.array([_seq(r) for r in rows], f32)
    assert np.array_equal(spec.view(np.uint32), loop.view(np.uint32))
    assert np.array_equal(spec.view(np.uint32), want.view(np.uint32))


@pytest.mark.parametrize("threads", [64, 96, 128, 256, 512, 1024])
def test_spec_sum_block_sizes(lib, threads):
    rng = np.random.default_rng(threads)
    rows = np.stack([_squares(rng.standard_normal(4096)) for _ in range(4)] +
                    [_squares(rng.standard_normal(4096) * 1e-3), _drifting_row(4096)])
    spec, loop, _, _, _ = _run(lib, rows, threads)
    want = np.array([_seq(r) for r in rows], f32)
    assert np.array_equal(spec.view(np.uint32), want.view(np.uint32))
    assert np.array_equal(loop.view(np.uint32), want.view(np.uint32))


@pytest.mark.parametrize("n", [4096, 8192])
def test_spec_sum_rows_that_defeat_the_estimates(lib, n):
    """Rows whose every add rounds the same way (the partial sums drift far from
    the exact prefix), a signed row and a row that overflows to inf: exact in
    every case; on the last the estimates fail and segments are summed again."""
    rng = np.random.default_rng(n + 1)
    rows = np.stack([_drifting_row(n, 1.0), _drifting_row(n, 1e-30), _drifting_row(n, 7.5),
                     (rng.standard_normal(n) * 1e4).astype(f32), np.full(n, f32(3e37))])
    spec, loop, misses, _, _ = _run(lib, rows)
    with np.errstate(all="ignore"):
        want = np.array([_seq(r) for r in rows], f32)
    assert np.array_equal(spec.view(np.uint32), want.view(np.uint32))
    assert np.array_equal(loop.view(np.uint32), want.view(np.uint32))
    assert misses[4] > 0  # after the overflow the shifts are inf - inf: segments summed by one thread


def test_spec_sum_signed_special_and_extreme_rows(lib):
    rng = np.random.default_rng(5)
    n = 4096
    rows = [
        rng.standard_normal(n).astype(f32),                               # signed terms
        np.zeros(n, f32),
        np.full(n, f32(1e-42)),                                           # subnormal terms
        np.full(n, f32(3e37)),                                            # overflows to inf part-way
        _squares(rng.standard_normal(n)),
        _squares(rng.standard_normal(n)),
        _squares(rng.standard_normal(n)),
        np.where(rng.uniform(size=n) < 0.5, f32(0.0), _squares(rng.standard_normal(n) * 100)),
    ]
    rows[4][1234] = np.inf
    rows[5][3000] = np.nan
    rows[6][100] = -np.inf
    rows = np.stack(rows).astype(f32)
    with np.errstate(all="ignore"):
        want = np.array([_seq(r) for r in rows], f32)
    spec, loop, _, _, _ = _run(lib, rows)
    # NaN results carry the GPU's NaN pattern on both paths: compare bits
    # between the two GPU paths, and values against the host loop
    assert np.array_equal(spec.view(np.uint32), loop.view(np.uint32))
    nan = np.isnan(want)
    assert np.array_equal(np.isnan(spec), nan)
    assert np.array_equal(spec[~nan].view(np.uint32), want[~nan].view(np.uint32))


def test_spec_sum_is_faster_than_the_loop(lib):
    """Latency of one row in SM cycles (a 4096-term row is the 8B model's
    RMSNorm, 8192 the 70B's); reported for the design notes."""
    rng = np.random.default_rng(11)
    for n in (4096, 8192):
        rows = np.stack([_squares(rng.standard_normal(n)) for _ in range(8)])
        spec, loop, misses, c_spec, c_loop = _run(lib, rows)
        assert np.array_equal(spec.view(np.uint32), loop.view(np.uint32))
        print(f"n={n}: block sum {np.median(c_spec):.0f} cycles, loop {np.median(c_loop):.0f} cycles, "
              f"misses per row {misses.tolist()}")
        assert np.median(c_spec) * 2 < np.median(c_loop)
