"""The chunked exact-sum scheme of the stats kernel, emulated on the CPU
against the reference's serial fp32 sum (the oracle's order).

The reference adds a group's terms t one at a time in fp32 (rows in order,
16 columns per row).  The kernel splits the rows into chunks processed in
parallel and proves, per run of 16 terms (one row), which binade the running
sum is in, from an fp64 prediction of the prefix and a rigorous bound on how
far the fp32 sum can drift from it.  Inside a known binade every add is an
integer add on that binade's grid, so a run is summarised by a transfer
function of the sum's parity (ties round to even).  Runs whose binade is not
proven ("windows") are replayed one term at a time by the assembler, which
walks the chunk programs in order starting from the exact sum.

This emulation follows those rules with numpy float32/float64 arithmetic and
checks the result bit for bit on inputs chosen to hit every branch."""
import math

import numpy as np
import pytest

F = np.float32
EPS = 2.0 ** -24


def serial(t: np.ndarray) -> np.float32:
    s = F(0)
    with np.errstate(over="ignore", invalid="ignore"):
        for x in t.reshape(-1):
            s = F(s + x)
    return s


def binade(x: float) -> int:
    return math.frexp(x)[1] - 1  # x in [2^e, 2^(e+1))


def run_tf(t: np.ndarray, e: int):
    """(inc[2], pout[2]) of one run of terms inside binade e."""
    x = (t.astype(np.float64) * 2.0 ** (23 - e)).astype(np.float32)  # exact power-of-2 scaling
    k = np.rint(x)
    tie = np.abs(x - k) == 0.5
    inc, pout = [0, 0], [0, 0]
    for p_in in (0, 1):
        p, acc = p_in, 0
        for c in range(t.size):
            if tie[c]:
                f = int(np.floor(x[c]))
                d = f + ((p + f) & 1)
            else:
                d = int(k[c])
            acc += d
            p = (p + d) & 1
        inc[p_in], pout[p_in] = acc, p
    return inc, pout


def compose(a, b):
    """Transfer function of a followed by b."""
    inc = [a[0][p] + b[0][a[1][p]] for p in (0, 1)]
    pout = [b[1][a[1][p]] for p in (0, 1)]
    return inc, pout


def chunk_program(t_runs, pr, p_start, run0, runs_per_chunk):
    """Items of one chunk: ("S", e, tf, a, b) stretches and ("W", a, b) windows
    (run indices a..b-1 within the group)."""
    items = []
    cur = None  # open stretch: [e, tf, a, b]
    p = p_start
    for j in range(run0, min(run0 + runs_per_chunk, len(t_runs))):
        t = t_runs[j]
        p_s, p_e = p, p + float(pr[j])
        p = p_e
        if not np.all(np.isfinite(t)):
            kind = "U"
        elif np.all(t == 0):
            kind = "Z"
        else:
            d_s, d_e = (16 * j + 64) * EPS, (16 * (j + 1) + 64) * EPS
            lo, hi = p_s * (1.0 - d_s), p_e * (1.0 + 2.0 * d_e)
            kind = "C" if (d_e < 0.25 and lo >= 2.0 ** -100 and binade(lo) == binade(hi)) else "U"
        if kind == "Z":
            if cur is not None and cur[0] != "W":
                cur[3] = j + 1
            elif cur is not None:
                cur[2] = j + 1
            continue
        if kind == "C":
            e = binade(lo)
            tf = run_tf(t, e)
            if cur is not None and cur[0] != "W" and cur[0] == e:
                cur[1] = compose(cur[1], tf)
                cur[3] = j + 1
            else:
                if cur is not None:
                    items.append(tuple(cur))
                cur = [e, tf, j, j + 1]
        else:
            if cur is not None and cur[0] == "W":
                cur[2] = j + 1
            else:
                if cur is not None:
                    items.append(tuple(cur))
                cur = ["W", j, j + 1]
    if cur is not None:
        items.append(tuple(cur))
    return items


def assemble(programs, t_runs, stats, any_nan=False, any_inf=False):
    """Walk the programs from S = 0.  Non-finite terms are settled per group:
    every term is >= 0 or NaN, so the serial sum ends NaN if any term is NaN,
    else inf if any term is inf (or the finite sum overflowed)."""
    if any_nan:
        return F(np.nan)
    if any_inf:
        return F(np.inf)
    s = F(0)
    for items in programs:
        if not np.isfinite(s):
            break
        for it in items:
            if not np.isfinite(s):
                break
            if it[0] == "W":
                for j in range(it[1], it[2]):
                    with np.errstate(over="ignore", invalid="ignore"):
                        for x in t_runs[j]:
                            s = F(s + x)
                stats["window_runs"] += it[2] - it[1]
                continue
            e, tf, a, b = it
            ok = bool(np.isfinite(s)) and s > 0 and binade(float(s)) == e
            if ok:
                m = int(float(s) * 2.0 ** (23 - e))
                m2 = m + tf[0][m & 1]
                ok = m2 < 2 ** 24
            if ok:
                s = F(m2 * 2.0 ** (e - 23))
            else:  # the proof failed: replay exactly
                stats["fallbacks"] += 1
                for j in range(a, b):
                    for x in t_runs[j]:
                        s = F(s + x)
    return s


def chunked_sum(x: np.ndarray, h: np.ndarray, rows_per_chunk: int, stats=None):
    """x: w*w as float32 [rows, 16]; h: [16] divisors (<= 1e-8: none)."""
    stats = {"window_runs": 0, "fallbacks": 0} if stats is None else stats
    div = h > 1e-8
    r = np.where(div, (1.0 / h.astype(np.float64)).astype(np.float32), F(1))
    with np.errstate(over="ignore", invalid="ignore", divide="ignore"):
        t = np.where(div[None, :], (x / np.where(div, h, F(1))[None, :]).astype(np.float32), x)
        pr_raw = (x.astype(np.float64) * r.astype(np.float64)).sum(axis=1)
    pr = np.where(np.isfinite(pr_raw), pr_raw, 0.0)
    n_runs = t.shape[0]
    programs, p_start = [], 0.0
    for run0 in range(0, n_runs, rows_per_chunk):
        programs.append(chunk_program(t, pr, p_start, run0, rows_per_chunk))
        p_start += float(pr[run0:run0 + rows_per_chunk].sum())
    any_nan = bool(np.isnan(pr_raw).any())
    any_inf = bool(np.isinf(pr_raw).any())
    return assemble(programs, t, stats, any_nan, any_inf), t, stats


def _case(kind: str, rows: int, seed: int):
    rng = np.random.default_rng(seed)
    w = (rng.standard_normal((rows, 16)) * 0.02).astype(np.float16)
    h = np.ones(16, np.float32)
    if kind == "lognormal":
        h = np.exp(rng.standard_normal(16) * 1.5).astype(np.float32)
    elif kind == "ties":      # few distinct values, h = 1: many exact halves
        w = (rng.integers(-8, 9, (rows, 16)) * 0.125).astype(np.float16)
    elif kind == "zeros":     # long zero stretches, then a jump
        w[: rows // 2] = 0
        w[rows // 2 + 3, 5] = 30.0
    elif kind == "tiny":      # subnormal fp16 squares, tiny h
        w = (rng.standard_normal((rows, 16)) * 1e-6).astype(np.float16)
        h = np.full(16, 2e-8, np.float32)
    elif kind == "range":     # huge dynamic range across rows
        w = (rng.standard_normal((rows, 16)) * np.exp(rng.uniform(-9, 9, (rows, 1)))).astype(np.float16)
        h = np.exp(rng.uniform(-20, 20, 16)).astype(np.float32)
    elif kind == "mixed_h":   # some columns without division, some huge divisors
        h = np.array([0, 1e-9, 1, 2, 3e30, 0.5, -1, 7, 1e-8, 1.1e-8, 4, 5, 6, 7, 8, 9], np.float32)
    elif kind == "inf":
        w[rows // 3, 2] = np.inf
    elif kind == "nan":
        w[rows // 2, 7] = np.nan
    elif kind == "growth":    # terms growing along the rows: many late crossings
        w = (rng.standard_normal((rows, 16)) * np.linspace(0.001, 1, rows)[:, None]).astype(np.float16)
    x = (w.astype(np.float32) ** 2).astype(np.float32)
    return x, h


KINDS = ["normal", "lognormal", "ties", "zeros", "tiny", "range", "mixed_h", "inf", "nan", "growth"]


@pytest.mark.parametrize("kind", KINDS)
@pytest.mark.parametrize("rows,chunk", [(2048, 128), (1000, 64), (37, 32), (4096, 256)])
def test_chunked_sum_bit_exact(kind, rows, chunk):
    x, h = _case(kind, rows, seed=rows + len(kind))
    stats = {"window_runs": 0, "fallbacks": 0}
    got, t, stats = chunked_sum(x, h, chunk, stats)
    want = serial(t)
    assert np.array_equal(np.array(got).view(np.uint32), np.array(want).view(np.uint32)) or \
        (np.isnan(got) and np.isnan(want)), (got, want)
    assert stats["fallbacks"] == 0


def test_windows_are_a_small_fraction():
    """On the benchmark-like distribution only runs near binade crossings are
    replayed term by term."""
    x, h = _case("lognormal", 4096, seed=1)
    stats = {"window_runs": 0, "fallbacks": 0}
    chunked_sum(x, h, 128, stats)
    assert stats["window_runs"] < 4096 * 0.05, stats
