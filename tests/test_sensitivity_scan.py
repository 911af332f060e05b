"""The exact block-scan used by the sensitivity kernel, emulated in numpy
float32 with the same rules as `sens_stage` in memboost_b200/csrc/quantize.cu,
against the reference's serial fp32 sum (the oracle).  CPU only; this checks
the algorithm's logic on inputs chosen to hit every branch: binade crossings,
exact rounding ties, long zero runs, tiny and huge terms, inf and NaN."""
import numpy as np
import pytest

F = np.float32


def _bits(x):
    return int(np.array(x, np.float32).view(np.uint32))


def _from_bits(b):
    return np.array(b, np.uint32).view(np.float32)[()]


def emulate(terms: np.ndarray, rows: int) -> np.float32:
    """terms: float32 (n,) in serial order; rows: threads per block (16 terms each)."""
    per = rows * 16
    n = terms.size
    t_all = np.zeros(((n + per - 1) // per) * per, np.float32)
    t_all[:n] = terms
    S = F(0)
    for st in range(t_all.size // per):
        t = t_all[st * per:(st + 1) * per].reshape(rows, 16)
        frm = 0
        while frm < rows:
            if np.isfinite(S) and S >= F(2.0 ** -103):
                E = (_bits(S) >> 23) & 0xFF
                inv_q = _from_bits((277 - E) << 23)
                q = _from_bits((E - 23) << 23)
                m = F(S * inv_q)
                limit = F(F(16777216.0) - m)
                with np.errstate(over="ignore", invalid="ignore"):
                    a = (t * inv_q).astype(np.float32)
                    k = np.rint(a).astype(np.float32)
                    d = np.abs(a - k).astype(np.float32)
                loc = np.zeros(rows, np.float32)
                for i in range(16):
                    loc = (loc + k[:, i]).astype(np.float32)
                dmax = np.where(np.isnan(d), 0, d).max(axis=1)
                loc[:frm] = 0
                incl = np.cumsum(loc, dtype=np.float32)
                idx = np.arange(rows)
                with np.errstate(invalid="ignore"):
                    special = (idx >= frm) & ((dmax == 0.5) | ~(incl < limit))
                if not special.any():
                    S = F(S + F(incl[-1] * q))
                    break
                ls = int(np.argmax(special))
                excl = incl[ls - 1] if ls > 0 else F(0)  # exact: lanes before ls are exact
                s = F(S + F(excl * q))
                for i in range(16):
                    s = F(s + t[ls, i])
                S, frm = s, ls + 1
            elif S == 0:
                nz = (t != 0).any(axis=1) | np.isnan(t).any(axis=1)
                nz[:frm] = False
                if not nz.any():
                    break
                ls = int(np.argmax(nz))
                s = S
                for i in range(16):
                    s = F(s + t[ls, i])
                S, frm = s, ls + 1
            elif not np.isfinite(S):
                with np.errstate(over="ignore", invalid="ignore"):
                    S = F(S + t[frm:].sum(dtype=np.float32))
                break
            else:
                s = S
                for i in range(16):
                    s = F(s + t[frm, i])
                S, frm = s, frm + 1
    return S


def serial(terms: np.ndarray) -> np.float32:
    s = F(0)
    with np.errstate(over="ignore", invalid="ignore"):
        for x in terms.astype(np.float32):
            s = F(s + x)
    return s


def same(a, b):
    return (np.isnan(a) and np.isnan(b)) or _bits(a) == _bits(b)


def gaussian_terms(n, rng, sigma=0.02, h=None):
    w = (rng.standard_normal(n) * sigma).astype(np.float16).astype(np.float32)
    x = (w * w).astype(np.float32)
    if h is None:
        return x
    return (x / h).astype(np.float32)


@pytest.mark.parametrize("rows", [128, 256])
def test_random_terms(rows):
    rng = np.random.default_rng(11)
    for trial in range(6):
        n = int(rng.integers(1000, 40000))
        h = np.exp(rng.standard_normal(n) * 1.5).astype(np.float32) if trial % 2 else None
        t = gaussian_terms(n, rng, h=h)
        assert same(emulate(t, rows), serial(t))


def test_exact_ties_are_resolved_serially():
    # S = 1.0 (ulp 2^-23): a term of exactly 2^-24 is a tie whose result
    # depends on the parity of S/ulp.
    rng = np.random.default_rng(2)
    t = np.full(6000, 2.0 ** -24, np.float32)
    t[0] = 1.0
    t[rng.integers(1, 6000, 300)] = 3 * 2.0 ** -24
    t[rng.integers(1, 6000, 300)] = 2.0 ** -20
    assert same(emulate(t, 128), serial(t))


def test_zero_runs_and_binade_crossings():
    t = np.zeros(9000, np.float32)
    t[4000] = 1e-30
    t[4001:] = np.float32(1e-3)
    t[7000] = np.float32(3e4)  # one huge jump
    assert same(emulate(t, 256), serial(t))
    assert same(emulate(np.zeros(5000, np.float32), 128), F(0))


def test_tiny_and_huge_terms():
    rng = np.random.default_rng(4)
    t = np.exp(rng.uniform(-230, 80, 5000)).astype(np.float32)
    assert same(emulate(t, 128), serial(t))
    t2 = np.exp(rng.uniform(-103 * 0.69, -90 * 0.69, 3000)).astype(np.float32)
    assert same(emulate(t2, 128), serial(t2))


def test_nonfinite_terms():
    rng = np.random.default_rng(6)
    t = gaussian_terms(5000, rng)
    t[2500] = np.inf
    assert same(emulate(t, 128), serial(t))
    t[3000] = np.nan
    assert np.isnan(emulate(t, 128)) and np.isnan(serial(t))
    t2 = np.full(4000, 3e38, np.float32)  # overflows to inf part way
    assert same(emulate(t2, 128), serial(t2))


def test_matches_oracle_on_group_layout(oracle):
    # the kernel's serial order is (row, column-in-group); compare through the
    # oracle's sensitivity of a whole matrix
    rng = np.random.default_rng(9)
    M, K = 700, 48
    w = (rng.standard_normal((M, K)) * 0.02).astype(np.float16)
    h = np.exp(rng.standard_normal(K) * 1.5).astype(np.float32)
    h[3] = 1e-10
    s = oracle.sensitivity(w, h)
    for g in range(3):
        blk = w[:, g * 16:(g + 1) * 16].astype(np.float32)
        x = (blk * blk).astype(np.float32)
        hh = h[g * 16:(g + 1) * 16]
        t = np.where(hh > np.float32(1e-8), (x / hh).astype(np.float32), x).reshape(-1)
        assert same(emulate(t.astype(np.float32), 128), s[g])
