"""The exact-sum path checked on every group.  mb_quantize quantizes most
groups' sensitivities only to a rigorous interval and computes the exact
serial fp32 sum (core/quantize.cu:72-98) for the groups straddling the 4-bit
boundary; mb_quantize_exact_sums sends every group through that path.  Each
sum must equal the oracle's serial fp32 sum bit for bit: tall matrices (many
binade crossings per group, long stretches between them), hessians spanning
many decades or below the division cut-off, zero and ragged rows, a partial
last group, exact half-ulp ties, and NaN / inf weights."""
import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu


def _normal(M, K, seed, scale=0.02):
    g = np.random.default_rng(seed)
    return (g.standard_normal((M, K)) * scale).astype(np.float16)


def _lognormal(K, seed, sigma=1.5):
    g = np.random.default_rng(seed + 1000)
    return np.exp(g.standard_normal(K) * sigma).astype(np.float32)


def _cases():
    out = []
    out.append(("tall", _normal(11008, 256, 1), _lognormal(256, 1)))
    out.append(("square_ones", _normal(4096, 4096, 2), np.ones(4096, np.float32)))
    g = np.random.default_rng(3)
    out.append(("decades", _normal(3000, 128, 3),
                np.exp(g.random(128) * 46.0 - 23.0).astype(np.float32)))
    w = _normal(2500, 96, 4)
    w[::7] = 0
    w[:, 32:48] = 0
    h = _lognormal(96, 4)
    h[::5] = 1e-10  # no division for these columns
    out.append(("zeros_cutoff", w, h))
    out.append(("ragged", _normal(3 * 128 + 5, 64, 5), _lognormal(64, 5)))
    out.append(("partial_group", _normal(1000, 40, 6), _lognormal(40, 6)))
    # first row's terms sum to 16; every later term is half an ulp of 16, a
    # tie that rounds to the even neighbour: the sum stays 16
    w = np.full((700, 64), 2.0 ** -10, np.float16)
    w[0] = 1.0
    w[:, 48:] = _normal(700, 16, 7)
    out.append(("half_ulp_ties", w, np.ones(64, np.float32)))
    w = _normal(600, 80, 8)
    w[100, 5] = np.float16(np.inf)
    w[200, 20] = np.float16(np.nan)
    out.append(("nonfinite", w, _lognormal(80, 8)))
    return out


@pytest.mark.parametrize("name,w,h", _cases(), ids=[c[0] for c in _cases()])
def test_exact_sums_equal_serial_fp32(name, w, h, oracle):
    from memboost_b200 import _C
    dev = torch.device("cuda", 0)
    sums, gp = _C.exact_sums(torch.from_numpy(w).to(dev), torch.from_numpy(h).to(dev), 0.5)
    torch.cuda.synchronize(dev)
    got = sums.cpu().numpy()
    want = oracle.sensitivity(w, h)
    assert np.array_equal(np.isnan(got), np.isnan(want)), name
    fin = ~np.isnan(want)
    bad = np.nonzero(got[fin].view(np.uint32) != want[fin].view(np.uint32))[0]
    assert bad.size == 0, (name, bad[:8], got[fin][bad[:8]], want[fin][bad[:8]])
    if name == "half_ulp_ties":
        assert got[0] == 16.0
    if np.isnan(want).any() or name == "half_ulp_ties":
        return  # NaN keys / equal sums: the reference's sort order is open
    assert np.array_equal(gp.cpu().numpy(), oracle.select(want, 0.5)), name
