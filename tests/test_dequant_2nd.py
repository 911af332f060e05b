"""The dequantize that rebuilds each group's scale from the compact 2nd-order
fields (no counterpart in the reference) -- oracle side, on CPU: its decode
is the reference dequantize when given scales_1st, its rebuilt scales lie
within one 2nd-order step of scales_1st, and the CSR outliers come back
exactly."""
import numpy as np
import pytest

from memboost_b200 import workloads
from oracle import oracle as O

CASES = [(300, 1040, "shifted", 12, 0.1), (17, 100, "normal", 3, 0.25),
         (129, 688, "normal", 13, 0.1), (64, 4104, "tiny", 11, 0.25), (33, 48, "const", 9, 0.25)]


def _q(M, K, kind, seed, ratio):
    mc = workloads.small_case(M, K, seed, kind)
    w = mc.weights.numpy()
    return w, O.quantize(w, ratio, mc.hessian_diag.numpy().astype(np.float32))


@pytest.mark.parametrize("M,K,kind,seed,ratio", CASES)
def test_decode_with_scales_1st_is_reference_dequantize(M, K, kind, seed, ratio):
    _, q = _q(M, K, kind, seed, ratio)
    a = O.decode_with_scales(q, q["scales_1st"])
    assert np.array_equal(a.view(np.uint16), O.dequantize(q).view(np.uint16))


@pytest.mark.parametrize("M,K,kind,seed,ratio", CASES)
def test_rebuilt_scales_within_one_step(M, K, kind, seed, ratio):
    _, q = _q(M, K, kind, seed, ratio)
    ng = O.num_groups(K)
    s_hat = O.rebuilt_scales(q).astype(np.float64).reshape(-1)
    s1 = q["scales_1st"].astype(np.float64).reshape(-1)
    step = q["scales_2nd"].astype(np.float64)[np.arange(M * ng) // O.GROUP_SIZE_2ND]
    # code and zero point each round by at most half a step; the fp16
    # results (s_hat, and scales_2nd itself) round by at most 2^-11 relative
    tol = step * 1.002 + (np.abs(s_hat) + np.abs(s1)) * 2.0 ** -10 + 1e-7
    assert np.all(np.abs(s_hat - s1) <= tol)


@pytest.mark.parametrize("M,K,kind,seed,ratio", CASES[:2])
def test_outliers_written_back(M, K, kind, seed, ratio):
    w, q = _q(M, K, kind, seed, ratio)
    out = O.dequantize_2nd(q, add_outliers=True)
    rows = np.repeat(np.arange(M), np.diff(q["outlier_row_ptrs"]))
    cols = q["outlier_col_indices"]
    assert np.array_equal(out[rows, cols].view(np.uint16), w[rows, cols].view(np.uint16))
    plain = O.dequantize_2nd(q, add_outliers=False)
    mask = np.ones((M, K), bool)
    mask[rows, cols] = False
    assert np.array_equal(out[mask].view(np.uint16), plain[mask].view(np.uint16))


def clustered_scales_case(M=16, K=256, seed=0):
    """Every group spans about the same +-0.1 range, so the 256 scales of a
    2nd-order chunk lie within a few percent of each other and
    round(-min / scale_2nd) falls far below -128."""
    rng = np.random.default_rng(seed)
    w = rng.uniform(-0.09, 0.09, size=(M, K)).astype(np.float32)
    ng = K // 16
    spread = rng.uniform(0.1, 0.104, size=ng)
    for g in range(ng):
        w[0, 16 * g] = -spread[g]
        w[1, 16 * g + 1] = spread[g]
    return w.astype(np.float16)


def test_zero2_wraps_for_clustered_scales():
    """The reference casts round(-min / scale_2nd) to int8 with wrap-around
    (core/quantize.cu:267-272); with tightly clustered scales the true zero
    point lies far outside [-128, 127], the stored one wraps, and scales
    rebuilt from the 2nd-order codes are badly wrong.  The oracle keeps the
    reference's cast (it is the format); the GPU path reports the chunk
    through FLAG_ZERO2_WRAP (tests/test_gpu_dequant_2nd.py)."""
    w = clustered_scales_case()
    q = O.quantize(w, 0.0, None)
    s1 = q["scales_1st"].astype(np.float32).reshape(-1)
    mn, mx = s1.min(), s1.max()
    assert mx / mn < 1.12
    sc2 = np.float32(max(np.float32(mx - mn) / np.float32(15.0), np.float32(1e-10)))
    true_zero = int(np.round(np.float64(-mn) / np.float64(sc2)))
    assert true_zero < -128
    stored = int(np.asarray(q["zeros_2nd"]).reshape(-1)[0])
    assert stored == ((true_zero + 128) % 256) - 128   # the int8 wrap
    s_hat = O.rebuilt_scales(q).astype(np.float32).reshape(-1)
    assert np.max(np.abs(s_hat - s1) / s1) > 0.5       # the format's limit: far off
