"""qgemv on sm_100a (through the C ABI, mb_qgemv) against the oracle: W from
the product's own quantized fields decoded by the oracle (the reference
dequantize, outliers written back or not), y = W x in fp64.  The kernel sums
in fp32, so the tolerance is the rigorous summation bound
(per-lane chain + 5 reduction steps + 2 per outlier) * 2^-24 * sum |w x|
(taken over both W with and without its outliers)."""
import numpy as np
import pytest
import torch

import memboost_b200 as mb
from memboost_b200 import workloads

pytestmark = pytest.mark.gpu

CASES = [(300, 1040, "shifted", 12, 0.1), (129, 688, "normal", 13, 0.1),
         (64, 4104, "tiny", 11, 0.25), (8191, 1000, "shifted", 25, 0.3),
         (5, 33, "shifted", 15, 0.5)]


def _fields(qt):
    return {k: (v.cpu().numpy() if isinstance(v, torch.Tensor) else v)
            for k, v in qt.__dict__.items()}


def _check(y, q, x, add, oracle):
    M, K = q["M"], q["K"]
    w_out = oracle.decode_with_scales(q, q["scales_1st"], add_outliers=True).astype(np.float64)
    w_plain = oracle.decode_with_scales(q, q["scales_1st"], add_outliers=False).astype(np.float64)
    w = w_out if add else w_plain
    xd = x.astype(np.float64)
    want = w @ xd
    ng = (K + 15) // 16
    nnz_row = np.diff(q["outlier_row_ptrs"]) if add else np.zeros(M, np.int64)
    chain = 16 * ((ng + 31) // 32) + 5 + 2 * nnz_row
    bound = (chain + 10) * 2.0 ** -24 * ((np.abs(w_out) + np.abs(w_plain)) @ np.abs(xd)) + 1e-30
    err = np.abs(y.astype(np.float64) - want)
    assert np.all(err <= bound), (err - bound).max()


@pytest.mark.parametrize("add", [True, False], ids=["outliers", "codes_only"])
@pytest.mark.parametrize("M,K,kind,seed,ratio", CASES)
def test_qgemv_matches_oracle(M, K, kind, seed, ratio, add, oracle):
    mc = workloads.small_case(M, K, seed, kind)
    qt = mb.quantize(mc.weights.cuda(), ratio, mc.hessian_diag.cuda())
    g = torch.Generator().manual_seed(seed)
    x = torch.randn(K, generator=g).half()
    y = mb.qgemv(qt, x.cuda(), add_outliers=add)
    torch.cuda.synchronize()
    _check(y.cpu().numpy(), _fields(qt), x.numpy(), add, oracle)


def test_qgemv_unaligned_x(oracle):
    mc = workloads.small_case(300, 1040, 12, "shifted")
    qt = mb.quantize(mc.weights.cuda(), 0.1, mc.hessian_diag.cuda())
    x = torch.randn(1040, generator=torch.Generator().manual_seed(1)).half()
    buf = torch.empty(1041, dtype=torch.float16, device="cuda")
    buf[1:] = x.cuda()
    y = mb.qgemv(qt, buf[1:])  # 2-byte aligned: the scalar path throughout
    torch.cuda.synchronize()
    _check(y.cpu().numpy(), _fields(qt), x.numpy(), True, oracle)
