"""dequantize_2nd_order on sm_100a (through the C ABI, mb_dequantize_2nd)
against the numpy oracle, bit for bit, on the product's own quantized
fields: with and without the outlier write-back, 16-byte and scalar store
paths, and an output that is not 16-byte aligned."""
import numpy as np
import pytest
import torch

import memboost_b200 as mb
from memboost_b200 import workloads

pytestmark = pytest.mark.gpu

CASES = [(300, 1040, "shifted", 12, 0.1), (17, 100, "normal", 3, 0.25),
         (129, 688, "normal", 13, 0.1), (64, 4104, "tiny", 11, 0.25),
         (8191, 1000, "shifted", 25, 0.3), (2, 16, "normal", 1, 0.0)]


def _fields(qt):
    return {k: (v.cpu().numpy() if isinstance(v, torch.Tensor) else v)
            for k, v in qt.__dict__.items()}


@pytest.mark.parametrize("add", [True, False], ids=["outliers", "no_outliers"])
@pytest.mark.parametrize("M,K,kind,seed,ratio", CASES)
def test_dequantize_2nd_matches_oracle(M, K, kind, seed, ratio, add, oracle):
    mc = workloads.small_case(M, K, seed, kind)
    qt = mb.quantize(mc.weights.cuda(), ratio, mc.hessian_diag.cuda())
    got = mb.dequantize_2nd_order(qt, add_outliers=add)
    torch.cuda.synchronize()
    want = oracle.dequantize_2nd(_fields(qt), add_outliers=add)
    assert np.array_equal(got.cpu().numpy().view(np.uint16), want.view(np.uint16))


def test_dequantize_2nd_unaligned_output(oracle):
    mc = workloads.small_case(129, 688, 13, "normal")
    qt = mb.quantize(mc.weights.cuda(), 0.1, mc.hessian_diag.cuda())
    buf = torch.empty(129 * 688 + 1, dtype=torch.float16, device="cuda")
    out = buf[1:].view(129, 688)  # 2-byte aligned only
    mb.dequantize_2nd_order(qt, out=out)
    torch.cuda.synchronize()
    want = oracle.dequantize_2nd(_fields(qt), add_outliers=True)
    assert np.array_equal(out.cpu().numpy().view(np.uint16), want.view(np.uint16))


def test_zero2_wrap_flag():
    """Clustered scales make the reference's int8 2nd-order zero point wrap;
    the quantize call reports it (FLAG_ZERO2_WRAP), and the outputs still
    equal the oracle's (the format is kept).  Ordinary inputs raise no flag."""
    from memboost_b200 import _C
    from test_dequant_2nd import clustered_scales_case
    from oracle import oracle as O
    w = clustered_scales_case()
    ws = _C.QuantizeWorkspace(*w.shape, torch.device("cuda"))
    out = _C.quantize(torch.from_numpy(w).cuda(), 0.0, None, ws)
    torch.cuda.synchronize()
    assert ws.flags() & _C.FLAG_ZERO2_WRAP
    want = O.quantize(w, 0.0, None)
    assert np.array_equal(out[5].cpu().numpy(), want["zeros_2nd"])
    mc = workloads.small_case(300, 1040, 12, "shifted")
    ws2 = _C.QuantizeWorkspace(300, 1040, torch.device("cuda"))
    _C.quantize(mc.weights.cuda(), 0.1, mc.hessian_diag.cuda(), ws2)
    assert not ws2.flags() & _C.FLAG_ZERO2_WRAP
