"""The reference's own Python tests (tests/test_ops.py, tests/test_gemm.py),
restated as pytest functions against memboost_b200."""
import io

import pytest
import torch

pytestmark = pytest.mark.gpu


def test_ops_smoke(mb):
    # tests/test_ops.py:8-40
    v = torch.tensor([0, 1, 2, 3] * 4, dtype=torch.uint8)
    assert torch.equal(mb.unpack_2bit(mb.pack_2bit(v), 16), v)
    v4 = torch.tensor([0, 3, 7, 15, 1, 8, 12, 4], dtype=torch.uint8)
    assert torch.equal(mb.unpack_4bit(mb.pack_4bit(v4), 8), v4)
    torch.manual_seed(0)
    w = torch.randn(64, 64, dtype=torch.float16, device="cuda")
    qt = mb.quantize(w, ratio_4bit=0.0)
    w_hat = mb.dequantize(qt)
    assert w_hat.shape == w.shape
    qt2 = mb.quantize(w, ratio_4bit=0.2)  # no hessian: stays all 2-bit
    assert qt2.num_4bit_groups == 0
    qt3 = mb.QuantizedTensor.from_state_dict(qt.state_dict())
    assert torch.equal(w_hat, mb.dequantize(qt3))


def test_gemm_roundtrip(mb):
    # tests/test_gemm.py:8-62
    torch.manual_seed(1)
    W = torch.randn(256, 256, dtype=torch.float16, device="cuda")
    qt = mb.quantize(W, ratio_4bit=0.0)
    Wd = mb.dequantize(qt)
    rel = (W.float() - Wd.float()).abs().mean().item() / W.float().abs().mean().item()
    assert rel < 2.0
    assert 1.5 < qt.avg_bits < 3.0
    assert Wd.shape == W.shape and Wd.dtype == torch.float16
    W2 = torch.randn(100, 80, dtype=torch.float16, device="cuda")
    assert mb.dequantize(mb.quantize(W2, ratio_4bit=0.0)).shape == (100, 80)
    W3 = torch.randn(4096, 4096, dtype=torch.float16, device="cuda")
    qt3 = mb.quantize(W3, ratio_4bit=0.0)
    assert W3.numel() * 2 / qt3.total_bytes > 3.0
    assert 1.5 < qt3.avg_bits < 3.0
    buf = io.BytesIO()
    torch.save(qt.state_dict(), buf)
    buf.seek(0)
    qt_l = mb.QuantizedTensor.from_state_dict(torch.load(buf))
    assert torch.equal(Wd, mb.dequantize(qt_l))


def test_hessian_selects_sensitive_groups(mb):
    torch.manual_seed(2)
    W = torch.randn(512, 1024, dtype=torch.float16, device="cuda") * 0.02
    h = torch.ones(1024, device="cuda")
    h[:64] = 1e-3  # groups 0-3 most sensitive (w^2 / h)
    qt = mb.quantize(W, ratio_4bit=4 / 64, hessian_diag=h)
    assert qt.group_precision[:4].tolist() == [1, 1, 1, 1] and qt.num_4bit_groups == 4
    assert qt.packed_2bit[:, :4].abs().sum() == 0 and qt.packed_4bit[:, 8:].abs().sum() == 0


def test_errors_on_gpu(mb):
    w = torch.randn(8, 32, dtype=torch.float16, device="cuda")
    with pytest.raises(RuntimeError, match="hessian_diag must be float32"):
        mb.quantize(w, 0.1, torch.ones(32, dtype=torch.float64, device="cuda"))
    with pytest.raises(RuntimeError, match="hessian_diag must be on CUDA"):
        mb.quantize(w, 0.1, torch.ones(32))
    with pytest.raises(RuntimeError, match="at least K"):
        mb.quantize(w, 0.1, torch.ones(16, device="cuda"))
    # ignored when the selection does not run (as in the reference)
    mb.quantize(w, 0.0, torch.ones(32, dtype=torch.float64))
    with pytest.raises(RuntimeError, match="non-empty"):
        mb.quantize(torch.zeros(0, 16, dtype=torch.float16, device="cuda"))
