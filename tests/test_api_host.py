"""Host-side API logic: argument validation (the reference's TORCH_CHECK
messages, core/torch_ops.cu:21-112, 150-151, 275-276) and QuantizedTensor
accounting / serialization (memboost/formats.py).  CPU only."""
import io

import numpy as np
import pytest
import torch


def test_public_surface(mb):
    for n in ("QuantizedTensor", "GROUP_SIZE_1ST", "GROUP_SIZE_2ND", "pack_2bit", "unpack_2bit",
              "pack_4bit", "unpack_4bit", "quantize", "dequantize"):
        assert hasattr(mb, n)
    assert mb.GROUP_SIZE_1ST == 16 and mb.GROUP_SIZE_2ND == 256
    assert mb.__version__ == "0.1.0"


@pytest.mark.parametrize("bad,msg", [
    (torch.zeros(4, 4), "weights must be float16"),
    (torch.zeros(16, dtype=torch.float16), "weights must be 2D"),
    (torch.zeros(4, 16, dtype=torch.float16), "weights must be on CUDA"),
])
def test_quantize_argument_errors(mb, bad, msg):
    with pytest.raises(RuntimeError, match=msg):
        mb.quantize(bad)


def test_pack_argument_errors(mb):
    with pytest.raises(RuntimeError, match="values must be uint8"):
        mb.pack_2bit(torch.zeros(16, dtype=torch.int32))
    with pytest.raises(RuntimeError, match="values must be 1D"):
        mb.pack_4bit(torch.zeros(2, 8, dtype=torch.uint8))
    with pytest.raises(RuntimeError, match="multiple of 8"):
        mb.pack_4bit(torch.zeros(12, dtype=torch.uint8))
    with pytest.raises(RuntimeError, match="packed must be int32"):
        mb.unpack_2bit(torch.zeros(1, dtype=torch.int64), 16)
    with pytest.raises(RuntimeError, match="num_elements too large"):
        mb.unpack_2bit(torch.zeros(1, dtype=torch.int32), 17)
    assert mb.pack_2bit(torch.zeros(0, dtype=torch.uint8)).numel() == 0


def test_dequantize_argument_errors(mb):
    from memboost_b200 import _C
    with pytest.raises(RuntimeError, match="packed_2bit must be on CUDA"):
        _C.dequantize(torch.zeros(4, 1, dtype=torch.int32), None, None, None, None, 4, 16)


def _qt_from_oracle(mb, oracle, M=40, K=100, ratio=0.25, seed=0):
    rng = np.random.default_rng(seed)
    w = (rng.standard_normal((M, K)) * 0.02).astype(np.float16)
    w[:, 16:32] += np.float16(0.3)  # one shifted group -> outliers
    q = oracle.quantize(w, ratio, np.exp(rng.standard_normal(K)).astype(np.float32))
    t = {k: torch.from_numpy(np.ascontiguousarray(v)) for k, v in q.items()
         if isinstance(v, np.ndarray)}
    return mb.QuantizedTensor(**t, M=M, K=K), q


def test_quantized_tensor_accounting(mb, oracle):
    qt, q = _qt_from_oracle(mb, oracle)
    M, K = 40, 100
    ng = 7
    assert qt.num_groups == ng and qt.nnz == q["outlier_values"].size > 0
    n4 = int(q["group_precision"].sum())
    assert qt.num_4bit_groups == n4 == int(0.25 * ng) and qt.num_2bit_groups == ng - n4
    n2e, n4e = (ng - n4) * 16 * M, n4 * 16 * M
    want = (n2e * 2 + n4e * 4 + (n2e + n4e) / 16 * 6 + qt.nnz * 32) / (M * K)
    assert qt.avg_bits == pytest.approx(want)
    other = sum(t.nbytes for t in (qt.scales_1st, qt.zeros_1st, qt.scales_2nd, qt.zeros_2nd,
                                   qt.scales_1st_quant, qt.group_precision, qt.outlier_values,
                                   qt.outlier_col_indices, qt.outlier_row_ptrs))
    assert qt.total_bytes == (ng - n4) * M * 4 + n4 * M * 8 + other
    assert qt.gpu_bytes == qt.packed_2bit.nbytes + qt.packed_4bit.nbytes + other
    mib = qt.memory_breakdown()
    assert set(mib) == {"packed_2bit", "packed_4bit", "scales_1st", "zeros_1st", "scales_2nd",
                        "zeros_2nd", "scales_1st_quant", "group_precision", "outlier_values",
                        "outlier_col_indices", "outlier_row_ptrs"}


def test_state_dict_roundtrip_through_torch_save(mb, oracle):
    qt, _ = _qt_from_oracle(mb, oracle, seed=3)
    sd = qt.state_dict()
    assert sorted(sd) == sorted(["packed_2bit", "packed_4bit", "scales_1st", "zeros_1st",
                                 "scales_2nd", "zeros_2nd", "scales_1st_quant", "group_precision",
                                 "outlier_values", "outlier_col_indices", "outlier_row_ptrs",
                                 "M", "K"])
    assert sd["M"].dim() == 0 and int(sd["K"]) == 100
    buf = io.BytesIO()
    torch.save(sd, buf)
    buf.seek(0)
    qt2 = mb.QuantizedTensor.from_state_dict(torch.load(buf))
    for f in ("packed_2bit", "packed_4bit", "scales_1st", "outlier_row_ptrs"):
        assert torch.equal(getattr(qt, f), getattr(qt2, f))
    assert (qt2.M, qt2.K) == (qt.M, qt.K)
    assert qt2.to("cpu").device.type == "cpu"
