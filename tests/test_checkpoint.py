"""On-disk format (CPU): state_dict keeps the reference's keys; the compact
layout stores only each group's own packed words and restores the arrays
exactly; save_quantized / load_quantized round-trip both layouts and read
a file laid out as the reference's driver writes it (models/llama.py:686-693)."""
import numpy as np
import pytest
import torch

from memboost_b200 import QuantizedTensor, load_quantized, save_quantized, workloads
from memboost_b200.formats import _TENSOR_FIELDS
from oracle import oracle as O

CASES = [(300, 1040, "shifted", 12, 0.1), (129, 688, "normal", 13, 0.5), (17, 100, "normal", 3, 0.0),
         (33, 48, "const", 9, 1.0)]
REF_KEYS = {"packed_2bit", "packed_4bit", "scales_1st", "zeros_1st", "scales_2nd", "zeros_2nd",
            "scales_1st_quant", "group_precision", "outlier_values", "outlier_col_indices",
            "outlier_row_ptrs", "M", "K"}


def _qt(M, K, kind, seed, ratio):
    mc = workloads.small_case(M, K, seed, kind)
    q = O.quantize(mc.weights.numpy(), ratio, mc.hessian_diag.numpy().astype(np.float32))
    ng = O.num_groups(K)
    shapes = {"packed_2bit": (M, ng), "packed_4bit": (M, 2 * ng), "scales_1st": (M, ng),
              "zeros_1st": (M, ng), "scales_1st_quant": (M, ng)}
    f = {}
    for k in _TENSOR_FIELDS:
        a = np.ascontiguousarray(q[k])
        if k in shapes:
            a = a.reshape(shapes[k])
        f[k] = torch.from_numpy(a.copy())
    return QuantizedTensor(**f, M=M, K=K)


def _same(a: QuantizedTensor, b: QuantizedTensor):
    assert (a.M, a.K) == (b.M, b.K)
    for k in _TENSOR_FIELDS:
        x, y = getattr(a, k), getattr(b, k)
        assert x.dtype == y.dtype, k
        assert torch.equal(x.reshape(-1), y.reshape(-1)), k


@pytest.mark.parametrize("case", CASES)
def test_compact_round_trip(case):
    qt = _qt(*case)
    d = qt.compact_state_dict()
    assert set(d) == REF_KEYS | {"packed_layout"}
    assert d["packed_2bit"].nbytes + d["packed_4bit"].nbytes == sum(qt._used_packed_bytes())
    assert qt.total_bytes == sum(v.nbytes for k, v in d.items()
                                 if k not in ("M", "K", "packed_layout"))
    _same(QuantizedTensor.from_state_dict(d), qt)


@pytest.mark.parametrize("compact", [False, True])
def test_save_load_round_trip(tmp_path, compact):
    layers = {f"layer{i}.mlp": _qt(*c) for i, c in enumerate(CASES)}
    path = tmp_path / "q.pt"
    save_quantized(layers, path, compact=compact, stats={"bytes": 1}, _model_name="synthetic")
    got, meta = load_quantized(path)
    assert meta == {"_stats": {"bytes": 1}, "_model_name": "synthetic"}
    assert set(got) == set(layers)
    for k in layers:
        _same(got[k], layers[k])


def test_reads_the_reference_driver_layout(tmp_path):
    qt = _qt(*CASES[0])
    d = {"model.layers.0.mlp.up_proj": qt.state_dict(), "_stats": {}, "_ratio_4bit": 0.1}
    assert set(d["model.layers.0.mlp.up_proj"]) == REF_KEYS
    torch.save(d, tmp_path / "ref.pt")
    got, meta = load_quantized(tmp_path / "ref.pt")
    _same(got["model.layers.0.mlp.up_proj"], qt)
    assert meta["_ratio_4bit"] == 0.1


def test_layer_names_must_not_look_like_metadata(tmp_path):
    with pytest.raises(ValueError):
        save_quantized({"_x": _qt(*CASES[2])}, tmp_path / "x.pt")
