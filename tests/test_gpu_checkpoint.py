"""The compact checkpoint layout on the product's own CUDA outputs: the
packed words it omits are zero as quantize writes them, so the round trip
is exact; save / load keeps the tensors on the requested device."""
import pytest
import torch

import memboost_b200 as mb
from memboost_b200 import QuantizedTensor, workloads
from memboost_b200.formats import _TENSOR_FIELDS

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("M,K,kind,seed,ratio", [(300, 1040, "shifted", 12, 0.1),
                                                 (1000, 4096, "normal", 3, 0.25)])
def test_compact_round_trip_on_device(M, K, kind, seed, ratio, tmp_path):
    mc = workloads.small_case(M, K, seed, kind)
    qt = mb.quantize(mc.weights.cuda(), ratio, mc.hessian_diag.cuda())
    back = QuantizedTensor.from_state_dict(qt.compact_state_dict())
    for k in _TENSOR_FIELDS:
        assert torch.equal(getattr(back, k), getattr(qt, k)), k
    mb.save_quantized({"w": qt}, tmp_path / "q.pt", compact=True)
    got, _ = mb.load_quantized(tmp_path / "q.pt", map_location="cuda")
    for k in _TENSOR_FIELDS:
        assert getattr(got["w"], k).is_cuda
        assert torch.equal(getattr(got["w"], k), getattr(qt, k)), k
