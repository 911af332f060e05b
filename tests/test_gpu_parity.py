"""Parity of the sm_100a kernels (through the C ABI, via memboost_b200._C)
against the CPU oracle and against the reference's own compiled kernels
(oracle/_ref), bit for bit on every output."""
import numpy as np
import pytest
import torch

from cases import OUTPUT_FIELDS, diff_fields, reference_defined, small_cases

pytestmark = pytest.mark.gpu

CASES = small_cases()
IDS = [c[0] for c in CASES]


def to_dict(tensors, M, K):
    d = {f: t.cpu().numpy() for f, t in zip(OUTPUT_FIELDS, tensors)}
    d["M"], d["K"] = M, K
    return d


def run_product(w, ratio, h):
    from memboost_b200 import _C
    wt = torch.from_numpy(w).cuda()
    ht = None if h is None else torch.from_numpy(h).cuda()
    return to_dict(_C.quantize(wt, ratio, ht), *w.shape)


def run_reference(ref, w, ratio, h):
    wt = torch.from_numpy(w).cuda()
    ht = torch.Tensor() if h is None else torch.from_numpy(h).cuda()
    out = ref.quantize(wt, ratio, ht)
    torch.cuda.synchronize()
    return to_dict(out, *w.shape)


@pytest.mark.parametrize("case", CASES, ids=IDS)
def test_quantize_matches_oracle(case, oracle):
    name, w, ratio, h = case
    got = run_product(w, ratio, h)
    want = oracle.quantize(w, ratio, h)
    assert diff_fields(got, want) == []


@pytest.mark.parametrize("case", CASES, ids=IDS)
def test_quantize_matches_reference_kernels(case, ref_module):
    name, w, ratio, h = case
    if not reference_defined(w, ratio, h):
        pytest.skip("reference behaviour undefined for ratio * ng > ng")
    got = run_product(w, ratio, h)
    want = run_reference(ref_module, w, ratio, h)
    assert diff_fields(got, want) == []


@pytest.mark.parametrize("case", CASES, ids=IDS)
def test_oracle_pinned_to_reference_kernels(case, ref_module, oracle):
    name, w, ratio, h = case
    if not reference_defined(w, ratio, h):
        pytest.skip("reference behaviour undefined for ratio * ng > ng")
    want = run_reference(ref_module, w, ratio, h)
    assert diff_fields(oracle.quantize(w, ratio, h), want) == []


def test_outlier_arithmetic_is_fused(ref_module, oracle):
    """The reference kernel's outlier test (quantize.cu:192-194) evaluates
    w - scale*(q-zero) with the product fused into the subtraction; the
    probe separates the two candidate evaluations."""
    from cases import fma_probe
    w = fma_probe(0)
    want = run_reference(ref_module, w, 0.0, None)
    fused = oracle.quantize(w, 0.0, None, fma_mode=1)
    rounded = oracle.quantize(w, 0.0, None, fma_mode=0)
    assert diff_fields(fused, rounded) != []
    assert diff_fields(fused, want) == [], "reference kernel is not the fused form"


@pytest.mark.parametrize("case", CASES, ids=IDS)
def test_dequantize_matches_oracle_and_reference(case, oracle, ref_module):
    from memboost_b200 import _C
    name, w, ratio, h = case
    q = oracle.quantize(w, ratio, h)
    args = [torch.from_numpy(np.ascontiguousarray(q[f])).cuda()
            for f in ("packed_2bit", "packed_4bit", "scales_1st", "zeros_1st", "group_precision")]
    M, K = w.shape
    got = _C.dequantize(*args, M, K).cpu().numpy()
    want = oracle.dequantize(q)
    assert np.array_equal(got.view(np.uint16), want.view(np.uint16))
    ref = ref_module.dequantize(*args, M, K).cpu().numpy()
    assert np.array_equal(got.view(np.uint16), ref.view(np.uint16))


def test_pack_unpack_match_reference(ref_module, mb):
    rng = np.random.default_rng(0)
    for n in (16, 160, 4096 * 16 + 16):
        v = torch.from_numpy(rng.integers(0, 256, n, dtype=np.uint8))
        assert torch.equal(mb.pack_2bit(v), ref_module.pack_2bit(v))
        assert torch.equal(mb.pack_4bit(v), ref_module.pack_4bit(v))
        p = mb.pack_2bit(v)
        for k in (n, n - 5, 1):
            assert torch.equal(mb.unpack_2bit(p, k), ref_module.unpack_2bit(p, k))
        p4 = mb.pack_4bit(v)
        assert torch.equal(mb.unpack_4bit(p4, n - 3), ref_module.unpack_4bit(p4, n - 3))
        # CUDA inputs: same results, CPU outputs (as the reference)
        out = mb.pack_2bit(v.cuda())
        assert out.device.type == "cpu" and torch.equal(out, ref_module.pack_2bit(v))


def test_selection_tie_flag(mb):
    """Equal sensitivities across the 4-bit boundary are reported."""
    from memboost_b200 import _C
    w = torch.zeros(64, 32 * 16, dtype=torch.float16)
    w[:, :] = torch.randn(64, 16).half().repeat(1, 32)
    ws = _C.QuantizeWorkspace(64, 512, torch.device("cuda"))
    t = _C.quantize(w.cuda(), 0.1, torch.ones(512, device="cuda"), ws)
    assert int(t[7].sum()) == 3 and t[7][:3].tolist() == [1, 1, 1]
    assert ws.flags() & _C.FLAG_SELECTION_TIE
    w2 = torch.randn(64, 512).half().cuda()
    _C.quantize(w2, 0.1, torch.ones(512, device="cuda"), ws)
    assert ws.flags() == 0
