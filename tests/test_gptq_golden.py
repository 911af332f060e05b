"""GPTQ oracles and host logic against fixtures made by the reference's own
models/llama.py on CPU tensors (tests/golden/make_gptq_golden.py).  CPU only."""
import glob
import os

import numpy as np
import pytest
import torch

from cases import gptq_division_probe
from oracle import gptq_torch

GOLDEN = sorted(glob.glob(os.path.join(os.path.dirname(__file__), "golden", "gptq_*.npz")))
IDS = [os.path.basename(p)[:-4] for p in GOLDEN]


def test_fixtures_present():
    assert len(GOLDEN) >= 7, "GPTQ fixtures missing (tests/golden/make_gptq_golden.py)"


@pytest.mark.parametrize("path", GOLDEN, ids=IDS)
def test_c_oracle_matches_reference(path, oracle):
    g = np.load(path)
    Q = oracle.gptq_quantize(g["W"], g["hinv_cho"], g["group_precision"],
                             div_mode=oracle.GPTQ_DIV_TRUE)
    assert gptq_torch.equal_up_to_zero_sign(torch.from_numpy(Q), torch.from_numpy(g["Q"]))


@pytest.mark.parametrize("path", GOLDEN, ids=IDS)
def test_torch_oracle_matches_reference(path):
    g = np.load(path)
    Q = gptq_torch.gptq_quantize(torch.from_numpy(g["W"]), torch.from_numpy(g["hinv_cho"]),
                                 torch.from_numpy(g["group_precision"]))
    assert gptq_torch.equal_up_to_zero_sign(Q, torch.from_numpy(g["Q"]))


@pytest.mark.parametrize("path", GOLDEN, ids=IDS)
def test_host_inverse_and_precision(path):
    """gptq_inverse / compute_group_precision of memboost_b200.gptq are torch
    host code: on the same CPU tensors they reproduce the reference."""
    from memboost_b200 import gptq
    g = np.load(path)
    H = torch.from_numpy(g["H"].copy())
    h_diag, hinv_cho = gptq.gptq_inverse(H)
    # LAPACK results can differ in the last bits between CPU builds
    assert torch.allclose(h_diag, torch.from_numpy(g["h_diag"]), rtol=1e-5, atol=0)
    assert torch.allclose(hinv_cho, torch.from_numpy(g["hinv_cho"]), rtol=1e-4, atol=1e-7)
    if bool(g["gp_from_sensitivity"]):
        gp = gptq.compute_group_precision(torch.from_numpy(g["W"]),
                                          torch.from_numpy(g["h_diag"]), float(g["ratio_4bit"]))
        assert torch.equal(gp, torch.from_numpy(g["group_precision"]))


def _forced_reference_loop(gp: torch.Tensor, K: int) -> torch.Tensor:
    """llama.py:356-364, one group at a time."""
    h = torch.ones(K, dtype=torch.float32)
    for g in range(K // 16):
        h[g * 16:g * 16 + 16] = 1e-10 if gp[g] == 1 else 1e10
    return h


@pytest.mark.parametrize("K", [16, 48, 200, 4096])
def test_forced_hessian_diag(K):
    from memboost_b200 import gptq
    gp = (torch.arange(K // 16) % 3 == 0).to(torch.uint8)
    got = gptq.forced_hessian_diag(gp, K)
    assert torch.equal(got, _forced_reference_loop(gp, K))


def test_division_modes_differ_on_probe(oracle):
    """The CUDA-tensor semantics (multiply by the reciprocal) is a different
    function from the CPU one; the probe matrix separates them."""
    W, Hc, gp = gptq_division_probe()
    a = oracle.gptq_quantize(W, Hc, gp, div_mode=oracle.GPTQ_DIV_TRUE)
    b = oracle.gptq_quantize(W, Hc, gp, div_mode=oracle.GPTQ_DIV_RECIPROCAL)
    assert (a != b).sum() >= W.shape[0] * W.shape[1] // 4
    t = gptq_torch.gptq_quantize(torch.from_numpy(W), torch.from_numpy(Hc), torch.from_numpy(gp))
    assert gptq_torch.equal_up_to_zero_sign(t, torch.from_numpy(a))  # CPU torch = IEEE quotient


def test_oracle_thread_count_invariant(oracle):
    g = np.load(GOLDEN[0])
    a = oracle.gptq_quantize(g["W"], g["hinv_cho"], g["group_precision"], nthreads=1)
    b = oracle.gptq_quantize(g["W"], g["hinv_cho"], g["group_precision"], nthreads=7)
    assert np.array_equal(a.view(np.uint32), b.view(np.uint32))
