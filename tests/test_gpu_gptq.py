"""GPTQ kernels on the GPU: the tcgen05 Hessian against an fp64 product
within an fp32-accumulation tolerance, and the blockwise GPTQ update bit for
bit against the reference's own results (fixtures), the CPU oracle and the
torch restatement run on CUDA tensors."""
import glob
import os

import numpy as np
import pytest
import torch

from cases import gptq_division_probe
from oracle import gptq_torch

pytestmark = pytest.mark.gpu

GOLDEN = sorted(glob.glob(os.path.join(os.path.dirname(__file__), "golden", "gptq_*.npz")))
IDS = [os.path.basename(p)[:-4] for p in GOLDEN]


@pytest.fixture(scope="module")
def gq():
    from memboost_b200 import gptq
    return gptq


# ---------------------------------------------------------------------------
# Hessian
# ---------------------------------------------------------------------------

def _hessian_bound(x: torch.Tensor, alpha: float = 1.0):
    """(fp64 alpha * x^T x, error bound).  Products of 16-bit values are exact
    in fp32; the tensor cores add them in fp32 in steps of 16 tokens, so the
    error of each entry stays below (steps + 16) * 2^-22 * alpha * (|x|^T |x|)
    plus the final scaling's rounding."""
    xd = x.double()
    exact = alpha * (xd.T @ xd)
    gabs = abs(alpha) * (xd.abs().T @ xd.abs())
    steps = (x.shape[0] + 15) // 16
    return exact, (steps + 16) * 2.0 ** -22 * gabs + 1e-30


@pytest.mark.parametrize("N,K,dtype", [
    (1024, 256, torch.float16), (4096, 512, torch.bfloat16), (333, 136, torch.float16),
    (64, 8, torch.float16), (5000, 1040, torch.bfloat16), (31, 264, torch.bfloat16),
    (2048, 768, torch.float16),
])
def test_hessian_matches_fp64(gq, N, K, dtype):
    from memboost_b200 import workloads
    x = workloads.calibration_activations(N, K, seed=N + K, dtype=dtype).cuda()
    status = torch.zeros(1, dtype=torch.int32, device="cuda")
    H = gq.hessian(x, status=status)
    torch.cuda.synchronize()
    assert int(status.item()) == 0
    exact, bound = _hessian_bound(x)
    err = (H.double() - exact).abs()
    assert bool((err <= bound).all()), float((err / bound).max())
    # off-diagonal 256-tiles are written mirrored: those entries are exactly symmetric
    tiles = torch.arange(K, device="cuda") // 256
    off = tiles.unsqueeze(0) != tiles.unsqueeze(1)
    assert torch.equal(H[off], H.T[off])


def test_hessian_alpha_and_accumulate(gq):
    from memboost_b200 import workloads
    x1 = workloads.calibration_activations(700, 384, seed=1, dtype=torch.float16).cuda()
    x2 = workloads.calibration_activations(900, 384, seed=2, dtype=torch.float16).cuda()
    H = gq.hessian(x1, alpha=0.5)
    gq.hessian(x2, alpha=0.5, out=H, accumulate=True)
    e1, b1 = _hessian_bound(x1, 0.5)
    e2, b2 = _hessian_bound(x2, 0.5)
    err = (H.double() - (e1 + e2)).abs()
    assert bool((err <= b1 + b2 + 2.0 ** -23 * (e1 + e2).abs()).all())


def test_hessian_accumulator_matches_reference_hook(gq):
    """The reference's hook: per-sample H += x^T x in fp32 (cuBLAS), then
    H /= tokens (llama.py:523-528, 547-551); compared within tolerance."""
    from memboost_b200 import workloads
    acc = gq.HessianAccumulator(512, "cuda")
    H_ref = torch.zeros(512, 512, device="cuda")
    prev = torch.backends.cuda.matmul.allow_tf32
    torch.backends.cuda.matmul.allow_tf32 = False
    try:
        for s in range(4):
            x = workloads.calibration_activations(128, 512, seed=40 + s,
                                                  dtype=torch.float16).cuda().view(1, 128, 512)
            acc.add(x)
            xf = x.float().view(-1, 512)
            H_ref.add_(xf.T @ xf)
    finally:
        torch.backends.cuda.matmul.allow_tf32 = prev
    H_ref.div_(512)
    H = acc.finalize()
    assert acc.tokens == 512
    rel = ((H - H_ref).abs().max() / H_ref.abs().max()).item()
    assert rel < 1e-5, rel


def test_hessian_config_shape(gq):
    """Config-4 geometry (K = 4096 features, bf16 activations) on 16384 tokens,
    against fp64 within the fp32 tensor-core accumulation bound.  (The tensor
    cores' fp32 sums round toward zero, so the deviation from a cuBLAS fp32
    GEMM grows with the token count: ~7.5e-5 of max|H| here.)"""
    from memboost_b200 import workloads
    x = workloads.calibration_activations(16384, 4096, seed=9, device="cuda")
    H = gq.hessian(x, alpha=1.0 / 16384)
    exact, bound = _hessian_bound(x, 1.0 / 16384)
    err = (H.double() - exact).abs()
    assert bool((err <= bound + 2.0 ** -23 * exact.abs()).all()), float((err / bound).max())
    assert float(err.max() / exact.abs().max()) < 2.5e-4


def test_hessian_config4_length(gq):
    """The full config-4 calibration length in one launch: 128 x 2048 =
    262144 tokens x 4096 features, bf16 (8192 pipeline stages per CTA),
    against fp64 within the fp32 tensor-core accumulation bound, by column
    blocks of H."""
    from memboost_b200 import workloads
    N, K = 262144, 4096
    x = workloads.calibration_activations(N, K, seed=17, device="cuda")
    status = torch.zeros(1, dtype=torch.int32, device="cuda")
    H = gq.hessian(x, alpha=1.0 / N, status=status)
    torch.cuda.synchronize()
    assert int(status.item()) == 0
    xd = x.double()
    worst, rel = 0.0, 0.0
    for c0 in range(0, K, 1024):
        blk = xd[:, c0:c0 + 1024]
        exact = (blk.T @ xd) / N
        gabs = (blk.abs().T @ xd.abs()) / N
        bound = (N // 16 + 16) * 2.0 ** -22 * gabs + 2.0 ** -23 * exact.abs() + 1e-30
        err = (H[c0:c0 + 1024].double() - exact).abs()
        worst = max(worst, float((err / bound).max()))
        rel = max(rel, float(err.max() / exact.abs().max()))
        del exact, gabs, bound, err
    assert worst <= 1.0, worst
    print(f"hessian 262144x4096: max |H - fp64| / max|H| = {rel:.3e}, "
          f"max err / bound = {worst:.3f}")


def test_hessian_rejects_bad_arguments(gq):
    x = torch.zeros(16, 12, dtype=torch.float16, device="cuda")
    with pytest.raises(RuntimeError, match="multiple of 8"):
        gq.hessian(x)
    with pytest.raises(RuntimeError, match="float16 or bfloat16"):
        gq.hessian(torch.zeros(16, 16, device="cuda"))


# ---------------------------------------------------------------------------
# GPTQ blockwise update
# ---------------------------------------------------------------------------

@pytest.mark.parametrize("path", GOLDEN, ids=IDS)
def test_gptq_true_division_matches_reference_cpu_run(gq, path):
    g = np.load(path)
    W = torch.from_numpy(g["W"]).cuda()
    Q = gq.gptq_quantize(W, torch.from_numpy(g["hinv_cho"]).cuda(),
                         torch.from_numpy(g["group_precision"]).cuda(),
                         scalar_division=gq.GPTQ_DIV_TRUE)
    assert gptq_torch.equal_up_to_zero_sign(Q, torch.from_numpy(g["Q"]))


@pytest.mark.parametrize("path", GOLDEN, ids=IDS)
def test_gptq_default_matches_reference_on_cuda(gq, path):
    """Default mode = the reference's column loop run on CUDA tensors."""
    g = np.load(path)
    W = torch.from_numpy(g["W"]).cuda()
    Hc = torch.from_numpy(g["hinv_cho"]).cuda()
    gp = torch.from_numpy(g["group_precision"]).cuda()
    want = gptq_torch.gptq_quantize(W, Hc, gp)
    assert gptq_torch.equal_up_to_zero_sign(gq.gptq_quantize(W, Hc, gp), want)


def test_gptq_division_probe_both_modes(gq, oracle):
    """On the probe the two modes differ in many codes; each matches its
    oracle, and torch on CUDA tensors is the reciprocal mode."""
    W, Hc, gp = gptq_division_probe(M=16, ng=24, seed=5)
    Wt, Ht, gt = (torch.from_numpy(a).cuda() for a in (W, Hc, gp))
    true_q = gq.gptq_quantize(Wt, Ht, gt, scalar_division=gq.GPTQ_DIV_TRUE)
    recip_q = gq.gptq_quantize(Wt, Ht, gt, scalar_division=gq.GPTQ_DIV_RECIPROCAL)
    o_true = torch.from_numpy(oracle.gptq_quantize(W, Hc, gp, div_mode=oracle.GPTQ_DIV_TRUE))
    o_recip = torch.from_numpy(oracle.gptq_quantize(W, Hc, gp,
                                                    div_mode=oracle.GPTQ_DIV_RECIPROCAL))
    assert gptq_torch.equal_up_to_zero_sign(true_q, o_true)
    assert gptq_torch.equal_up_to_zero_sign(recip_q, o_recip)
    assert not gptq_torch.equal_up_to_zero_sign(true_q, recip_q)
    assert gptq_torch.equal_up_to_zero_sign(gptq_torch.gptq_quantize(Wt, Ht, gt), recip_q)


@pytest.mark.parametrize("M,K,ratio,seed", [
    (300, 1040, 0.1, 1), (128, 4096, 0.1, 2), (1, 16, 1.0, 3), (129, 208, 0.5, 4),
    (257, 512, 0.0, 5),
])
def test_gptq_matches_oracle_random(gq, oracle, M, K, ratio, seed):
    from memboost_b200 import workloads
    x = workloads.calibration_activations(4 * K, K, seed=seed, dtype=torch.float16).cuda()
    H = gq.hessian(x, alpha=1.0 / x.shape[0])
    h_diag, Hc = gq.gptq_inverse(H)
    g = torch.Generator().manual_seed(seed)
    W = (torch.randn((M, K), generator=g) * 0.02).cuda()
    gp = gq.compute_group_precision(W, h_diag, ratio) if ratio > 0 else \
        torch.zeros(K // 16, dtype=torch.uint8, device="cuda")
    Wn, Hn, gn = W.cpu().numpy(), Hc.cpu().numpy(), gp.cpu().numpy()
    for mode in (gq.GPTQ_DIV_TRUE, gq.GPTQ_DIV_RECIPROCAL):
        Q = gq.gptq_quantize(W, Hc, gp, scalar_division=mode)
        want = oracle.gptq_quantize(Wn, Hn, gn, div_mode=mode)
        assert gptq_torch.equal_up_to_zero_sign(Q, torch.from_numpy(want)), mode


def test_gptq_full_size_matches_reference_on_cuda(gq):
    """A full 4096 x 4096 projection (32 blocks of 128 columns, ratio 0.1)
    against the reference's column loop run on CUDA tensors, bit for bit."""
    from memboost_b200 import workloads
    K, M = 4096, 4096
    x = workloads.calibration_activations(4 * K, K, seed=31, device="cuda")
    h_diag, Hc = gq.gptq_inverse(gq.hessian(x, alpha=1.0 / x.shape[0]))
    W = (torch.randn((M, K), generator=torch.Generator().manual_seed(8)) * 0.02).cuda()
    gp = gq.compute_group_precision(W, h_diag, 0.1)
    Q = gq.gptq_quantize(W, Hc, gp)
    want = gptq_torch.gptq_quantize(W, Hc, gp)
    assert gptq_torch.equal_up_to_zero_sign(Q, want)


def test_gptq_rejects_bad_arguments(gq):
    W = torch.zeros(4, 24, device="cuda")
    with pytest.raises(RuntimeError, match="multiple of 16"):
        gq.gptq_quantize(W, torch.eye(24, device="cuda"), torch.zeros(1, dtype=torch.uint8))
    W = torch.zeros(4, 32, device="cuda")
    with pytest.raises(RuntimeError, match="blocksize"):
        gq.gptq_quantize(W, torch.eye(32, device="cuda"), torch.zeros(2, dtype=torch.uint8),
                         blocksize=64)


# ---------------------------------------------------------------------------
# GPTQ -> memboost quantize
# ---------------------------------------------------------------------------

def test_make_quantized_linear_selects_gptq_groups(gq):
    from memboost_b200 import workloads
    K, M = 1024, 384
    x = workloads.calibration_activations(4096, K, seed=21, dtype=torch.float16).cuda()
    h_diag, Hc = gq.gptq_inverse(gq.hessian(x, alpha=1.0 / 4096))
    W = (torch.randn((M, K), generator=torch.Generator().manual_seed(3)) * 0.02).cuda()
    ql = gq.make_quantized_linear(W, h_diag, Hc, 0.1)
    gp = gq.compute_group_precision(W, h_diag, 0.1)
    assert torch.equal(ql.q_weight.group_precision, gp)
    y = ql(torch.randn(2, K, device="cuda"))
    assert y.shape == (2, M) and y.dtype == torch.float16
    ql0 = gq.make_quantized_linear(W, h_diag, Hc, 0.0)
    assert int(ql0.q_weight.group_precision.sum()) == 0


def test_quantize_layer_small(gq):
    from memboost_b200 import workloads
    weights, inputs = workloads.gptq_layer(tokens=8192, device="cuda", scale=8)
    out = gq.quantize_layer(weights, inputs, ratio_4bit=0.1)
    assert set(out) == set(weights)
    for name, qt in out.items():
        assert (qt.M, qt.K) == tuple(weights[name].shape)
        assert int(qt.group_precision.sum()) == int(0.1 * (qt.K // 16))


def test_quantize_layer_full_shapes(gq):
    """One Llama-7B layer at full weight shapes (calibration shortened to
    16384 tokens): every matrix quantized with GPTQ's own 4-bit groups."""
    from memboost_b200 import workloads
    weights, inputs = workloads.gptq_layer(tokens=16384, device="cuda")
    out = gq.quantize_layer(weights, inputs, ratio_4bit=0.1)
    for name, qt in out.items():
        M, K = weights[name].shape
        assert (qt.M, qt.K) == (M, K)
        assert int(qt.group_precision.sum()) == int(0.1 * (K // 16))


def test_quantize_layer_overlapped_equals_sequential(gq):
    """quantize_layer runs the inverses in worker threads beside the GPTQ
    updates; its tensors equal the plain sequence (Hessian, gptq_inverse,
    make_quantized_linear, one matrix after another) bit for bit."""
    from memboost_b200 import workloads
    weights, inputs = workloads.gptq_layer(tokens=4096, device="cuda", scale=8)
    out = gq.quantize_layer(weights, inputs, ratio_4bit=0.1)
    inv = {}
    for key, x in inputs.items():
        acc = gq.HessianAccumulator(x.shape[-1], x.device)
        acc.add(x)
        inv[key] = gq.gptq_inverse(acc.finalize())
    for name, W in weights.items():
        h_diag, hc = inv[gq.LAYER_INPUTS[name]]
        want = gq.make_quantized_linear(W, h_diag, hc, 0.1).q_weight
        got = out[name]
        for f in ("packed_2bit", "packed_4bit", "scales_1st", "zeros_1st", "scales_2nd",
                  "zeros_2nd", "scales_1st_quant", "group_precision", "outlier_values",
                  "outlier_col_indices", "outlier_row_ptrs"):
            a, b = getattr(got, f), getattr(want, f)
            if a.dtype == torch.float16:
                a, b = a.view(torch.int16), b.view(torch.int16)
            assert torch.equal(a, b), (name, f)
