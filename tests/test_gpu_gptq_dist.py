"""GPTQ with rows and calibration tokens split over ranks (ranks as threads
exchanging through rowsplit.LocalComm on one GPU), and the layer-streaming
driver over a small synthetic Llama."""
import pytest
import torch

from oracle import gptq_torch

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def gq():
    from memboost_b200 import gptq
    return gptq


def test_gptq_row_ranges_equal_full(gq):
    """mb_gptq_quantize_rows: any split of the rows reproduces the full Q bit
    for bit (group parameters over all rows)."""
    from memboost_b200 import workloads
    K, M = 512, 300
    x = workloads.calibration_activations(2048, K, seed=5, dtype=torch.float16).cuda()
    h_diag, hc = gq.gptq_inverse(gq.hessian(x, alpha=1.0 / 2048))
    W = (torch.randn((M, K), generator=torch.Generator().manual_seed(2)) * 0.02).cuda()
    gp = gq.compute_group_precision(W, h_diag, 0.25)
    full = gq.gptq_quantize(W, hc, gp)
    for world in (2, 3, 7):
        parts = [gq.gptq_quantize(W, hc, gp, rows=r) for r in gq.even_rows(M, world)]
        assert gptq_torch.equal_up_to_zero_sign(torch.cat(parts, 0), full)


def test_layer_distributed_equals_single_given_inverses(gq):
    from memboost_b200 import rowsplit, workloads
    weights, inputs = workloads.gptq_layer(tokens=4096, device="cuda", scale=8)
    inv = {k: gq.gptq_inverse(gq.hessian(x, alpha=1.0 / x.shape[0])) for k, x in inputs.items()}
    want = {n: gq.make_quantized_linear(W, *inv[gq.LAYER_INPUTS[n]], 0.1).q_weight
            for n, W in weights.items()}

    def rank_fn(comm, r):
        return gq.quantize_layer_distributed(weights, {}, comm, 0.1, inverses=inv)

    for got in rowsplit.run_local(3, rank_fn):
        for n, qt in got.items():
            a, b = qt.state_dict(), want[n].state_dict()
            for k in a:
                if isinstance(a[k], torch.Tensor):
                    assert torch.equal(a[k].cpu(), b[k].cpu()), (n, k)


def test_layer_distributed_token_split(gq):
    """Tokens split over 2 ranks: the all-reduced Hessians agree with one
    device's within fp32 summation order, and every rank gets the same
    tensors."""
    from memboost_b200 import rowsplit, workloads
    weights, inputs = workloads.gptq_layer(tokens=4096, device="cuda", scale=8)

    def rank_fn(comm, r):
        local = {k: x[r::2].contiguous() for k, x in inputs.items()}
        return gq.quantize_layer_distributed(weights, local, comm, 0.1)

    res = rowsplit.run_local(2, rank_fn)
    for n in weights:
        a, b = res[0][n].state_dict(), res[1][n].state_dict()
        for k in a:
            if isinstance(a[k], torch.Tensor):
                assert torch.equal(a[k].cpu(), b[k].cpu()), (n, k)
        assert int(res[0][n].group_precision.sum()) == int(0.1 * (res[0][n].K // 16))


def test_llama_streaming_small():
    from memboost_b200 import llama, rowsplit
    cfg = llama.LlamaConfig(n_embd=256, n_layer=2, n_head=4, n_kv_heads=4, n_inner=688)
    q, stats = llama.quantize_llama_synthetic(cfg, n_samples=8, seq_len=64)
    assert len(q) == 14 and len(stats["seconds_per_layer"]) == 2
    assert stats["compression_ratio"] > 3.0

    def rank_fn(comm, r):
        return llama.quantize_llama_synthetic(cfg, n_samples=8, seq_len=64, comm=comm)[0]

    res = rowsplit.run_local(2, rank_fn)
    assert sorted(res[0]) == sorted(q)
    for n in q:
        assert torch.equal(res[0][n].packed_2bit.cpu(), res[1][n].packed_2bit.cpu())
