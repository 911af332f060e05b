"""QuantizePlan (the repeated-quantization path the benchmark measures): plans
on streams of their own, launched back to back and finished later, give the
same outputs, bit for bit, as the public quantize() call -- including a
matrix with outliers, whose count reaches the host through pinned memory."""
import pytest
import torch

pytestmark = pytest.mark.gpu

FIELDS = ("packed_2bit", "packed_4bit", "scales_1st", "zeros_1st", "scales_2nd", "zeros_2nd",
          "scales_1st_quant", "group_precision", "outlier_values", "outlier_col_indices",
          "outlier_row_ptrs")


def _cases():
    from memboost_b200 import workloads
    return [workloads.small_case(300, 1040, seed=12, kind="shifted"),   # outliers
            workloads.small_case(1000, 4096, seed=3, kind="normal"),
            workloads.small_case(257, 272, seed=6, kind="ones")]


@pytest.mark.parametrize("use_streams", [False, True])
def test_plans_match_quantize(use_streams):
    import memboost_b200 as mb
    from memboost_b200 import _C
    dev = torch.device("cuda", 0)
    cases = _cases()
    W = [c.weights.to(dev) for c in cases]
    H = [c.hessian_diag.to(dev) for c in cases]
    want = [mb.quantize(w, 0.1, h) for w, h in zip(W, H)]
    assert int(want[0].outlier_values.numel()) > 0
    streams = [torch.cuda.Stream(dev) if use_streams else None for _ in cases]
    plans = [_C.QuantizePlan(*w.shape, dev, stream=s) for w, s in zip(W, streams)]
    for _ in range(2):  # twice in a row: buffers reused
        for p, w, h in zip(plans, W, H):
            p.launch(w, 0.1, h)
        got = [p.finish() for p in plans]
        for g, q in zip(got, want):
            for k, f in enumerate(FIELDS):
                a, b = g[k], getattr(q, f)
                assert a.shape == b.shape, f
                assert torch.equal(a.cpu(), b.cpu()), f


@pytest.mark.parametrize("capacity", [None, 5])
def test_batch_graph_matches_quantize(capacity):
    """QuantizeBatch (every matrix's launches recorded once into a CUDA graph,
    CSR extraction chained on the device) gives the public quantize()
    outputs bit for bit, replay after replay; with a capacity below the
    outlier count the batch falls back to a host-sized extraction."""
    import memboost_b200 as mb
    from memboost_b200 import _C
    from memboost_b200 import workloads
    dev = torch.device("cuda", 0)
    cases = _cases() + [workloads.small_case(640, 1024, seed=21, kind="ties"),
                        workloads.small_case(33, 48, seed=9, kind="const")]
    W = [c.weights.to(dev) for c in cases]
    H = [c.hessian_diag.to(dev) for c in cases]
    ratios = [0.1, 0.1, 0.1, 0.25, 0.0]
    want = [mb.quantize(w, r, h) for w, r, h in zip(W, ratios, H)]
    batch = _C.QuantizeBatch(W, ratios, H, dev, branches=3, csr_capacity=capacity)
    for rep in range(3):
        batch.launch()
        got = batch.finish()
        for g, q in zip(got, want):
            for k, f in enumerate(FIELDS):
                a, b = g[k], getattr(q, f)
                assert a.shape == b.shape, (rep, f)
                assert torch.equal(a.cpu(), b.cpu()), (rep, f)
    # new weights copied into the batch's buffers are picked up by the replay
    batch.weights[1].copy_(W[1].flip(0))
    batch.launch()
    got = batch.finish()
    again = mb.quantize(W[1].flip(0).contiguous(), 0.1, H[1])
    for k, f in enumerate(FIELDS):
        assert torch.equal(got[1][k].cpu(), getattr(again, f).cpu()), f
