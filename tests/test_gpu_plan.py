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
