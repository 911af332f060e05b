"""mb_quantize_csr_many: jobs that share launches (up to 8 matrices per launch
of each kernel, their CTAs split among the matrices) give exactly the
outputs, flags and diagnostics of one quantize call per matrix -- mixed
shapes, with and without the sensitivity pass, outliers, ties, more jobs
than one launch takes, and shapes that need the single-matrix encode."""
import pytest
import torch

pytestmark = pytest.mark.gpu

FIELDS = ("packed_2bit", "packed_4bit", "scales_1st", "zeros_1st", "scales_2nd", "zeros_2nd",
          "scales_1st_quant", "group_precision", "outlier_values", "outlier_col_indices",
          "outlier_row_ptrs")


def _cases():
    from memboost_b200 import workloads as wl
    return [(wl.small_case(1000, 4096, seed=3), 0.1),
            (wl.small_case(384, 1024, seed=12, kind="shifted"), 0.1),   # outliers
            (wl.small_case(640, 1024, seed=21, kind="ties"), 0.25),     # tie flag
            (wl.small_case(129, 256, seed=5), 0.1),
            (wl.small_case(4096, 512, seed=8, kind="tiny"), 0.2),
            (wl.small_case(300, 1040, seed=12, kind="shifted"), 0.1),   # ng % 16 != 0: alone
            (wl.small_case(520, 2048, seed=4), 0.0),                    # no sensitivity pass
            (wl.small_case(2048, 768, seed=30), 0.1),
            (wl.small_case(777, 1536, seed=31), 0.1),
            (wl.small_case(256, 4096, seed=32, kind="const"), 0.1),
            (wl.small_case(1100, 256, seed=33), 0.1)]


def _inputs(dev):
    cases = _cases()
    W = [c.weights.to(dev) for c, _ in cases]
    H = [c.hessian_diag.to(dev) for c, _ in cases]
    return W, [r for _, r in cases], H


def _same(got, want, tag):
    for k, f in enumerate(FIELDS):
        a, b = got[k], want[k] if isinstance(want, list) else getattr(want, f)
        assert a.shape == b.shape, (tag, f)
        assert torch.equal(a.cpu(), b.cpu()), (tag, f)


@pytest.mark.parametrize("per_launch", [8, 3])
def test_shared_launches_match_single(per_launch):
    import memboost_b200 as mb
    from memboost_b200 import _C
    dev = torch.device("cuda", 0)
    W, ratios, H = _inputs(dev)
    want = [mb.quantize(w, r, h) for w, r, h in zip(W, ratios, H)]
    # CSR arrays large enough for every matrix (no overflow flag on either side)
    cap = 1 << 22  # at least M * K for every case
    single = _C.QuantizeBatch(W, ratios, H, dev, branches=1, per_launch=1, csr_capacity=cap)
    shared = _C.QuantizeBatch(W, ratios, H, dev, branches=2, per_launch=per_launch,
                              csr_capacity=cap)
    single.launch()
    ref = single.finish()
    ref_info = [ws.info() for ws in single.ws]
    assert ref_info[2]["flags"] & _C.FLAG_SELECTION_TIE
    assert int(want[1].outlier_values.numel()) > 0
    for rep in range(2):
        shared.launch()
        got = shared.finish()
        for i in range(len(W)):
            _same(got[i], want[i], (rep, i))
            _same(got[i], ref[i], (rep, i))
            assert shared.ws[i].info() == ref_info[i], (rep, i)


def test_one_call_more_jobs_than_a_launch_takes():
    """All eleven jobs in one mb_quantize_csr_many call: it forms the launch
    groups itself (8 at most, broken by the single-matrix shapes and the job
    without a hessian)."""
    import ctypes
    import memboost_b200 as mb
    from memboost_b200 import _C
    dev = torch.device("cuda", 0)
    W, ratios, H = _inputs(dev)
    # ten jobs on the wide-tile encode with the sensitivity pass, in a row
    keep = [i for i in range(len(W)) if i not in (5, 6)]
    W = [W[i] for i in keep] + [W[0].flip(1).contiguous(), W[7].flip(0).contiguous()]
    H = [H[i] for i in keep] + [H[0].flip(0).contiguous(), H[7]]
    ratios = [ratios[i] for i in keep] + [0.1, 0.1]
    assert len(W) == 11
    want = [mb.quantize(w, r, h) for w, r, h in zip(W, ratios, H)]
    b = _C.QuantizeBatch(W, ratios, H, dev, branches=1, per_launch=1, csr_capacity=1 << 22)
    arr = (_C.QuantizeJob * len(W))(*b.jobs)
    stream = torch.cuda.current_stream(dev)
    _C._check(_C._lib.mb_quantize_csr_many(arr, len(W), ctypes.c_void_p(stream.cuda_stream)))
    torch.cuda.synchronize(dev)
    nnz = b.nnz_dev.cpu().tolist()
    for i in range(len(W)):
        assert nnz[i] <= b.cap[i]
        got = [*b.out[i], b.vals[i][:nnz[i]], b.cols[i][:nnz[i]], b.row_ptrs[i]]
        _same(got, want[i], i)


def test_bad_job_enqueues_nothing():
    """A job that fails validation stops the call before any launch: the
    other jobs' outputs stay as they were."""
    import ctypes
    from memboost_b200 import _C
    dev = torch.device("cuda", 0)
    W, ratios, H = _inputs(dev)
    b = _C.QuantizeBatch(W[:3], ratios[:3], H[:3], dev, branches=1, per_launch=1)
    for o in b.out[0]:
        o.fill_(7)
    jobs = list(b.jobs)
    jobs[2] = _C.QuantizeJob.from_buffer_copy(jobs[2])
    jobs[2].workspace_bytes = 16  # too small
    arr = (_C.QuantizeJob * 3)(*jobs)
    stream = torch.cuda.current_stream(dev)
    st = _C._lib.mb_quantize_csr_many(arr, 3, ctypes.c_void_p(stream.cuda_stream))
    assert st != 0
    assert b"workspace" in _C._lib.mb_last_error()
    torch.cuda.synchronize(dev)
    assert all(bool((o == 7).all()) for o in b.out[0])
