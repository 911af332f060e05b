"""Row-split quantize (memboost_b200.rowsplit): a matrix's rows split over
P slabs, the slabs' group records exchanged, selection, pending groups
settled from their gathered column strips, slab encodes -- run for all P
ranks in one process on one GPU.  The assembled result equals the
single-GPU quantize bit for bit (and so the reference kernels')."""
import pytest
import torch

from memboost_b200 import workloads

pytestmark = pytest.mark.gpu


def _same(a, b):
    bad = []
    for k, (x, y) in enumerate(zip(a, b)):
        if x.dtype == torch.float16:
            x, y = x.view(torch.int16), y.view(torch.int16)
        if x.shape != y.shape or not torch.equal(x.cpu(), y.cpu()):
            bad.append(k)
    return bad


def _check(case, world):
    from memboost_b200 import _C, rowsplit
    w, h = case.weights.cuda(), case.hessian_diag.cuda()
    want = _C.quantize(w, case.ratio_4bit, h)
    slabs = rowsplit.quantize_rows_local(w, world, case.ratio_4bit, h)
    got = rowsplit.assemble(slabs)
    torch.cuda.synchronize()
    assert _same(got, want) == [], (case.name, world)
    return slabs


@pytest.mark.parametrize("world", [2, 3, 8])
def test_rowsplit_small_cases(world):
    for M, K, kind, seed in ((640, 1024, "normal", 3), (300, 1040, "shifted", 12),
                             (257, 272, "ones", 6), (1000, 4104, "tiny", 11)):
        if M < world * 16:
            continue
        _check(workloads.small_case(M, K, seed, kind), world)


def test_rowsplit_pending_groups_settled():
    """Config 1 (4096x4096, hessian ones) leaves groups straddling the 4-bit
    boundary; their exact serial sums over all rows settle them."""
    slabs = _check(workloads.single_4096(), 4)
    assert slabs[0].n_pending > 0


@pytest.mark.parametrize("i", [0, 1])
def test_rowsplit_mlp_70b_eight_slabs(i):
    """Config 5: the Llama-70B MLP matrices split over 8 slabs."""
    _check(workloads.mlp_70b()[i], 8)


def test_rowsplit_no_hessian():
    c = workloads.small_case(512, 2048, 5, "normal")
    c.hessian_diag = torch.empty(0)
    c.ratio_4bit = 0.0
    _check(c, 4)


@pytest.mark.parametrize("world", [2, 4])
def test_rowsplit_spmd_threads(world):
    """The SPMD entry point (rowsplit.quantize_rows, one call per rank) with
    the ranks as threads exchanging through LocalComm: same collective
    sequence as over NCCL; the assembled result equals quantize()."""
    from memboost_b200 import _C, rowsplit
    for case in (workloads.single_4096(), workloads.small_case(1024, 1040, 12, "shifted")):
        w, h = case.weights.cuda(), case.hessian_diag.cuda()
        want = _C.quantize(w, case.ratio_4bit, h)
        bounds = rowsplit.slab_bounds(w.shape[0], w.shape[1], world)

        def rank_fn(comm, r):
            r0, r1 = bounds[r]
            return rowsplit.quantize_rows(w[r0:r1], w.shape[0], w.shape[1], case.ratio_4bit,
                                          h, comm)

        slabs = rowsplit.run_local(world, rank_fn)
        torch.cuda.synchronize()
        assert _same(rowsplit.assemble(slabs), want) == [], (case.name, world)


def test_rowsplit_too_few_rows_rejected_on_every_rank():
    """Fewer row periods than ranks: every rank refuses before any exchange
    (none is left waiting in a collective)."""
    from memboost_b200 import rowsplit
    case = workloads.small_case(300, 1040, 12, "shifted")  # 2 periods of 256 rows
    w, h = case.weights.cuda(), case.hessian_diag.cuda()

    def rank_fn(comm, r):
        try:
            rowsplit.quantize_rows(w[:0], 300, 1040, 0.1, h, comm)
        except RuntimeError as e:
            return "periods" in str(e)
        return False

    assert rowsplit.run_local(4, rank_fn) == [True] * 4
