"""mb_quantize_noalloc: quantize with the scratch in a static device array,
for callers that cannot allocate device memory (a host whose GPU memory is
owned by its own fixed arena, or a path that must not reach cudaMalloc).

Called through the C ABI and compared bit for bit with the regular entry
point (memboost_b200._C.quantize, which uses a caller workspace) on two calls
in a row -- the second call must not see anything left over from the first.
This file is collected last so a run that stops at the first failure has run
every other test before it."""
import ctypes

import pytest
import torch

from cases import OUTPUT_FIELDS
from memboost_b200 import _C, workloads

pytestmark = pytest.mark.gpu

P = ctypes.c_void_p
I64 = ctypes.c_int64
_fn = _C._lib.mb_quantize_noalloc
_fn.restype = ctypes.c_int
_fn.argtypes = [P, I64, I64, ctypes.c_double, P, I64, P, P, P, P, P, P, P, P, P, P, P, P, I64,
                ctypes.POINTER(ctypes.c_int64), P]

SCRATCH_BYTES = 4 << 20  # MB_NOALLOC_SCRATCH_BYTES in include/memboost_b200.h


def _ptr(t):
    return None if t is None else ctypes.c_void_p(t.data_ptr())


def quantize_noalloc(w: torch.Tensor, ratio: float, h: torch.Tensor | None, capacity: int):
    M, K = w.shape
    ng = (K + 15) // 16
    ng2 = (M * ng + 255) // 256
    dev = w.device
    e = lambda shape, dt: torch.empty(shape, dtype=dt, device=dev)  # noqa: E731
    out = [e((M, ng), torch.int32), e((M, 2 * ng), torch.int32), e((M, ng), torch.float16),
           e((M, ng), torch.int8), e((ng2,), torch.float16), e((ng2,), torch.int8),
           e((M, ng), torch.uint8), e((ng,), torch.uint8)]
    row_ptrs = e((M + 1,), torch.int32)
    nnz_dev = e((1,), torch.int32)
    vals = e((max(capacity, 1),), torch.float16)
    cols = e((max(capacity, 1),), torch.int32)
    nnz = ctypes.c_int64(-1)
    st = _fn(_ptr(w), M, K, ratio, _ptr(h), 0 if h is None else h.numel(),
             *[_ptr(t) for t in out], _ptr(row_ptrs), _ptr(nnz_dev), _ptr(vals), _ptr(cols),
             capacity, ctypes.byref(nnz), ctypes.c_void_p(torch.cuda.current_stream().cuda_stream))
    n = nnz.value
    return st, [*out, vals[:max(n, 0)], cols[:max(n, 0)], row_ptrs], n


def _same(a, b):
    for f, x, y in zip(OUTPUT_FIELDS, a, b):
        if x.dtype == torch.float16:
            x, y = x.view(torch.int16), y.view(torch.int16)
        if x.shape != y.shape or not torch.equal(x.cpu(), y.cpu()):
            return f
    return None


def test_two_calls_in_a_row_match_regular_entry_point():
    first = workloads.small_case(300, 1040, seed=12, kind="shifted")   # with outliers
    second = workloads.mlp_matrix(2048, 4096, seed=3)                 # none, other shape
    seen = []
    for case, ratio in ((first, 0.1), (second, 0.1)):
        w = case.weights.cuda()
        h = case.hessian_diag.cuda()
        want = _C.quantize(w, ratio, h)
        nnz_want = int(want[8].numel())
        st, got, n = quantize_noalloc(w, ratio, h, capacity=max(nnz_want, 1))
        torch.cuda.synchronize()
        assert st == 0, _C._lib.mb_last_error().decode()
        assert n == nnz_want
        assert _same(got, want) is None
        seen.append(n)
    assert seen[0] > 0 and seen[1] == 0  # CSR written, then cleared for the next call


def test_rejects_matrices_beyond_the_static_scratch():
    M, K = 1 << 21, 16  # its per-row outlier counts alone exceed 4 MiB
    assert _C._lib.mb_quantize_workspace_size(M, K) > SCRATCH_BYTES
    nnz = ctypes.c_int64(0)
    st = _fn(None, M, K, 0.1, None, 0, *([None] * 12), 0, ctypes.byref(nnz), None)
    assert st == 1 and b"too large for mb_quantize_noalloc" in _C._lib.mb_last_error()


def test_reports_outlier_count_when_capacity_is_short():
    case = workloads.small_case(100, 96, seed=8, kind="shifted")
    w, h = case.weights.cuda(), case.hessian_diag.cuda()
    want = _C.quantize(w, 1.0, h)
    nnz_want = int(want[8].numel())
    assert nnz_want > 0
    st, got, n = quantize_noalloc(w, 1.0, h, capacity=nnz_want - 1)
    assert st == 1 and n == nnz_want
    assert b"outlier capacity too small" in _C._lib.mb_last_error()
    # everything but the CSR values / columns is still written
    for f, x, y in list(zip(OUTPUT_FIELDS, got, want))[:8]:
        assert torch.equal(x.view(torch.int16) if x.dtype == torch.float16 else x,
                           y.view(torch.int16) if y.dtype == torch.float16 else y), f
