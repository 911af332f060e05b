"""Bit-exact parity (against the CPU oracle) at shapes that stress how the
stats kernel splits the tiles among its CTAs: each CTA streams a contiguous
column-major range of 128 x 128 tiles and keeps per-segment partials (its
chunks of one column tile); the CTA completing a column tile combines them.

  * one column tile split over every CTA of the grid (more segments than a
    warp's 32 lanes: the combine loops);
  * CTA ranges that cross two or three column tiles of two chunks each;
  * partial last chunks (rows) and partial last groups (columns), with and
    without outliers, with and without a hessian.
"""
import numpy as np
import pytest
import torch

from cases import OUTPUT_FIELDS, diff_fields
from memboost_b200 import workloads

pytestmark = pytest.mark.gpu

SHAPES = [
    # (M, K, kind, seed, ratio, hessian)
    (38400, 32, "normal", 21, 0.5, True),     # 300 row chunks of one column tile
    (38400, 16, "normal", 22, 0.0, False),    # the same without a hessian (no sums)
    (256, 65536, "normal", 23, 0.1, True),    # 512 column tiles of 2 chunks
    (130, 32768, "shifted", 24, 0.25, True),  # last chunk of 2 rows, outliers
    (8191, 1000, "normal", 25, 0.3, True),    # last chunk 127 rows, last group 8 columns
    (20000, 48, "shifted", 26, 0.5, True),    # 157 chunks, 3 groups in one column tile
]


def _case(M, K, kind, seed, hess):
    mc = workloads.small_case(M, K, seed, kind)
    w = mc.weights.numpy()
    h = mc.hessian_diag.numpy().astype(np.float32) if hess else None
    return w, h


@pytest.mark.parametrize("M,K,kind,seed,ratio,hess", SHAPES,
                         ids=[f"{s[0]}x{s[1]}_{s[2]}_r{s[4]}{'' if s[5] else '_nohess'}"
                              for s in SHAPES])
def test_segmented_stats_match_oracle(M, K, kind, seed, ratio, hess, oracle):
    from memboost_b200 import _C
    w, h = _case(M, K, kind, seed, hess)
    wt = torch.from_numpy(w).cuda()
    ht = None if h is None else torch.from_numpy(h).cuda()
    out = _C.quantize(wt, ratio, ht)
    got = {f: t.cpu().numpy() for f, t in zip(OUTPUT_FIELDS, out)}
    got["M"], got["K"] = M, K
    want = oracle.quantize(w, ratio, h)
    assert diff_fields(got, want) == []
