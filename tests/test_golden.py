"""The CPU oracle against golden fixtures produced by the reference's own
compiled kernels on a GPU (tests/golden/make_golden.py).  CPU only."""
import glob
import os

import numpy as np
import pytest

from cases import OUTPUT_FIELDS, diff_fields

GOLDEN = sorted(p for p in glob.glob(os.path.join(os.path.dirname(__file__), "golden", "*.npz"))
                if not os.path.basename(p).startswith("gptq_"))


def test_fixtures_present():
    assert len(GOLDEN) >= 22, "golden fixtures missing (tests/golden/make_golden.py)"


@pytest.mark.parametrize("path", GOLDEN, ids=[os.path.basename(p)[:-4] for p in GOLDEN])
def test_oracle_matches_golden(path, oracle):
    g = np.load(path)
    h = g["hessian_diag"] if bool(g["has_hessian"]) else None
    got = oracle.quantize(g["weights"], float(g["ratio_4bit"]), h)
    assert diff_fields(got, {f: g[f] for f in OUTPUT_FIELDS}) == []
    d = oracle.dequantize(got)
    assert np.array_equal(d.view(np.uint16), g["dequantized"].view(np.uint16))
