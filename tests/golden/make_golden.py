"""Generate golden fixtures from the reference's own compiled kernels.

Runs the reference extension built from its sources (oracle/_ref, see
oracle/build_ref.py) on a CUDA GPU over the seeded small cases of
tests/cases.py and writes one compressed .npz per case: the inputs and all
11 quantize outputs plus the dequantized matrix.  The committed fixtures pin
the CPU oracle without a GPU (tests/test_golden.py).

Usage (on a machine with a GPU): python tests/golden/make_golden.py [OUT_DIR]
"""
import os
import sys

import numpy as np
import torch

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.dirname(HERE))
sys.path.insert(0, os.path.dirname(os.path.dirname(HERE)))

from cases import OUTPUT_FIELDS, reference_defined, small_cases  # noqa: E402
from oracle import build_ref  # noqa: E402


def main(out_dir: str) -> None:
    ref = build_ref.load()
    os.makedirs(out_dir, exist_ok=True)
    for name, w, ratio, h in small_cases():
        if not reference_defined(w, ratio, h):
            print(name, "skipped: reference behaviour undefined")
            continue
        wt = torch.from_numpy(w).cuda()
        ht = torch.Tensor() if h is None else torch.from_numpy(h).cuda()
        out = ref.quantize(wt, ratio, ht)
        deq = ref.dequantize(out[0], out[1], out[2], out[3], out[7], *w.shape)
        torch.cuda.synchronize()
        rec = {f: t.cpu().numpy() for f, t in zip(OUTPUT_FIELDS, out)}
        rec["weights"] = w
        rec["ratio_4bit"] = np.float64(ratio)
        rec["hessian_diag"] = np.zeros(0, np.float32) if h is None else h
        rec["has_hessian"] = np.bool_(h is not None)
        rec["dequantized"] = deq.cpu().numpy()
        np.savez_compressed(os.path.join(out_dir, f"{name}.npz"), **rec)
        print(name, w.shape, int(rec["outlier_row_ptrs"][-1]))


if __name__ == "__main__":
    main(sys.argv[1] if len(sys.argv) > 1 else HERE)
