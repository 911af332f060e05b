"""Generate the GPTQ golden fixtures from the reference's own Python code.

Imports the reference's models/llama.py (its memboost package, with the
compiled reference extension from oracle/_ref standing in for memboost._C) and
runs, on CPU tensors, its gptq_inverse (llama.py:177-203),
compute_group_precision (llama.py:209-231) and gptq_quantize
(llama.py:234-294) on seeded synthetic inputs.  One .npz per case holds the
inputs and every intermediate, so tests/test_gptq_golden.py can pin the CPU
oracle and the GPU kernel without the reference present.

Usage (needs the reference checkout): python tests/golden/make_gptq_golden.py [REF_ROOT]
"""
import importlib.util
import os
import sys

import numpy as np
import torch

HERE = os.path.dirname(os.path.abspath(__file__))
REPO = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, REPO)


def load_reference_llama(ref_root: str):
    from oracle import build_ref

    sys.modules["memboost._C"] = build_ref.load()
    sys.path.insert(0, ref_root)
    import memboost  # noqa: F401  (the reference package)

    spec = importlib.util.spec_from_file_location("ref_llama",
                                                  os.path.join(ref_root, "models", "llama.py"))
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


def _workloads():
    spec = importlib.util.spec_from_file_location(
        "mb_workloads", os.path.join(REPO, "memboost_b200", "workloads.py"))
    mod = importlib.util.module_from_spec(spec)
    sys.modules["mb_workloads"] = mod
    spec.loader.exec_module(mod)
    return mod


KEEP_X_ELEMENTS = 300_000  # calibration inputs kept only for the smaller cases


def hessian_fp32(x16: torch.Tensor) -> torch.Tensor:
    """H = x^T x / tokens in fp32 on the CPU (the hook's arithmetic)."""
    x = x16.float()
    H = torch.zeros(x.shape[1], x.shape[1])
    H.add_(x.T @ x)
    H.div_(x.shape[0])
    return H


def cases(wl):
    """(name, W fp32, X fp16 | None, ratio, group_precision override | None)."""
    g = torch.Generator().manual_seed(2024)

    def normal(M, K, std=0.02):
        return torch.randn((M, K), generator=g) * std

    out = []
    out.append(("gptq_96x256_r0.25", normal(96, 256),
                wl.calibration_activations(1024, 256, 1, dtype=torch.float16), 0.25, None))
    out.append(("gptq_33x208_r0.1", normal(33, 208),
                wl.calibration_activations(700, 208, 2, dtype=torch.float16), 0.1, None))
    out.append(("gptq_16x256_r0", normal(16, 256),
                wl.calibration_activations(512, 256, 3, dtype=torch.float16), 0.0, None))
    w = normal(24, 128)
    w[:, 0:16] = 0.0125                 # constant group: scale 0 -> q = gmin
    w[5, 50] = float("nan")             # NaN in group 3 propagates through its block
    out.append(("gptq_24x128_const_nan", w,
                wl.calibration_activations(384, 128, 4, dtype=torch.float16), 0.0,
                torch.tensor([1, 0, 0, 1, 0, 0, 0, 0], dtype=torch.uint8)))
    w = torch.round(normal(40, 384) / 0.005) * 0.005   # coarse grid: exact .5 quotients
    out.append(("gptq_40x384_grid_r0.5", w,
                wl.calibration_activations(1536, 384, 5, dtype=torch.float16), 0.5, None))
    out.append(("gptq_128x384_r0.1", normal(128, 384),
                wl.calibration_activations(2048, 384, 6, dtype=torch.float16), 0.1, None))
    out.append(("gptq_7x48_r1.0", normal(7, 48, 1.0),
                wl.calibration_activations(64, 48, 7, dtype=torch.float16), 1.0, None))
    return out


def main(ref_root: str, out_dir: str) -> None:
    ref = load_reference_llama(ref_root)
    wl = _workloads()
    os.makedirs(out_dir, exist_ok=True)
    for name, W, X, ratio, gp_override in cases(wl):
        H = hessian_fp32(X)
        H_in = H.clone()
        h_diag, hinv_cho = ref.gptq_inverse(H)
        if gp_override is not None:
            gp = gp_override
        elif ratio > 0:
            gp = ref.compute_group_precision(W, h_diag, ratio)
        else:
            gp = torch.zeros(W.shape[1] // 16, dtype=torch.uint8)
        Q = ref.gptq_quantize(W, hinv_cho, gp, blocksize=128)
        extra = {"X": X.numpy()} if X.numel() <= KEEP_X_ELEMENTS else {}
        np.savez_compressed(
            os.path.join(out_dir, f"{name}.npz"), **extra,
            x_seed_shape=np.array(X.shape), H=H_in.numpy(), h_diag=h_diag.numpy(), hinv_cho=hinv_cho.numpy(),
            W=W.numpy(), ratio_4bit=np.float64(ratio), group_precision=gp.numpy(),
            gp_from_sensitivity=np.bool_(gp_override is None and ratio > 0), Q=Q.numpy())
        print(name, tuple(W.shape), int(gp.sum()), "nan" if torch.isnan(Q).any() else "")


if __name__ == "__main__":
    from oracle import build_ref
    main(sys.argv[1] if len(sys.argv) > 1 else build_ref.reference_dir(), HERE)
