"""Seeded parity cases shared by the GPU parity tests and the golden-fixture
generator (tests/golden/make_golden.py).  Each case is (name, weights fp16
[M, K] numpy, ratio_4bit, hessian_diag fp32 numpy or None)."""
from __future__ import annotations

import numpy as np

from memboost_b200 import workloads


def _np_case(mc):
    return mc.weights.numpy(), mc.ratio_4bit, mc.hessian_diag.numpy()


def fma_probe(seed: int = 0, M: int = 32, n_groups: int = 6) -> np.ndarray:
    """A matrix whose outlier set differs between the two candidate
    evaluations of the reference's outlier test (quantize.cu:192-194):
    |w - scale*(q-zero)| with the product rounded first, or fused into the
    subtraction.  Each 16-column group is all-positive (zero point clamped to
    0), holds its min and max, and is filled with fp16 values whose error sits
    on the threshold so that the two evaluations disagree."""
    F = np.float32
    allw = np.arange(65536, dtype=np.uint16).view(np.float16).astype(np.float32)
    allw = allw[np.isfinite(allw)]
    rng = np.random.default_rng(seed)
    W = np.zeros((M, 16 * n_groups), np.float16)
    g = 0
    while g < n_groups:
        gmin = F(np.float16(rng.uniform(0.001, 0.3)))
        gmax = F(np.float16(gmin + rng.uniform(0.001, 0.3)))
        if not gmax > gmin:
            continue
        scale = F(F(gmax - gmin) / F(3))
        thr = F(F(0.4) * F(gmax - gmin))
        w = allw[(allw >= gmin) & (allw <= gmax)]
        with np.errstate(invalid="ignore"):
            a = (w - gmin).astype(F) / scale
        q = np.clip(np.floor(a.astype(np.float64) + 0.5), 0, 3).astype(F)  # roundf for a >= 0
        sep = np.abs((w - (scale * q).astype(F)).astype(F))
        fused = np.abs((w.astype(np.float64) - np.float64(scale) * q.astype(np.float64)).astype(F))
        d = (sep > thr) != (fused > thr)
        if not d.any():
            continue
        cand = w[d]
        blk = rng.choice(cand, size=(M, 16)).astype(np.float16)
        blk[0, 0] = np.float16(gmin)
        blk[1, 0] = np.float16(gmax)
        W[:, 16 * g:16 * (g + 1)] = blk
        g += 1
    return W


def small_cases():
    """Small cases covering the reference's tests and the edge cases."""
    out = []
    rng = np.random.default_rng(123)
    # reference tests/test_ops.py: 64x64 randn, pure 2-bit and 0.2 without hessian
    w = rng.standard_normal((64, 64)).astype(np.float16)
    out.append(("ops_64x64_r0", w, 0.0, None))
    out.append(("ops_64x64_r02_nohess", w, 0.2, None))
    # reference tests/test_gemm.py shapes: 256x256 randn and 100x80
    out.append(("gemm_256", rng.standard_normal((256, 256)).astype(np.float16), 0.0, None))
    out.append(("gemm_100x80", rng.standard_normal((100, 80)).astype(np.float16), 0.0, None))
    # native self-test shape: 128x128 U(-0.5, 0.5), all 2-bit
    out.append(("native_128", rng.uniform(-0.5, 0.5, (128, 128)).astype(np.float16), 0.0, None))
    for (M, K, kind, seed, ratio) in [
        (1, 16, "normal", 1, 0.25), (3, 80, "normal", 2, 0.25), (17, 100, "normal", 3, 0.25),
        (17, 4104, "normal", 4, 0.1), (256, 256, "normal", 5, 0.1), (257, 272, "ones", 6, 0.1),
        (100, 96, "shifted", 7, 0.25), (100, 96, "shifted", 8, 1.0), (33, 48, "const", 9, 0.25),
        (64, 192, "ties", 10, 0.25), (64, 4104, "tiny", 11, 0.25), (300, 1040, "shifted", 12, 0.1),
        (129, 688, "normal", 13, 0.1), (77, 136, "normal", 14, 1.5), (5, 33, "shifted", 15, 0.5),
    ]:
        mc = workloads.small_case(M, K, seed, kind)
        wn, _, hn = _np_case(mc)
        out.append((f"{kind}_{M}x{K}_s{seed}_r{ratio}", wn, ratio, hn))
    out.append(("fma_probe", fma_probe(0), 0.0, None))
    out.append(("fma_probe_4bit", fma_probe(1), 1.0, np.ones(96, np.float32)))
    # hessian given but empty, and ratio 0 with hessian: no selection
    out.append(("empty_hess", rng.standard_normal((40, 64)).astype(np.float16), 0.3,
                np.zeros(0, np.float32)))
    out.append(("ratio0_hess", rng.standard_normal((40, 64)).astype(np.float16), 0.0,
                np.ones(64, np.float32)))
    return out


def reference_defined(w, ratio, h) -> bool:
    """False where the reference implementation has undefined behaviour and
    must not be run: with a hessian, ratio_4bit > 0 and int(ratio * ng) > ng
    its host top-k loop reads past the end of its index vector
    (core/torch_ops.cu:172-177; it crashed the reference process here).  This
    implementation and the oracle clamp the count to ng instead."""
    K = w.shape[1]
    ng = (K + 15) // 16
    selecting = h is not None and np.asarray(h).size > 0 and ratio > 0
    return not (selecting and int(ratio * ng) > ng)


OUTPUT_FIELDS = ("packed_2bit", "packed_4bit", "scales_1st", "zeros_1st", "scales_2nd",
                 "zeros_2nd", "scales_1st_quant", "group_precision", "outlier_values",
                 "outlier_col_indices", "outlier_row_ptrs")


def as_bits(a: np.ndarray) -> np.ndarray:
    """fp16 arrays compared by bit pattern."""
    return a.view(np.uint16) if a.dtype == np.float16 else a


def diff_fields(a: dict, b: dict, fields=OUTPUT_FIELDS) -> list[str]:
    bad = []
    for f in fields:
        x, y = np.asarray(a[f]), np.asarray(b[f])
        if x.shape != y.shape or x.dtype != y.dtype or not np.array_equal(as_bits(x), as_bits(y)):
            bad.append(f)
    return bad


def gptq_division_probe(M: int = 8, ng: int = 16, seed: int = 0):
    """(W, hinv_cho, group_precision) on which the two evaluations of
    gptq_quantize's (w - gmin) / sc (models/llama.py:278) give different
    codes: every group has min 0 and a max chosen so that sc's reciprocal is
    inexact, and its other entries sit within a few ulps of the (k + 0.5) * sc
    rounding boundaries where rint(w / sc) != rint(w * fl(1 / sc)).
    hinv_cho = I keeps the columns independent (every update adds err * 0)."""
    f = np.float32
    rng = np.random.default_rng(seed)
    K = 16 * ng
    W = np.zeros((M, K), f)
    gp = (np.arange(ng) % 2).astype(np.uint8)
    for g in range(ng):
        L = 16 if gp[g] else 4
        while True:
            gmax = f(rng.uniform(0.01, 0.1))
            sc = f(np.float64(gmax) / (L - 1))
            r = f(f(1) / sc)
            hits = []
            for k in range(L - 1):
                w = f((k + 0.5) * np.float64(sc))
                for _ in range(4):
                    w = np.nextafter(w, f(-1), dtype=f)
                for _ in range(9):
                    if 0 < w < gmax and np.rint(f(w / sc)) != np.rint(f(w * r)):
                        hits.append(w)
                    w = np.nextafter(w, f(1), dtype=f)
            if len(hits) >= 2:
                break
        block = rng.choice(np.array(hits, f), size=(M, 16))
        block[0, 0], block[0, 1] = f(0), gmax
        W[:, 16 * g:16 * g + 16] = block
    return W, np.eye(K, dtype=f), gp
