"""memboost oracle -- TEST INFRASTRUCTURE ONLY.

ctypes wrapper over ``oracle/libmb_oracle.so`` (the C++ restatement of the
reference pipeline in ``oracle/mb_oracle.cpp``).  Only ``tests/``,
``__graft_entry__.smoke()`` and ``bench.py``'s CPU-baseline leg use it, and
only as the checker; the product path (``memboost_b200``) never imports it.

All arrays are numpy; fp16 data is passed as ``np.float16`` (bit patterns are
what the oracle reads).  ``quantize`` returns the reference's 11-tensor list
order (core/torch_ops.cu:251-263) as a dict.
"""
from __future__ import annotations

import ctypes
import os
import subprocess

import numpy as np

_HERE = os.path.dirname(os.path.abspath(__file__))
_LIB_PATH = os.path.join(_HERE, "libmb_oracle.so")
_lib = None

GROUP_SIZE_1ST = 16
GROUP_SIZE_2ND = 256

# Outlier-test arithmetic of the reference kernel (quantize.cu:192-194):
# FMA_MODE = 1 evaluates |w - scale*(q-zero)| with a single rounding (the
# product fused into the subtraction), 0 rounds the product first.  The GPU
# parity tests against the compiled reference decide which one it is.
FMA_MODE = 1


def build() -> str:
    """Compile the oracle with its Makefile (idempotent)."""
    subprocess.run(["make", "-s", "-C", _HERE], check=True)
    return _LIB_PATH


def lib():
    global _lib
    if _lib is None:
        if not os.path.exists(_LIB_PATH):
            build()
        L = ctypes.CDLL(_LIB_PATH)
        P = ctypes.c_void_p
        I64 = ctypes.c_int64
        L.mbo_quantize.restype = ctypes.c_int
        L.mbo_quantize.argtypes = [P, I64, I64, ctypes.c_double, P, I64, ctypes.c_int, ctypes.c_int,
                                   P, P, P, P, P, P, P, P, P, P, P, I64, P, P, P, P]
        L.mbo_dequantize.restype = ctypes.c_int
        L.mbo_dequantize.argtypes = [P, P, P, P, P, I64, I64, P, ctypes.c_int]
        L.mbo_group_stats.argtypes = [P, I64, I64, P, P, ctypes.c_int]
        L.mbo_sensitivity.argtypes = [P, I64, I64, P, P, ctypes.c_int]
        L.mbo_select.argtypes = [P, I64, ctypes.c_double, P]
        for n in ("mbo_pack_2bit", "mbo_pack_4bit"):
            getattr(L, n).argtypes = [P, I64, P]
        for n in ("mbo_unpack_2bit", "mbo_unpack_4bit"):
            getattr(L, n).argtypes = [P, I64, I64, P]
        L.mbo_gptq_quantize.argtypes = [P, I64, I64, P, P, I64, ctypes.c_int, P, ctypes.c_int]
        L.mbo_f16_to_f32.restype = ctypes.c_float
        L.mbo_f16_to_f32.argtypes = [ctypes.c_uint16]
        L.mbo_f32_to_f16.restype = ctypes.c_uint16
        L.mbo_f32_to_f16.argtypes = [ctypes.c_float]
        _lib = L
    return _lib


def _p(a: np.ndarray):
    return a.ctypes.data_as(ctypes.c_void_p)


def num_groups(K: int) -> int:
    return (K + GROUP_SIZE_1ST - 1) // GROUP_SIZE_1ST


def quantize(w: np.ndarray, ratio_4bit: float = 0.1, hessian_diag: np.ndarray | None = None,
             fma_mode: int | None = None, nthreads: int = 0, debug: bool = False) -> dict:
    """Reference pipeline on the CPU (core/torch_ops.cu:105-264)."""
    w = np.ascontiguousarray(w, dtype=np.float16)
    assert w.ndim == 2
    M, K = w.shape
    ng = num_groups(K)
    ng2 = (M * ng + GROUP_SIZE_2ND - 1) // GROUP_SIZE_2ND
    fm = FMA_MODE if fma_mode is None else fma_mode
    out = {
        "packed_2bit": np.zeros((M, ng), np.int32),
        "packed_4bit": np.zeros((M, 2 * ng), np.int32),
        "scales_1st": np.zeros((M, ng), np.float16),
        "zeros_1st": np.zeros((M, ng), np.int8),
        "scales_2nd": np.zeros((ng2,), np.float16),
        "zeros_2nd": np.zeros((ng2,), np.int8),
        "scales_1st_quant": np.zeros((M, ng), np.uint8),
        "group_precision": np.zeros((ng,), np.uint8),
        "outlier_row_ptrs": np.zeros((M + 1,), np.int32),
    }
    if hessian_diag is not None:
        h = np.ascontiguousarray(hessian_diag, dtype=np.float32)
        assert h.size >= K or h.size == 0
        hp, hn = (_p(h), h.size) if h.size else (None, 0)
    else:
        h, hp, hn = None, None, 0
    gmin = np.zeros(ng, np.float32)
    gmax = np.zeros(ng, np.float32)
    sens = np.full(ng, np.nan, np.float32)
    cap = min(M * K, 1 << 20)
    while True:
        vals = np.zeros((cap,), np.float16)
        cols = np.zeros((cap,), np.int32)
        nnz = ctypes.c_int64(0)
        rc = lib().mbo_quantize(
            _p(w), M, K, float(ratio_4bit), hp, hn, fm, nthreads,
            _p(out["packed_2bit"]), _p(out["packed_4bit"]), _p(out["scales_1st"]), _p(out["zeros_1st"]),
            _p(out["scales_2nd"]), _p(out["zeros_2nd"]), _p(out["scales_1st_quant"]),
            _p(out["group_precision"]), _p(out["outlier_row_ptrs"]), _p(vals), _p(cols), cap,
            ctypes.byref(nnz), _p(gmin), _p(gmax), _p(sens))
        if rc == 1:
            cap = nnz.value
            continue
        if rc != 0:
            raise ValueError(f"oracle quantize failed: rc={rc}")
        break
    n = nnz.value
    out["outlier_values"] = vals[:n].copy()
    out["outlier_col_indices"] = cols[:n].copy()
    out["M"], out["K"] = M, K
    if debug:
        out["_gmin"], out["_gmax"], out["_sens"] = gmin, gmax, sens
    return out


def dequantize(q: dict, nthreads: int = 0) -> np.ndarray:
    """Reference dequantize (core/quantize.cu:386-444), no outlier add-back."""
    M, K = q["M"], q["K"]
    out = np.zeros((M, K), np.float16)
    args = [np.ascontiguousarray(q[k]) for k in
            ("packed_2bit", "packed_4bit", "scales_1st", "zeros_1st", "group_precision")]
    rc = lib().mbo_dequantize(*[_p(a) for a in args], M, K, _p(out), nthreads)
    if rc != 0:
        raise ValueError("oracle dequantize failed")
    return out


def dequantize_2nd(q: dict, add_outliers: bool = True) -> np.ndarray:
    """Dequantize from the compact scales (numpy; the reference has no such
    function -- it computes scales_1st_quant / scales_2nd / zeros_2nd in
    core/quantize.cu:245-280 and never reads them back).  Each group's scale
    is rebuilt by the reference's dequantize rule (core/quantize.cu:386-444)
    one level up, then the weights are decoded with it:
        s = fp16(f32(scales_2nd[c]) * (f32(q2) - f32(zeros_2nd[c]))),
            q2 = scales_1st_quant[r, g], c = (r * ng + g) // 256
        w = fp16(f32(s) * (f32(q) - f32(zeros_1st[r, g])))
    (fp32 subtraction and product each rounded); CSR outliers written back."""
    return decode_with_scales(q, rebuilt_scales(q), add_outliers)


def rebuilt_scales(q: dict) -> np.ndarray:
    """fp16 [M, ng]: each group's scale from its 4-bit 2nd-order code."""
    M, K = int(q["M"]), int(q["K"])
    ng = num_groups(K)
    c = np.arange(M * ng, dtype=np.int64) // GROUP_SIZE_2ND
    s2 = np.asarray(q["scales_2nd"]).reshape(-1).astype(np.float32)[c]
    z2 = np.asarray(q["zeros_2nd"]).reshape(-1).astype(np.float32)[c]
    q2 = np.asarray(q["scales_1st_quant"]).reshape(-1).astype(np.float32)
    s = (s2 * (q2 - z2).astype(np.float32)).astype(np.float32).astype(np.float16)
    return s.reshape(M, ng)


def decode_with_scales(q: dict, scales: np.ndarray, add_outliers: bool = False) -> np.ndarray:
    """fp16 [M, K] from the codes and zeros of q with the given fp16 [M, ng]
    scales (with q's scales_1st this is the reference dequantize)."""
    M, K = int(q["M"]), int(q["K"])
    ng = num_groups(K)
    s = np.asarray(scales, dtype=np.float16).reshape(M, ng).astype(np.float32)
    z1 = np.asarray(q["zeros_1st"]).reshape(M, ng).astype(np.float32)
    gp = np.asarray(q["group_precision"]).reshape(-1)[:ng] != 0
    p2 = np.asarray(q["packed_2bit"]).reshape(M, ng).astype(np.int64) & 0xFFFFFFFF
    p4 = np.asarray(q["packed_4bit"]).reshape(M, ng, 2).astype(np.int64) & 0xFFFFFFFF
    i = np.arange(16)
    code2 = (p2[:, :, None] >> (2 * i)) & 0x3
    code4 = (np.where(i < 8, p4[:, :, 0:1], p4[:, :, 1:2]) >> (4 * (i & 7))) & 0xF
    code = np.where(gp[None, :, None], code4, code2).astype(np.float32)
    w = (s[:, :, None] * (code - z1[:, :, None]).astype(np.float32)).astype(np.float32)
    out = w.astype(np.float16).reshape(M, ng * 16)[:, :K].copy()
    if add_outliers:
        rp = np.asarray(q["outlier_row_ptrs"]).reshape(-1)
        cols = np.asarray(q["outlier_col_indices"]).reshape(-1)
        vals = np.asarray(q["outlier_values"]).reshape(-1).astype(np.float16)
        if vals.size:
            rows = np.repeat(np.arange(M), np.diff(rp[:M + 1]))
            out[rows, cols] = vals
    return out


def group_stats(w: np.ndarray, nthreads: int = 0):
    w = np.ascontiguousarray(w, dtype=np.float16)
    M, K = w.shape
    ng = num_groups(K)
    mn, mx = np.zeros(ng, np.float32), np.zeros(ng, np.float32)
    lib().mbo_group_stats(_p(w), M, K, _p(mn), _p(mx), nthreads)
    return mn, mx


def sensitivity(w: np.ndarray, h: np.ndarray, nthreads: int = 0) -> np.ndarray:
    w = np.ascontiguousarray(w, dtype=np.float16)
    h = np.ascontiguousarray(h, dtype=np.float32)
    M, K = w.shape
    s = np.zeros(num_groups(K), np.float32)
    lib().mbo_sensitivity(_p(w), M, K, _p(h), _p(s), nthreads)
    return s


def select(sens: np.ndarray, ratio: float) -> np.ndarray:
    sens = np.ascontiguousarray(sens, dtype=np.float32)
    gp = np.zeros(sens.size, np.uint8)
    lib().mbo_select(_p(sens), sens.size, float(ratio), _p(gp))
    return gp


def pack_2bit(v: np.ndarray) -> np.ndarray:
    v = np.ascontiguousarray(v, dtype=np.uint8)
    assert v.size % 16 == 0
    out = np.zeros(v.size // 16, np.int32)
    lib().mbo_pack_2bit(_p(v), out.size, _p(out))
    return out


def unpack_2bit(p: np.ndarray, num_elements: int) -> np.ndarray:
    p = np.ascontiguousarray(p, dtype=np.int32)
    assert num_elements <= p.size * 16
    out = np.zeros(num_elements, np.uint8)
    lib().mbo_unpack_2bit(_p(p), p.size, num_elements, _p(out))
    return out


def pack_4bit(v: np.ndarray) -> np.ndarray:
    v = np.ascontiguousarray(v, dtype=np.uint8)
    assert v.size % 8 == 0
    out = np.zeros(v.size // 8, np.int32)
    lib().mbo_pack_4bit(_p(v), out.size, _p(out))
    return out


def unpack_4bit(p: np.ndarray, num_elements: int) -> np.ndarray:
    p = np.ascontiguousarray(p, dtype=np.int32)
    assert num_elements <= p.size * 8
    out = np.zeros(num_elements, np.uint8)
    lib().mbo_unpack_4bit(_p(p), p.size, num_elements, _p(out))
    return out


def f32_to_f16_bits(x: float) -> int:
    return int(lib().mbo_f32_to_f16(float(x)))


def f16_bits_to_f32(b: int) -> float:
    return float(lib().mbo_f16_to_f32(int(b)))


# (w - gmin) / sc in gptq_quantize (models/llama.py:278): PyTorch's IEEE
# quotient on CPU tensors, multiplication by the fp32 reciprocal on CUDA.
GPTQ_DIV_TRUE = 0
GPTQ_DIV_RECIPROCAL = 1


def gptq_quantize(W: np.ndarray, hinv_cho: np.ndarray, group_precision: np.ndarray,
                  blocksize: int = 128, div_mode: int = GPTQ_DIV_TRUE,
                  nthreads: int = 0) -> np.ndarray:
    """gptq_quantize of models/llama.py:234-294 on fp32 numpy arrays."""
    W = np.ascontiguousarray(W, dtype=np.float32)
    M, K = W.shape
    assert K % GROUP_SIZE_1ST == 0
    Hc = np.ascontiguousarray(hinv_cho, dtype=np.float32)
    assert Hc.shape == (K, K)
    gp = np.ascontiguousarray(group_precision, dtype=np.uint8)
    assert gp.shape == (K // GROUP_SIZE_1ST,)
    Q = np.empty_like(W)
    lib().mbo_gptq_quantize(_p(W), M, K, _p(Hc), _p(gp), blocksize, div_mode, _p(Q), nthreads)
    return Q
