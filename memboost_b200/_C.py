"""ctypes binding of libmemboost_b200.so -- the replacement for the
reference's pybind11 module ``memboost._C`` (core/bindings.cpp:6-39).

The six functions here take and return torch tensors with the reference's
names, argument meaning, output devices and error messages
(core/torch_ops.cu:20-301); underneath, each calls the C ABI of
include/memboost_b200.h on torch's current CUDA stream of the input's device.
There is no CPU implementation: if the library is missing the import fails,
and the ops require CUDA tensors (pack/unpack copy CPU inputs to the current
CUDA device first, and return CPU tensors as the reference does).
"""
from __future__ import annotations

import ctypes
import os

import torch

_LIB_PATH = os.path.join(os.path.dirname(os.path.abspath(__file__)), "libmemboost_b200.so")

if not os.path.exists(_LIB_PATH):
    raise ImportError(
        f"memboost_b200: native library {_LIB_PATH} is missing; build it with "
        "`python memboost_b200/build.py` (there is no CPU fallback)")

_lib = ctypes.CDLL(_LIB_PATH)

_P = ctypes.c_void_p
_I64 = ctypes.c_int64
_lib.mb_last_error.restype = ctypes.c_char_p
_lib.mb_version.restype = ctypes.c_char_p
_lib.mb_quantize_workspace_size.restype = ctypes.c_size_t
_lib.mb_quantize_workspace_size.argtypes = [_I64, _I64]
_lib.mb_quantize.restype = ctypes.c_int
_lib.mb_quantize.argtypes = [_P, _I64, _I64, ctypes.c_double, _P, _I64,
                             _P, _P, _P, _P, _P, _P, _P, _P, _P, _P, _P, ctypes.c_size_t, _P]
_lib.mb_quantize_extract_outliers.restype = ctypes.c_int
_lib.mb_quantize_extract_outliers.argtypes = [_P, _I64, _I64, _P, _P, _P, _P, ctypes.c_size_t, _P]
_lib.mb_quantize_flags.restype = ctypes.c_int
_lib.mb_quantize_flags.argtypes = [_P, ctypes.c_size_t, _I64, _I64,
                                   ctypes.POINTER(ctypes.c_uint32), _P]
_lib.mb_quantize_csr.restype = ctypes.c_int
_lib.mb_quantize_csr.argtypes = ([_P, _I64, _I64, ctypes.c_double, _P, _I64] + [_P] * 10 +
                                 [_P, _P, _I64, _P, ctypes.c_size_t, _P])


class QuantizeJob(ctypes.Structure):
    """mb_quantize_job: the arguments of one mb_quantize_csr call."""
    _fields_ = [("weights_fp16", _P), ("M", _I64), ("K", _I64), ("ratio_4bit", ctypes.c_double),
                ("hessian_diag", _P), ("hessian_numel", _I64), ("packed_2bit", _P),
                ("packed_4bit", _P), ("scales_1st_fp16", _P), ("zeros_1st", _P),
                ("scales_2nd_fp16", _P), ("zeros_2nd", _P), ("scales_1st_quant", _P),
                ("group_precision", _P), ("outlier_row_ptrs", _P), ("nnz_device", _P),
                ("outlier_values_fp16", _P), ("outlier_col_indices", _P),
                ("outlier_capacity", _I64), ("workspace", _P), ("workspace_bytes", ctypes.c_size_t)]


_lib.mb_quantize_csr_many.restype = ctypes.c_int
_lib.mb_quantize_csr_many.argtypes = [ctypes.POINTER(QuantizeJob), _I64, _P]
_lib.mb_quantize_exact_sums.restype = ctypes.c_int
_lib.mb_quantize_exact_sums.argtypes = [_P, _I64, _I64, ctypes.c_double, _P, _I64, _P, _P, _P,
                                        ctypes.c_size_t, _P]
_lib.mb_rows_record_bytes.restype = ctypes.c_size_t
_lib.mb_rows_record_bytes.argtypes = [_I64]
_lib.mb_rows_stats.restype = ctypes.c_int
_lib.mb_rows_stats.argtypes = [_P, _I64, _I64, ctypes.c_double, _P, _I64, _P, _P,
                               ctypes.c_size_t, _P]
_lib.mb_rows_select.restype = ctypes.c_int
_lib.mb_rows_select.argtypes = [_P, ctypes.c_int, _I64, _P, _I64, _I64, ctypes.c_double, _P, _I64,
                                _P, ctypes.c_size_t, _P, _P, _P]
_lib.mb_rows_set_precision.restype = ctypes.c_int
_lib.mb_rows_set_precision.argtypes = [_P, ctypes.c_size_t, _I64, _I64, _P, _P, _I64, _P]
_lib.mb_rows_encode.restype = ctypes.c_int
_lib.mb_rows_encode.argtypes = [_P, _I64, _I64, ctypes.c_double, _P, _I64] + [_P] * 10 + \
    [_P, ctypes.c_size_t, _P]
_lib.mb_quantize_info.restype = ctypes.c_int
_lib.mb_quantize_info.argtypes = [_P, ctypes.c_size_t, _I64, _I64,
                                  ctypes.POINTER(ctypes.c_uint32), _P]
_lib.mb_dequantize.restype = ctypes.c_int
_lib.mb_dequantize.argtypes = [_P, _P, _P, _P, _P, _I64, _I64, _P, _P]
_lib.mb_qgemv.restype = ctypes.c_int
_lib.mb_qgemv.argtypes = [_P] * 8 + [_I64, _I64, _I64, _P, _P, _P]
_lib.mb_dequantize_2nd.restype = ctypes.c_int
_lib.mb_dequantize_2nd.argtypes = [_P] * 10 + [_I64, _I64, _I64, _P, _P]
for _n in ("mb_pack_2bit", "mb_pack_4bit"):
    getattr(_lib, _n).restype = ctypes.c_int
    getattr(_lib, _n).argtypes = [_P, _I64, _P, _P]
for _n in ("mb_unpack_2bit", "mb_unpack_4bit"):
    getattr(_lib, _n).restype = ctypes.c_int
    getattr(_lib, _n).argtypes = [_P, _I64, _I64, _P, _P]

_lib.mb_hessian.restype = ctypes.c_int
_lib.mb_hessian.argtypes = [_P, _I64, _I64, ctypes.c_int, ctypes.c_float, ctypes.c_int, _P, _P, _P]
_lib.mb_gptq_workspace_size.restype = ctypes.c_size_t
_lib.mb_gptq_workspace_size.argtypes = [_I64, _I64]
_lib.mb_gptq_quantize_rows.restype = ctypes.c_int
_lib.mb_gptq_quantize_rows.argtypes = [_P, _I64, _I64, _I64, _I64, _P, _P, ctypes.c_int,
                                       ctypes.c_int, _P, _P, ctypes.c_size_t, _P]
_lib.mb_gptq_quantize.restype = ctypes.c_int
_lib.mb_gptq_quantize.argtypes = [_P, _I64, _I64, _P, _P, ctypes.c_int, ctypes.c_int, _P, _P,
                                  ctypes.c_size_t, _P]

GROUP_SIZE_1ST = 16
GROUP_SIZE_2ND = 256

# mb_gptq_quantize's evaluation of (w - gmin) / sc: the IEEE quotient
# (PyTorch on CPU tensors) or a product with the fp32 reciprocal (PyTorch on
# CUDA tensors).
GPTQ_DIV_TRUE = 0
GPTQ_DIV_RECIPROCAL = 1
LIB_PATH = _LIB_PATH

# mb_quantize_flags bit 0: a tie of equal sensitivities straddled the 4-bit
# selection boundary (broken by lowest group index); bit 1: a pipeline wait in
# a kernel ran out; bit 2: a 2nd-order zero point wrapped in its int8 cast (the
# reference format's limit: scales rebuilt from the 2nd-order codes are wrong
# for that chunk).
FLAG_SELECTION_TIE = 1
FLAG_TIMEOUT = 2
FLAG_ZERO2_WRAP = 4
FLAG_CSR_OVERFLOW = 8


def version() -> str:
    return _lib.mb_version().decode()


def _check(status: int) -> None:
    if status != 0:
        raise RuntimeError(_lib.mb_last_error().decode() or f"memboost_b200 error {status}")


def _ptr(t: torch.Tensor | None):
    return None if t is None else ctypes.c_void_p(t.data_ptr())


def _stream(device: torch.device):
    return ctypes.c_void_p(torch.cuda.current_stream(device).cuda_stream)


def _to_cuda(t: torch.Tensor) -> torch.Tensor:
    if t.is_cuda:
        return t.contiguous()
    if not torch.cuda.is_available():
        raise RuntimeError("memboost_b200 requires a CUDA device")
    return t.contiguous().to(torch.device("cuda", torch.cuda.current_device()))


# ---- pack / unpack (core/torch_ops.cu:20-102) ----

def _pack(values: torch.Tensor, per: int, fn) -> torch.Tensor:
    if values.dtype != torch.uint8:
        raise RuntimeError("values must be uint8")
    if values.dim() != 1:
        raise RuntimeError("values must be 1D")
    if values.size(0) % per != 0:
        raise RuntimeError(f"length must be multiple of {per}")
    n = values.size(0)
    if n == 0:
        return torch.zeros(0, dtype=torch.int32)
    v = _to_cuda(values)
    with torch.cuda.device(v.device):
        out = torch.empty(n // per, dtype=torch.int32, device=v.device)
        _check(fn(_ptr(v), n, _ptr(out), _stream(v.device)))
    return out.cpu()


def _unpack(packed: torch.Tensor, num_elements: int, per: int, fn) -> torch.Tensor:
    if packed.dtype != torch.int32:
        raise RuntimeError("packed must be int32")
    if packed.dim() != 1:
        raise RuntimeError("packed must be 1D")
    num_elements = int(num_elements)
    if num_elements > packed.size(0) * per:
        raise RuntimeError("num_elements too large")
    if num_elements < 0:
        raise RuntimeError("num_elements must be non-negative")
    if num_elements == 0:
        return torch.zeros(0, dtype=torch.uint8)
    p = _to_cuda(packed)
    with torch.cuda.device(p.device):
        out = torch.empty(num_elements, dtype=torch.uint8, device=p.device)
        _check(fn(_ptr(p), p.size(0), num_elements, _ptr(out), _stream(p.device)))
    return out.cpu()


def pack_2bit(values: torch.Tensor) -> torch.Tensor:
    return _pack(values, 16, _lib.mb_pack_2bit)


def unpack_2bit(packed: torch.Tensor, num_elements: int) -> torch.Tensor:
    return _unpack(packed, num_elements, 16, _lib.mb_unpack_2bit)


def pack_4bit(values: torch.Tensor) -> torch.Tensor:
    return _pack(values, 8, _lib.mb_pack_4bit)


def unpack_4bit(packed: torch.Tensor, num_elements: int) -> torch.Tensor:
    return _unpack(packed, num_elements, 8, _lib.mb_unpack_4bit)


# ---- quantize (core/torch_ops.cu:105-264) ----

class QuantizeWorkspace:
    """Device scratch for mb_quantize, reusable across calls of one shape."""

    def __init__(self, M: int, K: int, device: torch.device):
        self.M, self.K = M, K
        self.nbytes = int(_lib.mb_quantize_workspace_size(M, K))
        self.buf = torch.empty(self.nbytes, dtype=torch.uint8, device=device)
        self.nnz = torch.empty(1, dtype=torch.int32, device=device)

    def flags(self) -> int:
        f = ctypes.c_uint32(0)
        _check(_lib.mb_quantize_flags(_ptr(self.buf), self.nbytes, self.M, self.K,
                                      ctypes.byref(f), _stream(self.buf.device)))
        return int(f.value)

    def info(self) -> dict:
        """Diagnostics of the last quantize on this workspace (mb_quantize_info)."""
        a = (ctypes.c_uint32 * 4)()
        _check(_lib.mb_quantize_info(_ptr(self.buf), self.nbytes, self.M, self.K, a,
                                     _stream(self.buf.device)))
        return {"flags": int(a[0]), "straddling": int(a[1]), "exact_sums": int(a[2]),
                "any_irregular": int(a[3])}


def quantize(weights: torch.Tensor, ratio_4bit: float = 0.1,
             hessian_diag: torch.Tensor | None = None,
             workspace: QuantizeWorkspace | None = None) -> list:
    """Returns the reference's 11-tensor list (core/torch_ops.cu:251-263)."""
    if weights.dtype != torch.float16:
        raise RuntimeError("weights must be float16")
    if weights.dim() != 2:
        raise RuntimeError("weights must be 2D [M, K]")
    if not weights.is_cuda:
        raise RuntimeError("weights must be on CUDA")
    weights = weights.contiguous()
    M, K = int(weights.size(0)), int(weights.size(1))
    if M == 0 or K == 0:
        raise RuntimeError("weights must be non-empty")
    dev = weights.device
    ratio_4bit = float(ratio_4bit)
    h = None
    if hessian_diag is not None and hessian_diag.numel() > 0 and ratio_4bit > 0.0:
        if hessian_diag.dtype != torch.float32:
            raise RuntimeError("hessian_diag must be float32")
        if not hessian_diag.is_cuda:
            raise RuntimeError("hessian_diag must be on CUDA")
        if hessian_diag.device != dev:
            raise RuntimeError("hessian_diag must be on the same device as weights")
        if hessian_diag.numel() < K:
            raise RuntimeError("hessian_diag must hold at least K values")
        h = hessian_diag.contiguous().reshape(-1)
    ng = (K + GROUP_SIZE_1ST - 1) // GROUP_SIZE_1ST
    ng2 = (M * ng + GROUP_SIZE_2ND - 1) // GROUP_SIZE_2ND
    with torch.cuda.device(dev):
        if workspace is None or workspace.M != M or workspace.K != K or workspace.buf.device != dev:
            workspace = QuantizeWorkspace(M, K, dev)
        packed_2bit = torch.empty((M, ng), dtype=torch.int32, device=dev)
        packed_4bit = torch.empty((M, 2 * ng), dtype=torch.int32, device=dev)
        scales_1st = torch.empty((M, ng), dtype=torch.float16, device=dev)
        zeros_1st = torch.empty((M, ng), dtype=torch.int8, device=dev)
        scales_2nd = torch.empty((ng2,), dtype=torch.float16, device=dev)
        zeros_2nd = torch.empty((ng2,), dtype=torch.int8, device=dev)
        scales_1st_quant = torch.empty((M, ng), dtype=torch.uint8, device=dev)
        group_precision = torch.empty((ng,), dtype=torch.uint8, device=dev)
        row_ptrs = torch.empty((M + 1,), dtype=torch.int32, device=dev)
        s = _stream(dev)
        _check(_lib.mb_quantize(
            _ptr(weights), M, K, ratio_4bit, _ptr(h), 0 if h is None else h.numel(),
            _ptr(packed_2bit), _ptr(packed_4bit), _ptr(scales_1st), _ptr(zeros_1st),
            _ptr(scales_2nd), _ptr(zeros_2nd), _ptr(scales_1st_quant), _ptr(group_precision),
            _ptr(row_ptrs), _ptr(workspace.nnz), _ptr(workspace.buf), workspace.nbytes, s))
        nnz = int(workspace.nnz.item())
        if nnz > 0:
            outlier_values = torch.empty((nnz,), dtype=torch.float16, device=dev)
            outlier_col_indices = torch.empty((nnz,), dtype=torch.int32, device=dev)
            _check(_lib.mb_quantize_extract_outliers(
                _ptr(weights), M, K, _ptr(row_ptrs), _ptr(outlier_values),
                _ptr(outlier_col_indices), _ptr(workspace.buf), workspace.nbytes, s))
        else:
            outlier_values = torch.empty((0,), dtype=torch.float16, device=dev)
            outlier_col_indices = torch.empty((0,), dtype=torch.int32, device=dev)
    return [packed_2bit, packed_4bit, scales_1st, zeros_1st, scales_2nd, zeros_2nd,
            scales_1st_quant, group_precision, outlier_values, outlier_col_indices, row_ptrs]


# ---- dequantize (core/torch_ops.cu:267-301) ----

def dequantize(packed_2bit: torch.Tensor, packed_4bit: torch.Tensor, scales_1st: torch.Tensor,
               zeros_1st: torch.Tensor, group_precision: torch.Tensor, M: int, K: int,
               out: torch.Tensor | None = None) -> torch.Tensor:
    if not packed_2bit.is_cuda:
        raise RuntimeError("packed_2bit must be on CUDA")
    if packed_2bit.dtype != torch.int32:
        raise RuntimeError("packed_2bit must be int32")
    M, K = int(M), int(K)
    if M <= 0 or K <= 0:
        raise RuntimeError("M and K must be positive")
    dev = packed_2bit.device
    ng = (K + GROUP_SIZE_1ST - 1) // GROUP_SIZE_1ST
    expect = ((packed_2bit, torch.int32, M * ng, "packed_2bit"),
              (packed_4bit, torch.int32, 2 * M * ng, "packed_4bit"),
              (scales_1st, torch.float16, M * ng, "scales_1st"),
              (zeros_1st, torch.int8, M * ng, "zeros_1st"),
              (group_precision, torch.uint8, ng, "group_precision"))
    for t, dt, n, name in expect:
        if t.device != dev:
            raise RuntimeError(f"{name} must be on the same CUDA device as packed_2bit")
        if t.dtype != dt:
            raise RuntimeError(f"{name} must be {str(dt).replace('torch.', '')}")
        if t.numel() < n:
            raise RuntimeError(f"{name} too small for M={M}, K={K}")
    with torch.cuda.device(dev):
        args = [t.contiguous() for t, *_ in expect]
        if out is None:
            out = torch.empty((M, K), dtype=torch.float16, device=dev)
        elif out.dtype != torch.float16 or out.numel() < M * K or not out.is_contiguous() \
                or out.device != dev:
            raise RuntimeError("out must be a contiguous float16 tensor of at least M * K "
                               "values on packed_2bit's device")
        _check(_lib.mb_dequantize(*[_ptr(a) for a in args], M, K, _ptr(out), _stream(dev)))
    return out



def dequantize_2nd(packed_2bit: torch.Tensor, packed_4bit: torch.Tensor,
                   scales_1st_quant: torch.Tensor, scales_2nd: torch.Tensor,
                   zeros_2nd: torch.Tensor, zeros_1st: torch.Tensor,
                   group_precision: torch.Tensor, M: int, K: int,
                   outlier_row_ptrs: torch.Tensor | None = None,
                   outlier_col_indices: torch.Tensor | None = None,
                   outlier_values: torch.Tensor | None = None,
                   out: torch.Tensor | None = None) -> torch.Tensor:
    """fp16 [M, K] with each group's scale rebuilt from its 4-bit 2nd-order
    code (``mb_dequantize_2nd``); the CSR outliers are written back when
    given (no counterpart in the reference)."""
    if not packed_2bit.is_cuda:
        raise RuntimeError("packed_2bit must be on CUDA")
    M, K = int(M), int(K)
    if M <= 0 or K <= 0:
        raise RuntimeError("M and K must be positive")
    dev = packed_2bit.device
    ng = (K + GROUP_SIZE_1ST - 1) // GROUP_SIZE_1ST
    ng2 = (M * ng + GROUP_SIZE_2ND - 1) // GROUP_SIZE_2ND
    expect = [(packed_2bit, torch.int32, M * ng, "packed_2bit"),
              (packed_4bit, torch.int32, 2 * M * ng, "packed_4bit"),
              (scales_1st_quant, torch.uint8, M * ng, "scales_1st_quant"),
              (scales_2nd, torch.float16, ng2, "scales_2nd"),
              (zeros_2nd, torch.int8, ng2, "zeros_2nd"),
              (zeros_1st, torch.int8, M * ng, "zeros_1st"),
              (group_precision, torch.uint8, ng, "group_precision")]
    nnz = 0 if outlier_values is None else int(outlier_values.numel())
    if nnz > 0:
        if outlier_row_ptrs is None or outlier_col_indices is None:
            raise RuntimeError("outlier_row_ptrs and outlier_col_indices are needed with "
                               "outlier_values")
        expect += [(outlier_row_ptrs, torch.int32, M + 1, "outlier_row_ptrs"),
                   (outlier_col_indices, torch.int32, nnz, "outlier_col_indices"),
                   (outlier_values, torch.float16, nnz, "outlier_values")]
    for t, dt, n, name in expect:
        if t.device != dev:
            raise RuntimeError(f"{name} must be on the same CUDA device as packed_2bit")
        if t.dtype != dt:
            raise RuntimeError(f"{name} must be {str(dt).replace('torch.', '')}")
        if t.numel() < n:
            raise RuntimeError(f"{name} too small for M={M}, K={K}")
    with torch.cuda.device(dev):
        args = [t.contiguous() for t, *_ in expect]
        if out is None:
            out = torch.empty((M, K), dtype=torch.float16, device=dev)
        elif out.dtype != torch.float16 or out.numel() < M * K or not out.is_contiguous() \
                or out.device != dev:
            raise RuntimeError("out must be a contiguous float16 tensor of at least M * K "
                               "values on packed_2bit's device")
        ptrs = [_ptr(a) for a in args] + [None] * (10 - len(args))
        _check(_lib.mb_dequantize_2nd(*ptrs, nnz, M, K, _ptr(out), _stream(dev)))
    return out



def qgemv(packed_2bit: torch.Tensor, packed_4bit: torch.Tensor, scales_1st: torch.Tensor,
          zeros_1st: torch.Tensor, group_precision: torch.Tensor, outlier_row_ptrs: torch.Tensor,
          outlier_col_indices: torch.Tensor, outlier_values: torch.Tensor, M: int, K: int,
          x: torch.Tensor, out: torch.Tensor | None = None) -> torch.Tensor:
    """fp32 [M] = W x from the packed format (``mb_qgemv``); outliers with
    their exact values (pass empty CSR values to leave them out)."""
    if not packed_2bit.is_cuda:
        raise RuntimeError("packed_2bit must be on CUDA")
    M, K = int(M), int(K)
    if M <= 0 or K <= 0:
        raise RuntimeError("M and K must be positive")
    dev = packed_2bit.device
    ng = (K + GROUP_SIZE_1ST - 1) // GROUP_SIZE_1ST
    nnz = int(outlier_values.numel())
    expect = [(packed_2bit, torch.int32, M * ng, "packed_2bit"),
              (packed_4bit, torch.int32, 2 * M * ng, "packed_4bit"),
              (scales_1st, torch.float16, M * ng, "scales_1st"),
              (zeros_1st, torch.int8, M * ng, "zeros_1st"),
              (group_precision, torch.uint8, ng, "group_precision"),
              (outlier_row_ptrs, torch.int32, M + 1, "outlier_row_ptrs"),
              (outlier_col_indices, torch.int32, nnz, "outlier_col_indices"),
              (outlier_values, torch.float16, nnz, "outlier_values"),
              (x, torch.float16, K, "x")]
    for t, dt, n, name in expect:
        if t.device != dev:
            raise RuntimeError(f"{name} must be on the same CUDA device as packed_2bit")
        if t.dtype != dt:
            raise RuntimeError(f"{name} must be {str(dt).replace('torch.', '')}")
        if t.numel() < n:
            raise RuntimeError(f"{name} too small for M={M}, K={K}")
    with torch.cuda.device(dev):
        args = [t.contiguous() for t, *_ in expect]
        if out is None:
            out = torch.empty((M,), dtype=torch.float32, device=dev)
        elif out.dtype != torch.float32 or out.numel() < M or not out.is_contiguous() \
                or out.device != dev:
            raise RuntimeError("out must be a contiguous float32 tensor of at least M values "
                               "on packed_2bit's device")
        p = [_ptr(a) for a in args]
        _check(_lib.mb_qgemv(*p[:6], p[6] if nnz else None, p[7] if nnz else None, nnz, M, K,
                             p[8], _ptr(out), _stream(dev)))
    return out


class QuantizePlan:
    """Preallocated outputs and workspace for repeatedly quantizing [M, K]
    matrices on one device (whole-model loops, benchmarks).

    ``launch`` enqueues phase 1 (every output except the CSR arrays) on the
    current stream without synchronising, then an event.  The outlier count
    goes straight to pinned host memory (page-locked memory is addressable
    from the device under unified addressing, so the kernel writes it there);
    ``finish`` waits for the event only (work enqueued after this plan's
    launch keeps running), reads the count and extracts the CSR arrays.
    Launching several plans before finishing any keeps the GPU busy across
    matrices.  The tensors returned by ``finish`` alias the plan's buffers
    until the next ``launch``.  The fixed arguments of the C call are built
    once, so a launch costs little host time.

    ``stream`` (optional): the plan's work runs there instead of on the
    current stream (after the current stream's work, which produced the
    inputs); independent matrices on different streams overlap one matrix's
    latency-bound selection with another's streaming kernels.
    """

    def __init__(self, M: int, K: int, device=None, stream: torch.cuda.Stream | None = None):
        device = torch.device("cuda", torch.cuda.current_device()) if device is None else torch.device(device)
        self.M, self.K, self.device = M, K, device
        self.stream = stream
        ng = (K + GROUP_SIZE_1ST - 1) // GROUP_SIZE_1ST
        ng2 = (M * ng + GROUP_SIZE_2ND - 1) // GROUP_SIZE_2ND
        e = lambda shape, dt: torch.empty(shape, dtype=dt, device=device)  # noqa: E731
        self.ws = QuantizeWorkspace(M, K, device)
        self.out = [e((M, ng), torch.int32), e((M, 2 * ng), torch.int32), e((M, ng), torch.float16),
                    e((M, ng), torch.int8), e((ng2,), torch.float16), e((ng2,), torch.int8),
                    e((M, ng), torch.uint8), e((ng,), torch.uint8)]
        self.row_ptrs = e((M + 1,), torch.int32)
        self.nnz_host = torch.zeros((1,), dtype=torch.int32).pin_memory()
        self._nnz = self.nnz_host.numpy()
        self.done = torch.cuda.Event()
        self._w = None
        # outputs, row pointers, count, workspace: fixed for the plan's life
        self._fixed = (*(_ptr(t) for t in self.out), _ptr(self.row_ptrs), _ptr(self.nnz_host),
                       _ptr(self.ws.buf), ctypes.c_size_t(self.ws.nbytes))

    def launch(self, weights: torch.Tensor, ratio_4bit: float = 0.1,
               hessian_diag: torch.Tensor | None = None) -> None:
        assert weights.dtype == torch.float16 and weights.is_contiguous()
        assert tuple(weights.shape) == (self.M, self.K) and weights.device == self.device
        h = hessian_diag if (hessian_diag is not None and hessian_diag.numel() > 0
                             and ratio_4bit > 0) else None
        dev = self.device
        cur = torch.cuda.current_stream(dev)
        st = cur
        if self.stream is not None:
            self.stream.wait_stream(cur)
            st = self.stream
        args = (_ptr(weights), self.M, self.K, float(ratio_4bit), _ptr(h),
                0 if h is None else h.numel(), *self._fixed, ctypes.c_void_p(st.cuda_stream))
        if torch.cuda.current_device() == dev.index:
            _check(_lib.mb_quantize(*args))
        else:
            with torch.cuda.device(dev):
                _check(_lib.mb_quantize(*args))
        self.done.record(st)
        self._w = weights

    def finish(self) -> list:
        self.done.synchronize()
        nnz = int(self._nnz[0])
        dev = self.device
        vals = torch.empty((nnz,), dtype=torch.float16, device=dev)
        cols = torch.empty((nnz,), dtype=torch.int32, device=dev)
        if nnz > 0:
            with torch.cuda.device(dev):
                _check(_lib.mb_quantize_extract_outliers(
                    _ptr(self._w), self.M, self.K, _ptr(self.row_ptrs), _ptr(vals), _ptr(cols),
                    _ptr(self.ws.buf), self.ws.nbytes, _stream(dev)))
        return [*self.out, vals, cols, self.row_ptrs]

    def record_on(self, event: torch.cuda.Event) -> None:
        """Record ``event`` on the stream the plan's work runs on."""
        event.record(self.stream if self.stream is not None
                     else torch.cuda.current_stream(self.device))


# ---- GPTQ calibration (models/llama.py) ----

def hessian(x: torch.Tensor, alpha: float = 1.0, out: torch.Tensor | None = None,
            accumulate: bool = False, status: torch.Tensor | None = None) -> torch.Tensor:
    """out = alpha * x^T x, or out += alpha * x^T x with ``accumulate``.

    x: [N, K] fp16 or bf16 CUDA tensor (K a multiple of 8), computed by the
    tcgen05 kernel with fp32 accumulation; out: [K, K] fp32.  ``status``
    (int32 [1], zeroed by the caller) receives bit 0 if a pipeline wait in the
    kernel ran out."""
    if x.dim() != 2:
        raise RuntimeError("x must be 2D [tokens, features]")
    if x.dtype not in (torch.float16, torch.bfloat16):
        raise RuntimeError("x must be float16 or bfloat16")
    if not x.is_cuda:
        raise RuntimeError("x must be on CUDA")
    x = x.contiguous()
    N, K = int(x.size(0)), int(x.size(1))
    dev = x.device
    with torch.cuda.device(dev):
        if out is None:
            if accumulate:
                raise RuntimeError("accumulate needs an output tensor")
            out = torch.empty((K, K), dtype=torch.float32, device=dev)
        if out.dtype != torch.float32 or tuple(out.shape) != (K, K) or not out.is_contiguous() \
                or out.device != dev:
            raise RuntimeError("out must be a contiguous float32 [K, K] tensor on x's device")
        if N == 0:
            if not accumulate:
                out.zero_()
            return out
        _check(_lib.mb_hessian(_ptr(x), N, K, int(x.dtype == torch.bfloat16), float(alpha),
                               int(bool(accumulate)), _ptr(out), _ptr(status), _stream(dev)))
    return out


def gptq_quantize(W: torch.Tensor, Hinv_cho: torch.Tensor, group_precision: torch.Tensor,
                  blocksize: int = 128, scalar_division: int = GPTQ_DIV_RECIPROCAL,
                  out: torch.Tensor | None = None, rows: tuple | None = None) -> torch.Tensor:
    """gptq_quantize of models/llama.py:234-294 on the GPU (fp32 [M, K]);
    with ``rows`` = (r0, r1) only those rows of Q ([r1 - r0, K]), the group
    parameters still taken over all rows of W."""
    if W.dim() != 2 or W.dtype != torch.float32 or not W.is_cuda:
        raise RuntimeError("W must be a 2D float32 CUDA tensor")
    W = W.contiguous()
    M, K = int(W.size(0)), int(W.size(1))
    dev = W.device
    if tuple(Hinv_cho.shape) != (K, K) or Hinv_cho.dtype != torch.float32 \
            or Hinv_cho.device != dev:
        raise RuntimeError("Hinv_cho must be float32 [K, K] on W's device")
    gp = group_precision.to(device=dev, dtype=torch.uint8).contiguous()
    if gp.numel() != K // GROUP_SIZE_1ST:
        raise RuntimeError("group_precision must hold K // 16 entries")
    r0, r1 = (0, M) if rows is None else (int(rows[0]), int(rows[1]))
    with torch.cuda.device(dev):
        hc = Hinv_cho.contiguous()
        if out is None:
            out = torch.empty((r1 - r0, K), dtype=torch.float32, device=dev)
        elif tuple(out.shape) != (r1 - r0, K) or out.dtype != torch.float32 or \
                not out.is_contiguous() or out.device != dev:
            raise RuntimeError("out must be a contiguous float32 [rows, K] tensor on W's device")
        ws = torch.empty(int(_lib.mb_gptq_workspace_size(M, K)), dtype=torch.uint8, device=dev)
        _check(_lib.mb_gptq_quantize_rows(_ptr(W), M, K, r0, r1, _ptr(hc), _ptr(gp),
                                          int(blocksize), int(scalar_division), _ptr(out),
                                          _ptr(ws), ws.numel(), _stream(dev)))
    return out


def exact_sums(weights: torch.Tensor, hessian_diag: torch.Tensor, ratio_4bit: float = 0.5):
    """Every group's sensitivity (the reference's serial fp32 sum) from the
    exact-sum path, and the selection made from them (mb_quantize_exact_sums).
    Returns (sums float32 [ng], group_precision uint8 [ng])."""
    w = weights.to(torch.float16).contiguous()
    h = hessian_diag.to(device=w.device, dtype=torch.float32).contiguous()
    M, K = w.shape
    ng = (K + GROUP_SIZE_1ST - 1) // GROUP_SIZE_1ST
    with torch.cuda.device(w.device):
        ws = QuantizeWorkspace(M, K, w.device)
        sums = torch.empty((ng,), dtype=torch.float32, device=w.device)
        gp = torch.empty((ng,), dtype=torch.uint8, device=w.device)
        _check(_lib.mb_quantize_exact_sums(_ptr(w), M, K, float(ratio_4bit), _ptr(h), h.numel(),
                                           _ptr(sums), _ptr(gp), _ptr(ws.buf), ws.nbytes,
                                           _stream(w.device)))
    return sums, gp


class QuantizeBatch:
    """Quantizes a fixed list of matrices -- a model's weights -- with every
    launch recorded once into a CUDA graph and replayed.

    The batch owns device buffers for the weights (``weights[i]``; refill them
    in place between replays), hessian diagonals, every output, a workspace
    per matrix and CSR arrays with room for ``csr_capacity`` outliers each.
    Consecutive matrices form groups of up to ``per_launch`` (8 at most); each
    group is one ``mb_quantize_csr_many`` call: one launch of each kernel
    (stats, combine, tables, encode, CSR extraction, chained on the device, no
    host round trip) serves all its matrices, so launch and pipeline start-up
    costs are paid once per group.  The groups are spread over ``branches``
    parallel graph branches (largest first, each to the least loaded branch),
    so one group's latency-bound selection overlaps another's streaming.  ``launch`` replays the graph on the current
    stream (a few microseconds of host time for the whole list); ``finish``
    waits for it and returns the reference's 11-tensor list per matrix, views
    into the batch's buffers valid until the next ``launch``.  A matrix with
    more outliers than its capacity is re-extracted into larger arrays in
    ``finish`` (mb_quantize_extract_outliers).
    """

    def __init__(self, weights: list, ratios, hessians: list | None = None, device=None,
                 branches: int = 2, csr_capacity: int | None = None, per_launch: int = 8):
        device = torch.device("cuda", torch.cuda.current_device()) if device is None \
            else torch.device(device)
        self.device = device
        n = len(weights)
        if isinstance(ratios, (int, float)):
            ratios = [float(ratios)] * n
        hessians = [None] * n if hessians is None else list(hessians)
        e = lambda shape, dt: torch.empty(shape, dtype=dt, device=device)  # noqa: E731
        with torch.cuda.device(device):
            self.weights = [w.to(device=device, dtype=torch.float16).contiguous().clone()
                            for w in weights]
            self.hess = [None if (h is None or h.numel() == 0 or r <= 0) else
                         h.to(device=device, dtype=torch.float32).contiguous().clone()
                         for h, r in zip(hessians, ratios)]
            self.ratios = [float(r) for r in ratios]
            self.shapes = [tuple(int(x) for x in w.shape) for w in self.weights]
            self.out, self.ws, self.row_ptrs, self.vals, self.cols, self.cap = [], [], [], [], [], []
            for (M, K) in self.shapes:
                ng = (K + GROUP_SIZE_1ST - 1) // GROUP_SIZE_1ST
                ng2 = (M * ng + GROUP_SIZE_2ND - 1) // GROUP_SIZE_2ND
                self.out.append([e((M, ng), torch.int32), e((M, 2 * ng), torch.int32),
                                 e((M, ng), torch.float16), e((M, ng), torch.int8),
                                 e((ng2,), torch.float16), e((ng2,), torch.int8),
                                 e((M, ng), torch.uint8), e((ng,), torch.uint8)])
                self.ws.append(QuantizeWorkspace(M, K, device))
                self.row_ptrs.append(e((M + 1,), torch.int32))
                cap = max(1024, (M * K) // 256) if csr_capacity is None else int(csr_capacity)
                self.cap.append(cap)
                self.vals.append(e((max(cap, 1),), torch.float16))
                self.cols.append(e((max(cap, 1),), torch.int32))
            self.nnz_dev = torch.zeros((n,), dtype=torch.int32, device=device)
            self.nnz_host = torch.zeros((n,), dtype=torch.int32).pin_memory()
        # groups of consecutive matrices; branches: largest groups first, each
        # to the least loaded branch
        per = max(1, min(8, int(per_launch)))
        self.groups = [list(range(i, min(n, i + per))) for i in range(0, n, per)]
        size = [sum(self.shapes[i][0] * self.shapes[i][1] for i in g) for g in self.groups]
        nb = max(1, min(int(branches), len(self.groups)))
        load = [0] * nb
        self.branch_of = [0] * len(self.groups)
        for gi in sorted(range(len(self.groups)), key=lambda gi: -size[gi]):
            b = min(range(nb), key=lambda b: load[b])
            self.branch_of[gi] = b
            load[b] += size[gi]
        self.nbranch = nb
        self.jobs = [self._job(i) for i in range(n)]
        self.graph = None
        self.done = torch.cuda.Event()

    def kernel_launches(self) -> int:
        """Kernels one replay launches: five (stats, combine, tables, encode,
        CSR extraction) per launch set, formed as mb_quantize_csr_many forms
        them (consecutive matrices with 16 | column groups and the same
        sensitivity pass, 8 at most; any other matrix alone)."""
        def ng(i):
            return (self.shapes[i][1] + GROUP_SIZE_1ST - 1) // GROUP_SIZE_1ST

        def sens(i):
            return self.hess[i] is not None and int(self.ratios[i] * ng(i)) > 0

        sets = 0
        for idx in self.groups:
            i = 0
            while i < len(idx):
                e = i + 1
                if ng(idx[i]) % 16 == 0:
                    while (e < len(idx) and e - i < 8 and ng(idx[e]) % 16 == 0
                           and sens(idx[e]) == sens(idx[i])):
                        e += 1
                sets += 1
                i = e
        return 5 * sets

    def _job(self, i: int) -> QuantizeJob:
        M, K = self.shapes[i]
        h = self.hess[i]
        o = self.out[i]
        return QuantizeJob(
            _ptr(self.weights[i]), M, K, self.ratios[i], _ptr(h), 0 if h is None else h.numel(),
            *(_ptr(t) for t in o), _ptr(self.row_ptrs[i]),
            ctypes.c_void_p(self.nnz_dev.data_ptr() + 4 * i), _ptr(self.vals[i]),
            _ptr(self.cols[i]), self.cap[i], _ptr(self.ws[i].buf), self.ws[i].nbytes)

    def _enqueue(self, gi: int, stream) -> None:
        idx = self.groups[gi]
        arr = (QuantizeJob * len(idx))(*(self.jobs[i] for i in idx))
        _check(_lib.mb_quantize_csr_many(arr, len(idx), ctypes.c_void_p(stream.cuda_stream)))

    def _record(self, main) -> None:
        fork = torch.cuda.Event()
        fork.record(main)
        for st in self.streams:
            st.wait_event(fork)
        for gi in range(len(self.groups)):
            self._enqueue(gi, self.streams[self.branch_of[gi]])
        for st in self.streams:
            main.wait_stream(st)
        self.nnz_host.copy_(self.nnz_dev, non_blocking=True)

    def capture(self) -> None:
        """Record the graph (once; the first call of every kernel runs eagerly
        before it, so one-time set-up stays out of the capture)."""
        with torch.cuda.device(self.device):
            self.streams = [torch.cuda.Stream(self.device) for _ in range(self.nbranch)]
            main = torch.cuda.current_stream(self.device)
            self._record(main)
            torch.cuda.synchronize(self.device)
            self.graph = torch.cuda.CUDAGraph()
            with torch.cuda.graph(self.graph):
                self._record(torch.cuda.current_stream(self.device))
            torch.cuda.synchronize(self.device)

    def launch(self) -> None:
        if self.graph is None:
            self.capture()
        with torch.cuda.device(self.device):
            self.graph.replay()
            self.done.record()

    def finish(self) -> list:
        self.done.synchronize()
        nnz = self.nnz_host.tolist()
        res = []
        for i, (M, K) in enumerate(self.shapes):
            k = int(nnz[i])
            if k > self.cap[i]:
                with torch.cuda.device(self.device):
                    self.cap[i] = k
                    self.vals[i] = torch.empty((k,), dtype=torch.float16, device=self.device)
                    self.cols[i] = torch.empty((k,), dtype=torch.int32, device=self.device)
                    self.jobs[i] = self._job(i)
                    self.graph = None  # the graph holds the old arrays
                    _check(_lib.mb_quantize_extract_outliers(
                        _ptr(self.weights[i]), M, K, _ptr(self.row_ptrs[i]), _ptr(self.vals[i]),
                        _ptr(self.cols[i]), _ptr(self.ws[i].buf), self.ws[i].nbytes,
                        _stream(self.device)))
                    torch.cuda.current_stream(self.device).synchronize()
            res.append([*self.out[i], self.vals[i][:k], self.cols[i][:k], self.row_ptrs[i]])
        return res
