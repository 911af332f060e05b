"""Public memboost operations (memboost/ops.py:8-135), running on the
sm_100a kernels of libmemboost_b200.so."""
from __future__ import annotations

from typing import Optional

import torch

from . import _C
from .formats import QuantizedTensor


def pack_2bit(values: torch.Tensor) -> torch.Tensor:
    """Pack a 1-D uint8 tensor of 2-bit values (length % 16 == 0) into int32
    words, 16 values per word.  Returns a CPU tensor, as the reference."""
    return _C.pack_2bit(values)


def unpack_2bit(packed: torch.Tensor, num_elements: int) -> torch.Tensor:
    """Inverse of pack_2bit: the first ``num_elements`` values as CPU uint8."""
    return _C.unpack_2bit(packed, num_elements)


def pack_4bit(values: torch.Tensor) -> torch.Tensor:
    """Pack a 1-D uint8 tensor of 4-bit values (length % 8 == 0) into int32
    words, 8 values per word.  Returns a CPU tensor, as the reference."""
    return _C.pack_4bit(values)


def unpack_4bit(packed: torch.Tensor, num_elements: int) -> torch.Tensor:
    """Inverse of pack_4bit: the first ``num_elements`` values as CPU uint8."""
    return _C.unpack_4bit(packed, num_elements)


def quantize(weights: torch.Tensor, ratio_4bit: float = 0.1,
             hessian_diag: Optional[torch.Tensor] = None,
             workspace: Optional[_C.QuantizeWorkspace] = None) -> QuantizedTensor:
    """Quantize an fp16 [M, K] CUDA matrix to mixed 2/4-bit precision.

    Per 16-column group: range-aware min/max scale and zero, 2-bit codes (or
    4-bit for the ``int(ratio_4bit * ng)`` groups with the largest
    hessian-weighted sensitivity when ``hessian_diag`` [K] fp32 CUDA is
    given), 2nd-order 4-bit quantization of the scales, and CSR extraction of
    weights whose dequantization error exceeds the group threshold.  Results
    are bit-identical to the reference implementation.  ``workspace`` may be
    passed to reuse device scratch across calls of the same shape.
    """
    t = _C.quantize(weights, ratio_4bit, hessian_diag, workspace)
    M, K = weights.shape
    return QuantizedTensor(
        packed_2bit=t[0], packed_4bit=t[1], scales_1st=t[2], zeros_1st=t[3], scales_2nd=t[4],
        zeros_2nd=t[5], scales_1st_quant=t[6], group_precision=t[7], outlier_values=t[8],
        outlier_col_indices=t[9], outlier_row_ptrs=t[10], M=int(M), K=int(K))


def dequantize(qtensor: QuantizedTensor, out: Optional[torch.Tensor] = None) -> torch.Tensor:
    """fp16 [M, K] from the 1st-order codes, scales and zeros:
    ``w = scale * (q - zero)``.  Sparse outliers are not added back (as in
    the reference); they remain in the CSR fields."""
    return _C.dequantize(qtensor.packed_2bit, qtensor.packed_4bit, qtensor.scales_1st,
                         qtensor.zeros_1st, qtensor.group_precision, qtensor.M, qtensor.K, out)


def dequantize_2nd_order(qtensor: QuantizedTensor, add_outliers: bool = True,
                         out: Optional[torch.Tensor] = None) -> torch.Tensor:
    """fp16 [M, K] as a consumer of the compact format sees it: each group's
    scale is rebuilt from its 4-bit code ``scales_1st_quant`` with the
    256-group chunk's ``scales_2nd`` / ``zeros_2nd``
    (``s = scales_2nd * (q2 - zeros_2nd)`` in fp16), then ``w = s * (q -
    zero)``; with ``add_outliers`` the CSR outliers are written back.  The
    reference computes these fields but has no function that reads them."""
    nnz = int(qtensor.outlier_values.numel()) if add_outliers else 0
    return _C.dequantize_2nd(
        qtensor.packed_2bit, qtensor.packed_4bit, qtensor.scales_1st_quant, qtensor.scales_2nd,
        qtensor.zeros_2nd, qtensor.zeros_1st, qtensor.group_precision, qtensor.M, qtensor.K,
        qtensor.outlier_row_ptrs if nnz else None, qtensor.outlier_col_indices if nnz else None,
        qtensor.outlier_values if nnz else None, out)


def qgemv(qtensor: QuantizedTensor, x: torch.Tensor, add_outliers: bool = True,
          out: Optional[torch.Tensor] = None) -> torch.Tensor:
    """fp32 [M] = W x straight from the packed format: W as ``dequantize``
    gives it, and with ``add_outliers`` every outlier's exact value in place
    of its code's.  The matrix is never expanded in memory.  The reference
    has no matmul over its format."""
    vals = qtensor.outlier_values if add_outliers else qtensor.outlier_values[:0]
    cols = qtensor.outlier_col_indices if add_outliers else qtensor.outlier_col_indices[:0]
    return _C.qgemv(qtensor.packed_2bit, qtensor.packed_4bit, qtensor.scales_1st,
                    qtensor.zeros_1st, qtensor.group_precision, qtensor.outlier_row_ptrs, cols,
                    vals, qtensor.M, qtensor.K, x.reshape(-1), out)
