"""memboost_b200 -- memboost's mixed 2/4-bit weight quantization hot path,
rebuilt for NVIDIA B200 (sm_100a).

Drop-in for the reference package: ``import memboost_b200 as memboost``
exposes the same API (quantize, dequantize, pack/unpack, QuantizedTensor,
GROUP_SIZE_1ST / GROUP_SIZE_2ND) with bit-identical results.
"""
__version__ = "0.1.0"

from .checkpoint import load_quantized, save_quantized
from .formats import GROUP_SIZE_1ST, GROUP_SIZE_2ND, QuantizedTensor
from .ops import (dequantize, dequantize_2nd_order, pack_2bit, pack_4bit, qgemv, quantize,
                  unpack_2bit, unpack_4bit)

__all__ = [
    "QuantizedTensor",
    "GROUP_SIZE_1ST",
    "GROUP_SIZE_2ND",
    "pack_2bit",
    "unpack_2bit",
    "pack_4bit",
    "unpack_4bit",
    "quantize",
    "dequantize",
    "dequantize_2nd_order",
    "save_quantized",
    "load_quantized",
    "qgemv",
]
