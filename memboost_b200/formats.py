"""QuantizedTensor -- the output format of memboost.quantize.

The field set, dtypes, shapes, size accounting and state_dict keys are the
reference's (memboost/formats.py:11-202), kept identical so quantized
checkpoints and code written against memboost read the same way:

  packed_2bit        int32 [M, ng]       16 codes per word (zeros for 4-bit groups)
  packed_4bit        int32 [M, 2*ng]     8 codes per word  (zeros for 2-bit groups)
  scales_1st         fp16  [M, ng]
  zeros_1st          int8  [M, ng]
  scales_2nd         fp16  [ng2]
  zeros_2nd          int8  [ng2]
  scales_1st_quant   uint8 [M, ng]
  group_precision    uint8 [ng]          0 = 2-bit, 1 = 4-bit
  outlier_values     fp16  [nnz]         CSR
  outlier_col_indices int32 [nnz]
  outlier_row_ptrs   int32 [M+1]
with ng = ceil(K/16) and ng2 = ceil(M*ng/256).
"""
from __future__ import annotations

from dataclasses import dataclass

import torch

GROUP_SIZE_1ST = 16   # columns per 1st-order group (memboost/formats.py:7)
GROUP_SIZE_2ND = 256  # scales per 2nd-order group  (memboost/formats.py:8)

# compact_state_dict(): packed arrays hold only each group's own words
PACKED_LAYOUT_KEY = "packed_layout"

_TENSOR_FIELDS = (
    "packed_2bit", "packed_4bit", "scales_1st", "zeros_1st", "scales_2nd", "zeros_2nd",
    "scales_1st_quant", "group_precision", "outlier_values", "outlier_col_indices",
    "outlier_row_ptrs",
)


@dataclass
class QuantizedTensor:
    """All packed components of one quantized [M, K] weight matrix."""

    packed_2bit: torch.Tensor
    packed_4bit: torch.Tensor
    scales_1st: torch.Tensor
    zeros_1st: torch.Tensor
    scales_2nd: torch.Tensor
    zeros_2nd: torch.Tensor
    scales_1st_quant: torch.Tensor
    group_precision: torch.Tensor
    outlier_values: torch.Tensor
    outlier_col_indices: torch.Tensor
    outlier_row_ptrs: torch.Tensor
    M: int = 0
    K: int = 0

    @property
    def num_groups(self) -> int:
        return (self.K + GROUP_SIZE_1ST - 1) // GROUP_SIZE_1ST

    @property
    def nnz(self) -> int:
        return self.outlier_values.numel()

    @property
    def num_2bit_groups(self) -> int:
        return int((self.group_precision == 0).sum().item())

    @property
    def num_4bit_groups(self) -> int:
        return int((self.group_precision == 1).sum().item())

    @property
    def avg_bits(self) -> float:
        """Approximate bits per weight (memboost/formats.py:60-72): 2 or 4
        bits per code, 6 bits of scale/zero per 16-code group, 32 bits per
        outlier."""
        total = self.M * self.K
        if total == 0:
            return 0.0
        n2 = self.num_2bit_groups * GROUP_SIZE_1ST * self.M
        n4 = self.num_4bit_groups * GROUP_SIZE_1ST * self.M
        bits = n2 * 2.0 + n4 * 4.0 + (n2 + n4) / GROUP_SIZE_1ST * 6 + self.nnz * 32
        return bits / total

    def _used_packed_bytes(self) -> tuple[int, int]:
        return self.num_2bit_groups * self.M * 4, self.num_4bit_groups * self.M * 8

    @property
    def total_bytes(self) -> int:
        """Footprint counting only the packed words of each group's own
        precision (memboost/formats.py:74-95)."""
        p2, p4 = self._used_packed_bytes()
        rest = sum(getattr(self, f).nbytes for f in _TENSOR_FIELDS[2:])
        return p2 + p4 + rest

    @property
    def gpu_bytes(self) -> int:
        """Bytes actually allocated, unused packed words included
        (memboost/formats.py:97-112)."""
        return sum(getattr(self, f).nbytes for f in _TENSOR_FIELDS)

    @property
    def total_mb(self) -> float:
        return self.total_bytes / (1024 * 1024)

    def memory_breakdown(self) -> dict[str, float]:
        """Per-component MiB, printed largest first (memboost/formats.py:119-143)."""
        p2, p4 = self._used_packed_bytes()
        comp = {"packed_2bit": p2, "packed_4bit": p4}
        for f in _TENSOR_FIELDS[2:]:
            comp[f] = getattr(self, f).nbytes
        mib = {k: v / (1024 * 1024) for k, v in comp.items()}
        for name, size in sorted(mib.items(), key=lambda kv: -kv[1]):
            print(f"  {name:25s} {size:8.3f} MiB")
        total = sum(mib.values())
        print(f"  {'TOTAL':25s} {total:8.3f} MiB")
        gpu_mib = self.gpu_bytes / (1024 * 1024)
        if gpu_mib > total + 0.001:
            print(f"  {'GPU allocated':25s} {gpu_mib:8.3f} MiB")
        return mib

    @property
    def device(self) -> torch.device:
        return self.packed_2bit.device

    def to(self, device) -> "QuantizedTensor":
        return QuantizedTensor(**{f: getattr(self, f).to(device) for f in _TENSOR_FIELDS},
                               M=self.M, K=self.K)

    def state_dict(self) -> dict:
        """Same keys and tensors as memboost/formats.py:167-184 (M, K as 0-d tensors)."""
        d = {f: getattr(self, f) for f in _TENSOR_FIELDS}
        d["M"] = torch.tensor(self.M)
        d["K"] = torch.tensor(self.K)
        return d

    def compact_state_dict(self) -> dict:
        """state_dict() without the packed words of the other precision:
        ``packed_2bit`` keeps the words of the 2-bit groups ([M, n2]) and
        ``packed_4bit`` the two words of each 4-bit group ([M, 2 n4]), both in
        group order, marked by ``packed_layout`` = 1.  The packed bytes are
        the ones ``total_bytes`` counts; the omitted words are zero by
        construction, so ``from_state_dict`` restores the arrays exactly."""
        M, ng = self.M, self.num_groups
        four = self.group_precision[:ng].to(torch.bool)
        idx2 = torch.nonzero(~four).flatten()
        idx4 = torch.nonzero(four).flatten()
        d = self.state_dict()
        d["packed_2bit"] = self.packed_2bit.reshape(M, ng).index_select(1, idx2).contiguous()
        d["packed_4bit"] = (self.packed_4bit.reshape(M, ng, 2).index_select(1, idx4)
                            .reshape(M, 2 * idx4.numel()).contiguous())
        d[PACKED_LAYOUT_KEY] = torch.tensor(1)
        return d

    @classmethod
    def from_state_dict(cls, d: dict) -> "QuantizedTensor":
        """From ``state_dict()`` (the reference's keys) or
        ``compact_state_dict()``."""
        M, K = int(d["M"].item()), int(d["K"].item())
        fields = {f: d[f] for f in _TENSOR_FIELDS}
        if PACKED_LAYOUT_KEY in d and int(d[PACKED_LAYOUT_KEY].item()) == 1:
            ng = (K + GROUP_SIZE_1ST - 1) // GROUP_SIZE_1ST
            four = fields["group_precision"][:ng].to(torch.bool)
            idx2 = torch.nonzero(~four).flatten()
            idx4 = torch.nonzero(four).flatten()
            dev = fields["packed_2bit"].device
            p2 = torch.zeros((M, ng), dtype=torch.int32, device=dev)
            p4 = torch.zeros((M, ng, 2), dtype=torch.int32, device=dev)
            p2[:, idx2.to(dev)] = fields["packed_2bit"].reshape(M, idx2.numel())
            p4[:, idx4.to(dev)] = fields["packed_4bit"].reshape(M, idx4.numel(), 2)
            fields["packed_2bit"] = p2
            fields["packed_4bit"] = p4.reshape(M, 2 * ng)
        return cls(**fields, M=M, K=K)
