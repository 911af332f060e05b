"""GPTQ oracle in torch -- TEST INFRASTRUCTURE ONLY.

A restatement of the reference's gptq_quantize (models/llama.py:234-294) that
evaluates every step with the same torch tensor operations and Python-float
scalars as the reference, column by column.  Run on CPU tensors it gives the
reference's CPU result (pinned by tests/golden/gptq_*.npz); run on CUDA
tensors it gives what the reference computes on a GPU, where PyTorch divides
a tensor by a Python float as a multiplication by the fp32 reciprocal.  Only
the tests use it, as the checker of the sm_100a kernel's two division modes.
"""
from __future__ import annotations

import torch

GROUP = 16


def group_parameters(W: torch.Tensor, group_precision: torch.Tensor):
    """Per-group (levels, fp32 min, fp32 scale) -- llama.py:248-263: min/max
    as Python floats via .item(), scale (gmax - gmin) / (L - 1) in Python
    arithmetic stored into an fp32 tensor, 0.0 unless gmax > gmin."""
    ng = W.shape[1] // GROUP
    levels = [16 if int(p) == 1 else 4 for p in group_precision.cpu().tolist()]
    lo = torch.zeros(ng, device=W.device)
    scale = torch.zeros(ng, device=W.device)
    for g in range(ng):
        block = W[:, g * GROUP:(g + 1) * GROUP]
        mn, mx = block.min().item(), block.max().item()
        lo[g] = mn
        scale[g] = (mx - mn) / (levels[g] - 1) if mx > mn else 0.0
    return levels, lo, scale


def gptq_quantize(W: torch.Tensor, hinv_cho: torch.Tensor, group_precision: torch.Tensor,
                  blocksize: int = 128) -> torch.Tensor:
    """Q (fp32 [M, K]) by the reference's column loop, on W's device."""
    K = W.shape[1]
    levels, lo, scale = group_parameters(W, group_precision)
    Q = W.clone()
    for b0 in range(0, K, blocksize):
        b1 = min(b0 + blocksize, K)
        work = Q[:, b0:b1].clone()          # the block before any of it is written
        for j in range(b1 - b0):
            c = b0 + j
            g = c // GROUP
            gmin = lo[g].item()
            sc = scale[g].item()
            col = work[:, j]
            if sc > 0:
                q_int = ((col - gmin) / sc).round().clamp(0, levels[g] - 1)
                q = sc * (q_int - round(-gmin / sc))
            else:
                q = torch.full_like(col, gmin)
            err = (col - q) / hinv_cho[c, c]
            Q[:, c] = q
            if j + 1 < b1 - b0:
                work[:, j + 1:] -= err.unsqueeze(1) * hinv_cho[c, c + 1:b1].unsqueeze(0)
    return Q


def equal_up_to_zero_sign(a: torch.Tensor, b: torch.Tensor) -> bool:
    """Bitwise equality, except that +0.0 and -0.0 compare equal (the sign of
    an exact zero from clamp(-0.0, 0, L-1) depends on the min/max
    instruction) and NaN matches NaN."""
    if a.shape != b.shape:
        return False
    a, b = a.detach().float().cpu(), b.detach().float().cpu()
    nan_a, nan_b = torch.isnan(a), torch.isnan(b)
    if not torch.equal(nan_a, nan_b):
        return False
    return bool(torch.equal(a[~nan_a], b[~nan_b]))
