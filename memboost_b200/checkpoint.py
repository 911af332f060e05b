"""Quantized checkpoints on disk.

``save_quantized`` writes what the reference's model driver writes
(models/llama.py:686-693): one ``torch.save`` file holding
``{layer name: QuantizedTensor.state_dict()}`` plus metadata entries whose
names start with ``_`` (``_stats``, ``_model_name``, ``_ratio_4bit``).  With
``compact=True`` each layer is stored as ``compact_state_dict()`` instead:
only the packed words of each group's own precision, about half the packed
bytes at 10% 4-bit groups.  ``load_quantized`` reads both layouts (and
files written by the reference).
"""
from __future__ import annotations

import os
from typing import Any

import torch

from .formats import QuantizedTensor


def save_quantized(layers: dict[str, QuantizedTensor], path: str | os.PathLike,
                   compact: bool = False, **metadata: Any) -> None:
    """Write ``layers`` and ``metadata`` (keys given without or with the
    leading ``_``) to ``path`` with ``torch.save``."""
    out: dict[str, Any] = {}
    for name, qt in layers.items():
        if name.startswith("_"):
            raise ValueError(f"layer names must not start with '_': {name!r}")
        out[name] = qt.compact_state_dict() if compact else qt.state_dict()
    for k, v in metadata.items():
        out[k if k.startswith("_") else "_" + k] = v
    torch.save(out, path)


def load_quantized(path: str | os.PathLike, map_location=None
                   ) -> tuple[dict[str, QuantizedTensor], dict[str, Any]]:
    """Read a file written by ``save_quantized`` or by the reference's
    driver: (layers, metadata)."""
    d = torch.load(path, map_location=map_location, weights_only=False)
    layers = {k: QuantizedTensor.from_state_dict(v) for k, v in d.items()
              if not k.startswith("_")}
    meta = {k: v for k, v in d.items() if k.startswith("_")}
    return layers, meta
