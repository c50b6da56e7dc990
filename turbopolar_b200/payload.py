"""Payload containers with the reference's field names, holding CUDA tensors.

``PolarKeyBlock`` mirrors ``rfsn_v11/quant/polar/payload.py:6-15`` and ``QuantizedVBlock``
mirrors ``rfsn_v11/quant/v_quant/encoder.py:5-9``.  Unified shapes are ``(B, H, S, 64, .)``;
single-block payloads drop the ``S`` axis.
"""

from __future__ import annotations

from dataclasses import dataclass, field
from typing import Any, Dict, Optional, Tuple

import torch


@dataclass
class PolarKeyBlock:
    radii: torch.Tensor
    angle_codes_l1: torch.Tensor
    angle_codes_deep: torch.Tensor
    shape: Tuple[int, ...]
    block_size: int
    head_dim: int
    metadata: Dict[str, Any]
    radii_scales: Optional[torch.Tensor] = field(default=None)


@dataclass(frozen=True)
class QuantizedVBlock:
    codes: torch.Tensor
    scales: torch.Tensor
    group_size: int


def block_metadata(fmt: dict, block_size: int = 64, head_dim: int = 128) -> Dict[str, Any]:
    """The metadata dict the reference encoder attaches (``encoder.py:85-97``)."""
    split_half = fmt["split_dim"] // 2
    return {
        "l1_scale": float(2 ** fmt["l1_bits"] - 1),
        "deep_scale": float(2 ** fmt["deep_bits"] - 1),
        "split_dim": fmt["split_dim"],
        "l1_packed": fmt["l1_bits"] == 4,
        "deep_packed": fmt["deep_bits"] in (2, 4),
        "deep_bits": fmt["deep_bits"],
        "l1_bits": fmt["l1_bits"],
        "int8_radii": bool(fmt["int8_radii"]),
        "log_radii": bool(fmt["int8_radii"]),
        "l1_original_len": split_half,
        "deep_original_len": head_dim // 2 - split_half,
    }


def format_of_metadata(md: Dict[str, Any], radii: torch.Tensor) -> dict:
    """Inverse of :func:`block_metadata` for a payload handed in by a caller."""
    return dict(l1_bits=int(md.get("l1_bits", 4)), deep_bits=int(md.get("deep_bits", 2)),
                split_dim=int(md.get("split_dim", 64)), int8_radii=int(radii.dtype == torch.int8))
