"""``TurboPolarConfig``: the supported-configuration contract.

Same fields, defaults, validation order and error messages as the reference's frozen
dataclass (``rfsn_v11/candidates/turbo_polar_config.py:6-55``), because callers and tests
match on them.  ``to_format()`` maps the key-format fields to the C ABI's ``tp_format``.
"""

from __future__ import annotations

import math
from dataclasses import dataclass, field
from typing import Any, Dict


@dataclass(frozen=True)
class TurboPolarConfig:
    k_angle_bits_level1: int = 4
    k_angle_bits_deep: int = 4
    use_int8_radii: bool = False
    v_bits: int = 8
    block_size: int = 64
    head_dim: int = 128
    qjl_proj_dim: int = 64
    use_qjl: bool = False
    storage_mode: str = "kv_quant"
    seed: int = 42
    split_dim: int = 64
    attention_scale: float = 0.0  # 0 selects 1/sqrt(head_dim)
    num_q_heads: int = 32
    num_kv_heads: int = 8
    metadata: Dict[str, Any] = field(default_factory=dict)

    def __post_init__(self):
        checks = (
            (self.block_size <= 0, "block_size must be positive"),
            (self.head_dim <= 0, "head_dim must be positive"),
            (self.head_dim % 2 != 0, "head_dim must be divisible by 2 for polar pair coordinate mapping"),
            (self.qjl_proj_dim <= 0, "qjl_proj_dim must be positive"),
            (self.qjl_proj_dim % 8 != 0, "qjl_proj_dim must be divisible by 8 for bit packing"),
            (self.v_bits != 8, "v_bits must be 8 (4-bit V quantization is not yet implemented)"),
            (self.storage_mode not in {"k_only_first", "kv_quant", "dense_v_debug"}, "unknown storage_mode"),
            (self.block_size != 64, "TurboPolar only supports block_size == 64 in this release"),
            (self.head_dim != 128, "TurboPolar only supports head_dim == 128 in this release"),
            (self.use_qjl, "QJL is not supported in this release; set use_qjl=False"),
            (self.storage_mode != "kv_quant", "TurboPolar only supports storage_mode='kv_quant' in this release"),
            (self.split_dim < 0 or self.split_dim > self.head_dim or self.split_dim % 2 != 0,
             "split_dim must be even and within [0, head_dim]"),
            (self.num_q_heads % self.num_kv_heads != 0, "num_q_heads must be divisible by num_kv_heads for GQA"),
        )
        for bad, msg in checks:
            if bad:
                raise ValueError(msg)
        if self.attention_scale == 0.0:
            object.__setattr__(self, "attention_scale", 1.0 / math.sqrt(self.head_dim))

    @property
    def num_queries_per_kv(self) -> int:
        return self.num_q_heads // self.num_kv_heads

    def format_fields(self) -> dict:
        return dict(l1_bits=int(self.k_angle_bits_level1), deep_bits=int(self.k_angle_bits_deep),
                    split_dim=int(self.split_dim), int8_radii=int(bool(self.use_int8_radii)))
