"""Grouped int8 value codec restated in NumPy (oracle; test infrastructure only).

Follows ``rfsn_v11/quant/v_quant/encoder.py:16-38``: groups of 32 channels, scale
``max|v|/127`` stored as float16 with a zero scale replaced by float16(1e-4), codes
``clip(round(v / scale), -128, 127)``.  For float16 input the division by the scale rounds
to float16 before the half-to-even round (every MLX op runs in the input dtype).
"""

from __future__ import annotations

import numpy as np

GROUP = 32


def quantize(v: np.ndarray):
    """``(..., 128)`` float16/float32 values -> (int8 codes ``(..., 128)``, float16 scales
    ``(..., 4)``)."""
    v = np.asarray(v)
    dt = v.dtype
    if dt not in (np.float16, np.float32):
        raise ValueError("quantize expects float16 or float32 values")
    g = v.reshape(v.shape[:-1] + (v.shape[-1] // GROUP, GROUP))
    max_abs = np.max(np.abs(g), axis=-1, keepdims=True)
    scales = (max_abs / dt.type(127.0)).astype(dt).astype(np.float16)
    scales = np.where(scales == 0, np.float16(1e-4), scales).astype(np.float16)
    if dt == np.float16:
        ratio = (g / scales).astype(np.float16)
    else:
        ratio = (g / scales.astype(np.float32)).astype(np.float32)
    codes = np.clip(np.round(ratio), -128, 127).astype(np.int8)
    return codes.reshape(v.shape), scales[..., 0]


def dequantize(codes: np.ndarray, scales: np.ndarray) -> np.ndarray:
    """``codes * scale`` in float32, stored as float16 (``encoder.py:32-38``)."""
    codes = np.asarray(codes)
    g = codes.reshape(codes.shape[:-1] + (codes.shape[-1] // GROUP, GROUP)).astype(np.float32)
    out = (g * np.asarray(scales)[..., None].astype(np.float32)).astype(np.float32)
    return out.reshape(codes.shape).astype(np.float16)
