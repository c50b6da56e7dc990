"""Deterministic inputs of the golden fixtures (``numpy.random.default_rng``, PCG64).

Shared by ``make_golden.py`` (which ran the reference on them) and the tests (which rebuild
them instead of storing them in the fixture file).
"""

from __future__ import annotations

import numpy as np

CODEC_CASES = {
    # name: (TurboPolarConfig overrides, input dtype, seed)
    "default_f16": ({}, np.float16, 10),
    "default_f32": ({}, np.float32, 11),
    "adapter_f16": (dict(use_int8_radii=True, k_angle_bits_deep=8, split_dim=0), np.float16, 12),
    "adapter_f32": (dict(use_int8_radii=True, k_angle_bits_deep=8, split_dim=0), np.float32, 13),
    "l1x8_deep2_split32_f16": (dict(k_angle_bits_level1=8, k_angle_bits_deep=2, split_dim=32), np.float16, 14),
    "l1x4_deep8_split128_f16": (dict(k_angle_bits_deep=8, split_dim=128), np.float16, 15),
    "int8radii_default_f16": (dict(use_int8_radii=True), np.float16, 16),
}

SHAPE_TS = (1, 32, 63, 64, 65, 127, 128, 129)
GROWTH_TS = (1, 70, 5, 64, 200, 63, 1, 300)
ADAPTER_CASES = {
    "int8": dict(use_int8_radii=True),
    "adapter_fmt": dict(use_int8_radii=True, k_angle_bits_deep=8, split_dim=0),
}
ADAPTER_STEPS = 130


def channel_scale() -> np.ndarray:
    """Fixed per-channel scale ~ U(0.5, 4) that mimics key-channel outliers (seed 1)."""
    return np.random.default_rng(1).uniform(0.5, 4.0, size=128).astype(np.float32)


def codec_inputs(name: str):
    """One 64-token block ``(1,4,64,128)`` of K and V, with special values planted in
    head 0: axis points, signed zeros, a tiny and a large pair, and an all-zero V group."""
    _, dtype, seed = CODEC_CASES[name]
    rng = np.random.default_rng(seed)
    k = (rng.standard_normal((1, 4, 64, 128)).astype(np.float32) * channel_scale()).astype(dtype)
    v = rng.standard_normal((1, 4, 64, 128)).astype(dtype)
    k[0, 0, 0, :16] = np.array([0, 0, -0.0, 0, 1, 0, -1, 0, 0, 1, 0, -1, -1, -0.0, 3e-5, -2e-5], dtype)
    k[0, 0, 1, :4] = np.array([200.0, -150.0, -0.5, 0.5], dtype)
    v[0, 0, 0, :32] = 0
    return k, v


def c1_inputs():
    """README case (config 1): 100 tokens of K and V ``(1,4,1,128)`` fp16 and a query
    ``(1,8,128)`` fp16, all N(0,1) from seed 0."""
    rng = np.random.default_rng(0)
    ks = rng.standard_normal((100, 1, 4, 1, 128)).astype(np.float16)
    vs = rng.standard_normal((100, 1, 4, 1, 128)).astype(np.float16)
    q = rng.standard_normal((1, 8, 128)).astype(np.float16)
    return ks, vs, q


def shape_inputs(t: int, gqa: int):
    h = 4 // gqa
    rng = np.random.default_rng(100 + t * 10 + gqa)
    k = rng.standard_normal((1, h, t, 128)).astype(np.float32)
    v = rng.standard_normal((1, h, t, 128)).astype(np.float32)
    return k, v


def growth_inputs():
    rng = np.random.default_rng(5)
    out = []
    for t in GROWTH_TS:
        k = rng.standard_normal((1, 2, t, 128)).astype(np.float16)
        v = rng.standard_normal((1, 2, t, 128)).astype(np.float16)
        out.append((k, v))
    return out


def adapter_inputs():
    rng = np.random.default_rng(2026)
    n = ADAPTER_STEPS
    qs = rng.standard_normal((n, 1, 4, 1, 128)).astype(np.float16)
    ks = rng.standard_normal((n, 1, 2, 1, 128)).astype(np.float16)
    vs = rng.standard_normal((n, 1, 2, 1, 128)).astype(np.float16)
    return qs, ks, vs


def prefill_inputs():
    rng = np.random.default_rng(77)
    kp = rng.standard_normal((1, 2, 100, 128)).astype(np.float16)
    vp = rng.standard_normal((1, 2, 100, 128)).astype(np.float16)
    kp2 = rng.standard_normal((1, 2, 30, 128)).astype(np.float16)
    vp2 = rng.standard_normal((1, 2, 30, 128)).astype(np.float16)
    return kp, vp, kp2, vp2


DENSE_V_CASES = {
    # name: (TurboPolarConfig overrides, seed); 8 query / 2 KV heads, 192 tokens (3 pages)
    "default": ({}, 31),
    "adapter_fmt": (dict(use_int8_radii=True, k_angle_bits_deep=8, split_dim=0), 32),
}
DENSE_V_LENGTHS = (192, 150, 70)


def dense_v_inputs(name: str):
    """K ``(1,2,192,128)`` fp16 (N(0,1) times the channel scale), V ``(1,2,192,128)`` fp16 and a
    query ``(1,8,128)`` fp16, N(0,1)."""
    _, seed = DENSE_V_CASES[name]
    rng = np.random.default_rng(seed)
    k = (rng.standard_normal((1, 2, 192, 128)).astype(np.float32) * channel_scale()).astype(np.float16)
    v = rng.standard_normal((1, 2, 192, 128)).astype(np.float16)
    q = rng.standard_normal((1, 8, 128)).astype(np.float16)
    return k, v, q
