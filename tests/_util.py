"""Shared test helpers (seeded synthetic inputs, oracle adapters)."""

import numpy as np

from oracle import attention as oatt
from oracle import polar, vquant

ATOL = 2e-3  # attention outputs: max-abs error in fp16 against the float64 oracle


def kv_inputs(seed: int, heads: int, t: int, dtype=np.float16, channel_scaled: bool = True):
    """K ~ N(0,1) * c (c a fixed per-channel U(0.5,4) vector, seed 1) and V ~ N(0,1): the
    synthetic distribution of the benchmark configurations."""
    rng = np.random.default_rng(seed)
    k = rng.standard_normal((1, heads, t, 128)).astype(np.float32)
    if channel_scaled:
        k = k * np.random.default_rng(1).uniform(0.5, 4.0, size=128).astype(np.float32)
    v = rng.standard_normal((1, heads, t, 128)).astype(np.float32)
    return k.astype(dtype), v.astype(dtype)


def oracle_cache(k: np.ndarray, v: np.ndarray, fmt: dict, int8_radii: bool):
    """Pages (reference unified shapes without B) and tail for keys/values ``(1,H,T,128)``."""
    t = k.shape[2]
    n = t // 64
    pages = None
    if n:
        kb = k[0, :, :n * 64].reshape(k.shape[1], n, 64, 128)
        vb = v[0, :, :n * 64].reshape(v.shape[1], n, 64, 128)
        enc = polar.encode_block(kb, int8_radii=int8_radii, **fmt)
        codes, scales = vquant.quantize(vb)
        pages = dict(radii=enc["radii"], angle_codes_l1=enc["angle_codes_l1"], angle_codes_deep=enc["angle_codes_deep"],
                     radii_scales=None if enc["radii_scales"] is None else enc["radii_scales"][..., 0, 0],
                     v_codes=codes, v_scales=scales)
    tail_k = k[0, :, n * 64:]
    tail_v = v[0, :, n * 64:]
    return pages, tail_k, tail_v


def oracle_attention(q: np.ndarray, k: np.ndarray, v: np.ndarray, fmt: dict, int8_radii: bool, scale: float,
                     seq_len=None):
    pages, tk, tv = oracle_cache(k, v, fmt, int8_radii)
    seq = k.shape[2] if seq_len is None else seq_len
    # The kernels read queries as float16 (like the reference's Metal kernels).
    q16 = np.asarray(q, np.float16).astype(np.float64)
    return oatt.attention_dense_tail(q16, pages, fmt, tk.astype(np.float64), tv.astype(np.float64), seq, scale)


def fmt_of(cfg) -> dict:
    return dict(l1_bits=cfg.k_angle_bits_level1, deep_bits=cfg.k_angle_bits_deep, split_dim=cfg.split_dim)
