"""Polar key codec restated in NumPy (oracle; test infrastructure only).

Follows ``rfsn_v11/quant/polar/encoder.py:24-130`` (encode, 4-bit / 2-bit packing) and
``rfsn_v11/quant/polar/decoder.py:7-85`` (decode, unpacking).

Per-op rounding: the reference encoder runs every op in the input dtype.  For float16 input
that means ``x*x``, ``y*y``, their sum, ``sqrt``, ``atan2``, ``+ pi`` and ``/ 2pi`` each round
to float16, with the constants themselves rounded to float16 first (pi -> 3.140625,
2pi -> 6.28125, 1-1e-6 -> 1.0).  The ``mx.where(..., mx.array(0.0), ...)`` at
``encoder.py:50-51`` promotes the normalised angle to float32 (``mx.array(0.0)`` is a
float32 scalar), so the multiply by ``2**bits - 1`` and the half-to-even round happen in
float32.  Transcendentals are modelled as a correctly rounded float32 libm (float64
evaluation rounded to float32) followed by the store in the working dtype.
"""

from __future__ import annotations

import numpy as np

HEAD_DIM = 128
BLOCK = 64
PAIRS = HEAD_DIM // 2


def _cr32(fn, *args, dtype):
    """Correctly rounded float32 evaluation of ``fn``, stored in ``dtype``."""
    r = fn(*[np.asarray(a, dtype=np.float64) for a in args])
    return r.astype(np.float32).astype(dtype)


def packed_len(n_codes: int, bits: int) -> int:
    """Bytes per token row for ``n_codes`` angle codes of ``bits`` bits
    (``tests/benchmarks/test_turbo_polar_offline.py:26-34``)."""
    if bits == 8:
        return n_codes
    per = 8 // bits
    return (n_codes + per - 1) // per


def pack_4bit(codes: np.ndarray) -> np.ndarray:
    """Even index -> low nibble, odd -> high nibble (``encoder.py:100-113``)."""
    n = codes.shape[-1]
    if n % 2:
        codes = np.concatenate([codes, np.zeros(codes.shape[:-1] + (1,), np.uint8)], axis=-1)
    return ((codes[..., 0::2] & 0x0F) | ((codes[..., 1::2] & 0x0F) << 4)).astype(np.uint8)


def pack_2bit(codes: np.ndarray) -> np.ndarray:
    """Four codes per byte, least significant bits first (``encoder.py:115-130``)."""
    n = codes.shape[-1]
    pad = (4 - n % 4) % 4
    if pad:
        codes = np.concatenate([codes, np.zeros(codes.shape[:-1] + (pad,), np.uint8)], axis=-1)
    out = np.zeros(codes.shape[:-1] + (codes.shape[-1] // 4,), np.uint8)
    for i in range(4):
        out |= ((codes[..., i::4] & 0x03) << (2 * i)).astype(np.uint8)
    return out


def unpack_4bit(packed: np.ndarray, n: int) -> np.ndarray:
    """Inverse of :func:`pack_4bit` (``decoder.py:69-75``)."""
    out = np.stack([packed & 0x0F, (packed >> 4) & 0x0F], axis=-1).reshape(packed.shape[:-1] + (-1,))
    return out[..., :n]


def unpack_2bit(packed: np.ndarray, n: int) -> np.ndarray:
    """Inverse of :func:`pack_2bit` (``decoder.py:77-85``)."""
    out = np.stack([(packed >> (2 * i)) & 0x03 for i in range(4)], axis=-1).reshape(packed.shape[:-1] + (-1,))
    return out[..., :n]


def _pack(codes: np.ndarray, bits: int) -> np.ndarray:
    if bits == 8:
        return codes
    if bits == 4:
        return pack_4bit(codes)
    if bits == 2:
        return pack_2bit(codes)
    raise ValueError(f"unsupported angle bits: {bits}")


def _unpack(packed: np.ndarray, n: int, bits: int) -> np.ndarray:
    if bits == 8:
        return packed[..., :n]
    if bits == 4:
        return unpack_4bit(packed, n)
    if bits == 2:
        return unpack_2bit(packed, n)
    raise ValueError(f"unsupported angle bits: {bits}")


def encode_block(k: np.ndarray, l1_bits: int = 4, deep_bits: int = 4, split_dim: int = 64,
                 int8_radii: bool = False) -> dict:
    """Encode one 64-token block (or any ``(..., L, 128)`` array) of keys.

    Returns ``radii`` (float16, or int8 log codes), ``angle_codes_l1``, ``angle_codes_deep``
    (packed uint8) and ``radii_scales`` (float16 ``(..., 1, 1)`` or ``None``), the fields of
    ``PolarKeyBlock`` built at ``encoder.py:85-97``.
    """
    if l1_bits not in (4, 8):
        raise ValueError(f"unsupported k_angle_bits_level1: {l1_bits}")
    if deep_bits not in (2, 4, 8):
        raise ValueError(f"unsupported k_angle_bits_deep: {deep_bits}")
    k = np.asarray(k)
    dt = k.dtype
    if dt not in (np.float16, np.float32):
        raise ValueError("encode_block expects float16 or float32 keys")
    split_half = split_dim // 2
    x = k[..., 0::2]
    y = k[..., 1::2]
    # encoder.py:33 -- sqrt(x*x + y*y) in the working dtype, stored as float16.
    s = (x * x + y * y).astype(dt)
    radii_fp = _cr32(np.sqrt, s, dtype=dt).astype(np.float16)
    radii_scales = None
    if int8_radii:
        # encoder.py:34-45 -- log-int8 radii with one scale per (batch, head, block).
        floor = np.float16(1e-6)
        log_r = _cr32(np.log, np.maximum(radii_fp, floor), dtype=np.float16).astype(np.float32)
        log_scale = np.max(np.abs(log_r), axis=(-2, -1), keepdims=True)
        log_scale = np.where(log_scale == 0, np.float32(1e-6), log_scale).astype(np.float32)
        log_scale = (log_scale / np.float32(127.0)).astype(np.float32).astype(np.float16)
        q = np.round((log_r / log_scale.astype(np.float32)).astype(np.float32))
        radii = np.clip(q, -128, 127).astype(np.int8)
        radii_scales = log_scale
    else:
        radii = radii_fp
    # encoder.py:46-51 -- normalised angle in [0, 1] in the working dtype.
    angles = _cr32(np.arctan2, y, x, dtype=dt)
    shifted = (angles + dt.type(np.pi)).astype(dt)
    norm = (shifted / dt.type(2.0 * np.pi)).astype(dt)
    norm = np.clip(norm, dt.type(0.0), dt.type(1.0)).astype(dt)
    norm = np.where(norm > dt.type(1.0 - 1e-6), np.float32(0.0), norm.astype(np.float32)).astype(np.float32)
    # encoder.py:52-55 -- level-1 pairs [0, split/2), deep pairs after; float32 scale + round.
    l1_levels, deep_levels = 2 ** l1_bits, 2 ** deep_bits
    c_l1 = np.clip(np.round(norm[..., :split_half] * np.float32(l1_levels - 1)), 0, l1_levels - 1).astype(np.uint8)
    c_deep = np.clip(np.round(norm[..., split_half:] * np.float32(deep_levels - 1)), 0, deep_levels - 1).astype(np.uint8)
    # encoder.py:56-75 -- level-1 codes packed only at 4 bits; deep at 4 or 2 bits.
    return {
        "radii": radii,
        "angle_codes_l1": pack_4bit(c_l1) if l1_bits == 4 else c_l1,
        "angle_codes_deep": _pack(c_deep, deep_bits),
        "radii_scales": radii_scales,
    }


def angle_of_code(code: np.ndarray, bits: int) -> np.ndarray:
    """Decoder angle for an integer code: ``code/(2**bits-1) * 2pi - pi`` in float32
    (``decoder.py:36-56``)."""
    norm = (np.asarray(code).astype(np.float32) / np.float32(2 ** bits - 1)).astype(np.float32)
    return (norm * np.float32(2.0 * np.pi) - np.float32(np.pi)).astype(np.float32)


def decode_block(radii, angle_codes_l1, angle_codes_deep, radii_scales=None, l1_bits: int = 4,
                 deep_bits: int = 4, split_dim: int = 64) -> np.ndarray:
    """Reconstruct float16 keys ``(..., L, 128)`` from a block payload (``decoder.py:7-67``).

    Leading dims are free; ``radii_scales`` (int8 radii only) broadcasts against
    ``radii[..., :1, :1]``.
    """
    split_half = split_dim // 2
    n_deep = PAIRS - split_half
    codes_l1 = _unpack(np.asarray(angle_codes_l1), split_half, l1_bits)
    codes_deep = _unpack(np.asarray(angle_codes_deep), n_deep, deep_bits)
    ang = np.concatenate([angle_of_code(codes_l1, l1_bits), angle_of_code(codes_deep, deep_bits)], axis=-1)
    radii = np.asarray(radii)
    if radii_scales is not None:
        # decoder.py:57-61 -- exp(code * scale) for log-int8 radii, in float32.
        arg = (radii.astype(np.float32) * np.asarray(radii_scales).astype(np.float32)).astype(np.float32)
        r = _cr32(np.exp, arg, dtype=np.float32)
    else:
        r = radii.astype(np.float32)
    kx = (r * _cr32(np.cos, ang, dtype=np.float32)).astype(np.float32)
    ky = (r * _cr32(np.sin, ang, dtype=np.float32)).astype(np.float32)
    return np.stack([kx, ky], axis=-1).reshape(radii.shape[:-1] + (HEAD_DIM,)).astype(np.float16)


def cos_sin_table(bits: int) -> np.ndarray:
    """float32 ``(cos, sin)`` of the decoder angle of every code value, shape ``(2**bits, 2)``."""
    a = angle_of_code(np.arange(2 ** bits), bits)
    return np.stack([_cr32(np.cos, a, dtype=np.float32), _cr32(np.sin, a, dtype=np.float32)], axis=-1)
