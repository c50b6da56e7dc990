"""Fallback attention of the reference restated in NumPy float64 (oracle; test only).

Follows ``rfsn_v11/kernels/turbo_polar/metal.py``:

* ``_cpu_fused_qk`` (``:254-260``): decode K, repeat KV heads over the GQA group,
  ``scores = sum(q * k) * attention_scale``;
* ``_cpu_online_attention_dense_tail`` (``:293-332``) and ``_cpu_online_attention``
  (``:267-291``): decode K, dequantize V, append the dense tail, repeat over the GQA
  group, mask token indices ``>= actual_seq_len`` with -1e9, softmax, weighted sum of V.

The reference evaluates these in MLX float16; here the same formula runs in float64 on the
float16-rounded K and V so that the kernel's float32 arithmetic can be checked against a
result that carries no reduction error of its own.
"""

from __future__ import annotations

import numpy as np

from . import polar, vquant


def decode_pages(pages: dict, fmt: dict):
    """Dense float16 K and V ``(H_kv, S*64, 128)`` from a page set.

    ``pages`` holds ``radii (H,S,64,64)``, ``angle_codes_l1``, ``angle_codes_deep``,
    ``radii_scales (H,S)`` or ``None``, ``v_codes (H,S,64,128)``, ``v_scales (H,S,64,4)``;
    ``fmt`` holds ``l1_bits``, ``deep_bits``, ``split_dim``.
    """
    rs = pages.get("radii_scales")
    if rs is not None:
        rs = np.asarray(rs)[..., None, None]
    k = polar.decode_block(pages["radii"], pages["angle_codes_l1"], pages["angle_codes_deep"], rs,
                           fmt["l1_bits"], fmt["deep_bits"], fmt["split_dim"])
    v = vquant.dequantize(pages["v_codes"], pages["v_scales"])
    h, s = k.shape[0], k.shape[1]
    return k.reshape(h, s * polar.BLOCK, polar.HEAD_DIM), v.reshape(h, s * polar.BLOCK, polar.HEAD_DIM)


def fused_scores(q: np.ndarray, k: np.ndarray, scale: float) -> np.ndarray:
    """``scores[hq, t] = scale * q[hq] . k[hq // G, t]`` in float64 (``metal.py:254-260``)."""
    q = np.asarray(q, np.float64)
    k = np.asarray(k, np.float64)
    g = q.shape[0] // k.shape[0]
    kk = np.repeat(k, g, axis=0)
    return np.einsum("hd,htd->ht", q, kk) * float(scale)


def attention(q, k, v, actual_seq_len: int, scale: float) -> np.ndarray:
    """Masked softmax attention of ``q (H_q,128)`` over ``k, v (H_kv,T,128)``; float64 result.

    Token ``t`` takes part iff ``t < actual_seq_len`` (the -1e9 mask of ``metal.py:318-319``);
    with every token masked the softmax is uniform over all of them, as in the reference.
    """
    s = fused_scores(q, k, scale)
    t = s.shape[-1]
    s = np.where(np.arange(t)[None, :] < actual_seq_len, s, -1e9)
    s = s - s.max(axis=-1, keepdims=True)
    w = np.exp(s)
    w /= w.sum(axis=-1, keepdims=True)
    g = s.shape[0] // np.asarray(v).shape[0]
    vv = np.repeat(np.asarray(v, np.float64), g, axis=0)
    return np.einsum("ht,htd->hd", w, vv)


def attention_dense_tail(q, pages: dict | None, fmt: dict, tail_k, tail_v, actual_seq_len: int,
                         scale: float) -> np.ndarray:
    """Compressed pages followed by a dense tail (``metal.py:293-332``); float64 ``(H_q,128)``."""
    parts_k, parts_v = [], []
    if pages is not None and np.asarray(pages["radii"]).shape[1] > 0:
        k, v = decode_pages(pages, fmt)
        parts_k.append(k.astype(np.float64))
        parts_v.append(v.astype(np.float64))
    if tail_k is not None and np.asarray(tail_k).shape[1] > 0:
        parts_k.append(np.asarray(tail_k, np.float64))
        parts_v.append(np.asarray(tail_v, np.float64))
    return attention(q, np.concatenate(parts_k, axis=1), np.concatenate(parts_v, axis=1), actual_seq_len, scale)


def attention_dense_v(q, pages: dict, fmt: dict, v_dense, actual_seq_len: int, scale: float) -> np.ndarray:
    """Compressed keys with dense values (``execute_online_attention_dense_v``'s fallback,
    ``metal.py:587-603`` into ``_cpu_online_attention``, ``:267-291``); float64 ``(H_q,128)``.

    ``v_dense`` is ``(H_kv, S*64, 128)``; the value codes in ``pages`` are not used.
    """
    k, _ = decode_pages(pages, fmt)
    return attention(q, k.astype(np.float64), np.asarray(v_dense, np.float64), actual_seq_len, scale)


def partial(q, k, v, scale: float) -> np.ndarray:
    """Unnormalised softmax partial of ``q (H_q,128)`` over one token range ``k, v (H_kv,T,128)``:
    ``[H_q, 130]`` records ``(m, l, o[128])`` with ``m`` the maximum score in base-2 units,
    ``l = sum 2^(s - m)`` and ``o = sum 2^(s - m) v`` (``s`` = score in base-2 units).

    No reference counterpart (the reference runs on one device): this is the record the
    sequence-sharded path exchanges between GPUs; an empty range gives ``m = -inf``.
    """
    q = np.asarray(q, np.float64)
    hq = q.shape[0]
    if np.asarray(k).shape[1] == 0:
        rec = np.zeros((hq, 130))
        rec[:, 0] = -np.inf
        return rec
    s = fused_scores(q, k, scale) / np.log(2.0)
    m = s.max(axis=-1, keepdims=True)
    w = np.exp2(s - m)
    g = hq // np.asarray(v).shape[0]
    vv = np.repeat(np.asarray(v, np.float64), g, axis=0)
    return np.concatenate([m, w.sum(axis=-1, keepdims=True), np.einsum("ht,htd->hd", w, vv)], axis=-1)


def combine(partials: np.ndarray) -> np.ndarray:
    """Merge ``[n, H_q, 130]`` partials (log-sum-exp): ``M = max m_r``, ``L = sum l_r 2^(m_r-M)``,
    ``O = sum o_r 2^(m_r-M) / L``; float64 ``(H_q, 128)``."""
    p = np.asarray(partials, np.float64)
    m = p[..., 0]
    M = m.max(axis=0)
    w = np.where(np.isneginf(m), 0.0, np.exp2(m - M))
    L = (p[..., 1] * w).sum(axis=0)
    O = (p[..., 2:] * w[..., None]).sum(axis=0)
    return O / L[:, None]
