"""``CudaKernelBridge``: the reference bridge's ``execute_*`` API over the CUDA library.

Mirrors ``MetalKernelBridge`` (``rfsn_v11/kernels/turbo_polar/metal.py:57-792``): same
method names, arguments (payload blocks, optional QJL tensors, config, ``actual_seq_len``)
and ``(output, trace)`` results.  There is no fallback: the reference silently drops to MLX
on the CPU when its dispatch probe fails (``metal.py:495-496, :729-734``); here a missing
library or device raises.  The trace keeps the reference's keys, with ``metal_used`` False
and ``cuda_used`` True.
"""

from __future__ import annotations

import ctypes
from typing import Any, Dict, Optional, Tuple

import torch

from . import _lib
from .codec import pool_of_block, _stream
from .pages import PAGE
from .payload import PolarKeyBlock, QuantizedVBlock


def _qcode(q: torch.Tensor) -> int:
    if q.dtype == torch.float16:
        return _lib.TP_F16
    if q.dtype == torch.float32:
        return _lib.TP_F32
    raise ValueError(f"query dtype must be float16 or float32, got {q.dtype}")


class CudaKernelBridge:
    """Process-wide singleton like the reference's (``metal.py:68-86``); holds workspaces."""

    _instance: "CudaKernelBridge | None" = None

    def __new__(cls):
        if cls._instance is None:
            cls._instance = super().__new__(cls)
            cls._instance._ws = {}
        return cls._instance

    def _workspace(self, device, heads: int, q_heads: int) -> torch.Tensor:
        need = _lib.lib().tp_decode_attention_workspace_size(heads, q_heads)
        if need == 0:
            raise ValueError("num_q_heads must be divisible by num_kv_heads for GQA")
        key = (str(device), heads, q_heads)
        ws = self._ws.get(key)
        if ws is None:
            ws = torch.zeros(need, dtype=torch.uint8, device=device)
            self._ws[key] = ws
        return ws

    @staticmethod
    def _reject_qjl(use_qjl: bool):
        if use_qjl:
            raise NotImplementedError("QJL is not supported in this release; set use_qjl=False")

    # ------------------------------------------------------------------ scores
    def execute_fused_qk(self, q: torch.Tensor, block: PolarKeyBlock, config) -> torch.Tensor:
        """Scores ``(B, H_q, S*64)`` float16 (``metal.py:494-530``)."""
        pool, B, H, S = pool_of_block(block)
        q = q.contiguous()
        Hq = q.shape[1]
        out = torch.empty((B, Hq, S * PAGE), dtype=torch.float16, device=q.device)
        _lib.check(_lib.lib().tp_fused_scores(ctypes.byref(pool.struct()), S, q.data_ptr(), _qcode(q), B * Hq,
                                              float(config.attention_scale), out.data_ptr(), _stream(q.device)))
        return out

    # ------------------------------------------------------------------ attention
    def _attention(self, q, block: Optional[PolarKeyBlock], quant_v: Optional[QuantizedVBlock], tail_k, tail_v,
                   config, actual_seq_len: int) -> torch.Tensor:
        if block is not None:
            pool, B, H, S = pool_of_block(block, quant_v)
        else:
            pool, B, H, S = None, tail_k.shape[0], tail_k.shape[1], 0
        q = q.contiguous()
        Hq = q.shape[1]
        heads = B * H
        t = 0 if tail_k is None else int(tail_k.shape[2])
        if t > PAGE:
            raise ValueError("dense tail must hold at most 64 tokens")
        tdt = torch.float16 if (tail_k is None or tail_k.dtype == torch.float16) else torch.float32
        tk = torch.zeros((heads, PAGE, 128), dtype=tdt, device=q.device)
        tv = torch.zeros_like(tk)
        if t:
            tk[:, :t] = tail_k.reshape(heads, t, 128).to(tdt)
            tv[:, :t] = tail_v.reshape(heads, t, 128).to(tdt)
        tail = _lib.Tail(tk.data_ptr(), tv.data_ptr(), _lib.TP_F16 if tdt == torch.float16 else _lib.TP_F32)
        if pool is None:
            fmt = config.format_fields()
            st = _lib.empty_pool(heads, fmt)
        else:
            st = pool.struct()
        out = torch.empty((B, Hq, 128), dtype=torch.float16, device=q.device)
        ws = self._workspace(q.device, heads, B * Hq)
        _lib.check(_lib.lib().tp_decode_attention(
            ctypes.byref(st), ctypes.byref(tail), _lib.State(S, t, int(actual_seq_len), 0), None, q.data_ptr(),
            _qcode(q), B * Hq, float(config.attention_scale), out.data_ptr(), None, ws.data_ptr(), ws.numel(),
            _stream(q.device)))
        return out

    def execute_online_attention_quant_v(self, q, block, quant_v, qjl_payload, q_proj_signs, config,
                                         actual_seq_len: int, use_qjl: bool = False) -> Tuple[torch.Tensor, Dict[str, Any]]:
        """Compressed pages only (``metal.py:651-715``)."""
        self._reject_qjl(use_qjl)
        out = self._attention(q, block, quant_v, None, None, config, actual_seq_len)
        return out, self._trace("tp_decode_attention", q, block, actual_seq_len, tail=None)

    def execute_online_attention_quant_v_dense_tail(self, q, block, quant_v, tail_k, tail_v, qjl_payload,
                                                    q_proj_signs, config, actual_seq_len: int,
                                                    use_qjl: bool = False) -> Tuple[torch.Tensor, Dict[str, Any]]:
        """Compressed pages followed by a dense tail (``metal.py:717-792``)."""
        self._reject_qjl(use_qjl)
        out = self._attention(q, block, quant_v, tail_k, tail_v, config, actual_seq_len)
        return out, self._trace("tp_decode_attention_dense_tail", q, block, actual_seq_len, tail=tail_k)

    def execute_online_attention_dense_v(self, q, block, v_dense, qjl_payload, q_proj_signs, config,
                                         actual_seq_len: int, use_qjl: bool = False) -> Tuple[torch.Tensor, Dict[str, Any]]:
        """Compressed keys with dense values (``metal.py:587-649``): ``v_dense`` is
        ``(B, H_kv, S, 64, 128)`` or ``(B, H_kv, S*64, 128)``, read as float16 as the reference's
        kernel reads it (``tqpolar_online_attention.metal:16``).  Tokens ``>= actual_seq_len``
        are masked; ``actual_seq_len`` beyond ``S*64`` attends to every token.  The configuration
        contract still rejects dense-V storage (``turbo_polar_config.py:48-49``): this entry point
        serves callers that hold the values themselves, as the reference's debug kernel does."""
        self._reject_qjl(use_qjl)
        pool, B, H, S = pool_of_block(block)
        q = q.contiguous()
        Hq = q.shape[1]
        heads = B * H
        tokens = S * PAGE
        if v_dense.numel() != heads * tokens * 128:
            raise ValueError(f"v_dense must hold (B, H_kv, S*64, 128) = ({B}, {H}, {tokens}, 128) values")
        if int(actual_seq_len) < 1:
            raise ValueError("actual_seq_len must be at least 1")
        v = v_dense.reshape(heads, tokens, 128).to(torch.float16).contiguous()
        out = torch.empty((B, Hq, 128), dtype=torch.float16, device=q.device)
        ws = self._workspace(q.device, heads, B * Hq)
        _lib.check(_lib.lib().tp_decode_attention_dense_v(
            ctypes.byref(pool.struct()), _lib.State(S, 0, min(int(actual_seq_len), tokens), 0), v.data_ptr(),
            tokens * 128, tokens, q.data_ptr(), _qcode(q), B * Hq, float(config.attention_scale), out.data_ptr(), None,
            ws.data_ptr(), ws.numel(), _stream(q.device)))
        tr = self._trace("tp_decode_attention_dense_v", q, block, actual_seq_len, tail=None)
        tr["quant_v_used"] = False
        return out, tr

    @staticmethod
    def _trace(name, q, block, actual_seq_len, tail) -> Dict[str, Any]:
        h_kv = block.radii.shape[1] if block is not None else tail.shape[1]
        tr = {
            "kernel_name": name,
            "metal_used": False,
            "cuda_used": True,
            "fallback_used": False,
            "qjl_used": False,
            "quant_v_used": True,
            "actual_seq_len": actual_seq_len,
            "num_queries_per_kv": q.shape[1] // h_kv,
        }
        if tail is not None:
            tr["tail_length"] = int(tail.shape[2])
        return tr
