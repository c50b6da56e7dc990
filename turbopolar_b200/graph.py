"""CUDA-graph capture of decode steps.

A decode step of one cache layer is ``append(1 token) + attention(q)``, one tp_decode_step
call: its kernels read the cache counters from the runtime's device state words and advance
them, so one captured graph replays correctly at every sequence position.  The host mirror of the
counters is advanced on each replay with the same deterministic rule the append kernel uses.

Requirements: the runtime was created with ``max_seq_len`` (the pool never grows while a
graph holds its pointers) and has seen at least one append (buffers exist).
"""

from __future__ import annotations

import ctypes
from typing import Optional, Sequence

import torch

from . import _lib
from .cache import TurboPolarKVCacheRuntime
from .pages import PAGE


def launch_append(rt: TurboPolarKVCacheRuntime, k: torch.Tensor, v: torch.Tensor) -> None:
    """Enqueue tp_append of one token ``(B, H_kv, 1, 128)`` reading the device counters."""
    B, H, T, D = k.shape
    kf = k.reshape(B * H, T, D)
    _lib.check(_lib.lib().tp_append(
        ctypes.byref(rt.pool.struct()), ctypes.byref(rt.tail_struct()), rt.d_state.data_ptr(), kf.data_ptr(),
        v.reshape(B * H, T, D).data_ptr(), _lib.TP_F16 if k.dtype == torch.float16 else _lib.TP_F32,
        kf.stride(0), kf.stride(1), 1, torch.cuda.current_stream(k.device).cuda_stream))


def launch_attention(rt: TurboPolarKVCacheRuntime, q: torch.Tensor, out: Optional[torch.Tensor], scale: float,
                     partial_out: Optional[torch.Tensor] = None, exchange=None) -> None:
    """Enqueue tp_decode_attention reading the device counters (tp_decode_attention_sharded
    with an ``exchange``: merged across ranks into ``out``)."""
    B, Hq = q.shape[0], q.shape[-2]
    ws = rt._workspace_for(B * Hq)
    if exchange is not None:
        _lib.check(_lib.lib().tp_decode_attention_sharded(
            ctypes.byref(rt.pool_struct()), ctypes.byref(rt.tail_struct()), rt.state(), rt.d_state.data_ptr(),
            q.data_ptr(), _lib.TP_F16 if q.dtype == torch.float16 else _lib.TP_F32, B * Hq, float(scale),
            out.data_ptr(), ctypes.byref(exchange.struct), ws.data_ptr(), ws.numel(),
            torch.cuda.current_stream(q.device).cuda_stream))
        return
    _lib.check(_lib.lib().tp_decode_attention(
        ctypes.byref(rt.pool_struct()), ctypes.byref(rt.tail_struct()), rt.state(), rt.d_state.data_ptr(),
        q.data_ptr(), _lib.TP_F16 if q.dtype == torch.float16 else _lib.TP_F32, B * Hq, float(scale),
        out.data_ptr() if out is not None else None, partial_out.data_ptr() if partial_out is not None else None,
        ws.data_ptr(), ws.numel(), torch.cuda.current_stream(q.device).cuda_stream))


def launch_decode_step(rt: TurboPolarKVCacheRuntime, k: torch.Tensor, v: torch.Tensor, q: torch.Tensor,
                       out: Optional[torch.Tensor], scale: float, partial_out: Optional[torch.Tensor] = None,
                       exchange=None) -> None:
    """Enqueue tp_decode_step (append one token ``(B, H_kv, 1, 128)``, then attend) on the
    device counters (tp_decode_step_sharded with an ``exchange``)."""
    B, H, T, D = k.shape
    kf = k.reshape(B * H, D)
    vf = v.reshape(B * H, D)
    if kf.stride() != vf.stride() or kf.stride(-1) != 1:
        raise ValueError("new K and V rows must share one layout with contiguous channels")
    Bq, Hq = q.shape[0], q.shape[-2]
    ws = rt._workspace_for(Bq * Hq)
    kvd = _lib.TP_F16 if k.dtype == torch.float16 else _lib.TP_F32
    qd = _lib.TP_F16 if q.dtype == torch.float16 else _lib.TP_F32
    if exchange is not None:
        _lib.check(_lib.lib().tp_decode_step_sharded(
            ctypes.byref(rt.pool_struct()), ctypes.byref(rt.tail_struct()), rt.d_state.data_ptr(), kf.data_ptr(),
            vf.data_ptr(), kvd, kf.stride(0), q.data_ptr(), qd, Bq * Hq, float(scale), out.data_ptr(),
            ctypes.byref(exchange.struct), ws.data_ptr(), ws.numel(), torch.cuda.current_stream(q.device).cuda_stream))
        return
    _lib.check(_lib.lib().tp_decode_step(
        ctypes.byref(rt.pool_struct()), ctypes.byref(rt.tail_struct()), rt.d_state.data_ptr(), kf.data_ptr(),
        vf.data_ptr(), _lib.TP_F16 if k.dtype == torch.float16 else _lib.TP_F32, kf.stride(0), q.data_ptr(),
        _lib.TP_F16 if q.dtype == torch.float16 else _lib.TP_F32, Bq * Hq, float(scale),
        out.data_ptr() if out is not None else None, partial_out.data_ptr() if partial_out is not None else None,
        ws.data_ptr(), ws.numel(), torch.cuda.current_stream(q.device).cuda_stream))


def advance_host(rt: TurboPolarKVCacheRuntime, n_tokens: int = 1) -> None:
    """Advance the host mirror exactly as ``n_tokens`` single-token device appends do."""
    for _ in range(n_tokens):
        rt.actual_seq_len += 1
        rt.tail_len += 1
        if rt.tail_len == PAGE:
            rt.tail_len = 0
            rt._flushed(1)


def _check_room(rts: Sequence[TurboPolarKVCacheRuntime]) -> None:
    for rt in rts:
        if rt.tail_len == PAGE - 1 and rt.n_pages + 1 > rt.capacity:
            raise RuntimeError("TurboPolar page pool is full; create the runtime with a larger max_seq_len")


class DecodeStep:
    """One captured decode step over one or more cache layers.

    ``layers`` is a list of ``(runtime, k_in, v_in, q_in, out)``: fixed input/output buffers
    the caller refills between replays.  ``extra`` (optional callable) is captured after the
    attention launches, e.g. a collective on the outputs.
    """

    def __init__(self, rt, k_in=None, v_in=None, q_in=None, out=None, scale: Optional[float] = None, layers=None,
                 extra=None):
        if layers is None:
            layers = [(rt, k_in, v_in, q_in, out)]
        self.layers = layers
        for r, *_ in layers:
            if not r._initialized or r.pool is None or not r.max_seq_len:
                raise ValueError("capture needs an initialised runtime created with max_seq_len")
        self.scales = [float(r.config.attention_scale if scale is None else scale) for r, *_ in layers]
        # Warm the launch path (kernel attributes, workspaces) outside the capture; attention
        # reads the cache without changing it.
        for (r, _k, _v, q, o), s in zip(layers, self.scales):
            r._workspace_for(q.shape[0] * q.shape[-2])
            if r.n_pages or r.tail_len:
                launch_attention(r, q, o, s)
        torch.cuda.synchronize()
        self.graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(self.graph):
            for (r, k, v, q, o), s in zip(layers, self.scales):
                launch_decode_step(r, k, v, q, o, s)
            if extra is not None:
                extra()

    def replay(self) -> None:
        rts = [r for r, *_ in self.layers]
        _check_room(rts)
        self.graph.replay()
        for r in rts:
            advance_host(r, 1)
