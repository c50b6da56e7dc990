"""Sequence-sharded decode attention over the GPUs of one node (one process per GPU).

The reference is single-device (no collective exists in it).  For contexts too long for one
GPU's bandwidth, the pages of every KV head are split into contiguous ranges, one per rank;
the last rank also holds the dense tail and receives the new tokens.  Each rank computes, for
every query head, an unnormalised partial (m in log2 units, l, o[128]) over its range, and the
partials are merged with ``M = max m_r, L = sum l_r 2^(m_r-M), O = sum o_r 2^(m_r-M) / L``.

Two exchanges: ``PeerExchange`` (the default) does it inside the attention launch -- every
rank's split-combine CTAs store their records into every rank's buffer over NVLink (buffers
mapped through CUDA IPC) as 64-bit words carrying the call's epoch, wait (bounded) until the
other ranks' words carry it and merge;
the NCCL path (``exchange=False``) writes ``partial_out``, all-gathers it and runs
``tp_combine_partials``.
"""

from __future__ import annotations

import ctypes
import time
from typing import List, Tuple

import torch
import torch.distributed as dist

from . import _lib, graph
from .cache import TurboPolarKVCacheRuntime


def page_range(n_pages: int, rank: int, world: int) -> Tuple[int, int]:
    """Contiguous page range ``[lo, hi)`` of ``rank`` for ``n_pages`` full pages."""
    return rank * n_pages // world, (rank + 1) * n_pages // world


def combine(partials: torch.Tensor, out: torch.Tensor) -> torch.Tensor:
    """Merge ``partials [n, H_q, 130]`` (float32) into fp16 ``out [.., H_q, 128]``."""
    n, hq = partials.shape[0], partials.shape[1]
    _lib.check(_lib.lib().tp_combine_partials(partials.data_ptr(), n, hq, out.data_ptr(),
                                              torch.cuda.current_stream(partials.device).cuda_stream))
    return out


def sharded_attention(rt: TurboPolarKVCacheRuntime, q: torch.Tensor, group=None) -> torch.Tensor:
    """Eager sharded attention: local partial, all-gather over ``group``, combine."""
    B, Hq = q.shape[0], q.shape[-2]
    part = torch.empty((B * Hq, _lib.PARTIAL_FLOATS), dtype=torch.float32, device=q.device)
    if rt.n_pages or rt.tail_len:
        rt.attention(q, partial_out=part)
    else:
        part.zero_()
        part[:, 0] = float("-inf")
    world = dist.get_world_size(group)
    gathered = torch.empty((world, B * Hq, _lib.PARTIAL_FLOATS), dtype=torch.float32, device=q.device)
    dist.all_gather_into_tensor(gathered, part, group=group)
    out = torch.empty((B, Hq, 128), dtype=torch.float16, device=q.device)
    return combine(gathered, out)


class RankFailure(RuntimeError):
    """A rank did not reach a step of a sharded decode in time (it raised, exited or skipped)."""


class StepMonitor:
    """Host-side liveness of the ranks of a sharded decode.

    Before launching step ``k`` every rank announces it in the process group's key-value store
    (one key per rank and step) and waits, within ``timeout_s``, until every rank has announced
    step ``k`` (``step``).  A rank that raised, exited or skipped the step never announces it,
    so the others raise RankFailure on the host, naming it, instead of launching work that
    would wait for its records (the peer exchange's bounded wait, or a collective).  Keys are
    tested with ``store.check``, which never blocks; a rank deletes its own key of step k - 2
    when it announces step k (every rank has passed step k - 1's check by then, so nobody reads
    it any more).
    """

    def __init__(self, rank: int, world: int, store=None, prefix: str = "tp_steps", timeout_s: float = 30.0,
                 poll_s: float = 0.001):
        if store is None:
            store = dist.distributed_c10d._get_default_store()
        self.store, self.rank, self.world = store, rank, world
        self.prefix, self.timeout_s, self.poll_s = prefix, float(timeout_s), float(poll_s)
        self.steps = 0
        self._announced: List[int] = []

    def _key(self, r: int, k: int) -> str:
        return f"{self.prefix}/{r}/{k}"

    def step(self, k: int = None) -> int:
        """Announce step ``k`` (default: the step after the last one announced here) and return
        it once every rank has announced it; raise RankFailure naming the first rank that has
        not within timeout_s."""
        k = self.steps + 1 if k is None else int(k)
        self.store.set(self._key(self.rank, k), "1")
        self._announced.append(k)
        if len(self._announced) > 2:
            self.store.delete_key(self._key(self.rank, self._announced.pop(0)))
        deadline = time.monotonic() + self.timeout_s
        for r in range(self.world):
            key = self._key(r, k)
            while not self.store.check([key]):
                if time.monotonic() > deadline:
                    raise RankFailure(f"rank {r} did not reach step {k} within {self.timeout_s:g} s "
                                      f"(seen from rank {self.rank})")
                time.sleep(self.poll_s)
        self.steps = k
        return k


class PeerExchange:
    """This rank's exchange buffer and every other rank's, mapped into this process through
    CUDA IPC (handles all-gathered over ``group``).  One per call site that is replayed in
    step: every rank must make the same sequence of sharded calls on it."""

    def __init__(self, num_q_heads: int, group=None):
        self.world = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        if not 2 <= self.world <= _lib.MAX_RANKS:
            raise ValueError(f"peer exchange needs 2..{_lib.MAX_RANKS} ranks, got {self.world}")
        lib = _lib.lib()
        nbytes = lib.tp_exchange_bytes(self.world, num_q_heads)
        own = ctypes.c_void_p()
        handle = (ctypes.c_ubyte * 64)()
        _lib.check(lib.tp_ipc_alloc(nbytes, ctypes.byref(own), handle))
        handles = [None] * self.world
        dist.all_gather_object(handles, bytes(handle), group=group)
        self._own = own.value
        self._opened = []
        bufs = []
        for r, h in enumerate(handles):
            if r == self.rank:
                bufs.append(self._own)
                continue
            p = ctypes.c_void_p()
            hb = (ctypes.c_ubyte * 64).from_buffer_copy(h)
            _lib.check(lib.tp_ipc_open(hb, ctypes.byref(p)))
            self._opened.append(p.value)
            bufs.append(p.value)
        arr = (ctypes.c_void_p * _lib.MAX_RANKS)(*(bufs + [None] * (_lib.MAX_RANKS - self.world)))
        self.struct = _lib.Exchange(self.world, self.rank, arr)
        self._group = group

    def close(self) -> None:
        """Unmap the peers' buffers and free this one (collective: peers may still write into it
        until every rank is past its last call)."""
        if self._own is None:
            return
        torch.cuda.synchronize()
        dist.barrier(group=self._group)
        lib = _lib.lib()
        for p in self._opened:
            lib.tp_ipc_close(p)
        dist.barrier(group=self._group)
        lib.tp_ipc_free(self._own)
        self._own = None


def exchange_attention(rt: TurboPolarKVCacheRuntime, q: torch.Tensor, exchange: PeerExchange,
                       out: torch.Tensor = None) -> torch.Tensor:
    """Eager sharded attention merged inside the launch (``tp_decode_attention_sharded``)."""
    B, Hq = q.shape[0], q.shape[-2]
    if out is None:
        out = torch.empty((B, Hq, 128), dtype=torch.float16, device=q.device)
    qf = q.reshape(B * Hq, 128).contiguous()
    ws = rt._workspace_for(B * Hq)
    _lib.check(_lib.lib().tp_decode_attention_sharded(
        ctypes.byref(rt.pool_struct()), ctypes.byref(rt.tail_struct()), rt.state(), None, qf.data_ptr(),
        _lib.TP_F16 if qf.dtype == torch.float16 else _lib.TP_F32, B * Hq, float(rt.config.attention_scale),
        out.data_ptr(), ctypes.byref(exchange.struct), ws.data_ptr(), ws.numel(),
        torch.cuda.current_stream(q.device).cuda_stream))
    return out


class ShardedDecodeStep:
    """One captured decode step over all layers (the last rank appends the new token in the same
    call, tp_decode_step).  With ``exchange`` (the default) each layer is one sharded attention
    call that merges the ranks' partials inside its launch over NVLink; otherwise a local
    partial, an NCCL all-gather and tp_combine_partials.  The graph must be released
    (``release()``) before the process group is destroyed.  With a ``monitor`` (StepMonitor) every
    replay first checks on the host that all ranks have reached the step."""

    def __init__(self, layers: List[TurboPolarKVCacheRuntime], k_in, v_in, q_in, out, rank: int, world: int,
                 group=None, exchange: bool = True, monitor: "StepMonitor" = None):
        self.layers, self.rank, self.world, self.group = layers, rank, world, group
        self.monitor = monitor
        self.last = rank == world - 1
        dev = q_in[0].device
        hq = q_in[0].shape[0] * q_in[0].shape[-2]
        self.partials = [torch.empty((hq, _lib.PARTIAL_FLOATS), dtype=torch.float32, device=dev) for _ in layers]
        for rt, q in zip(layers, q_in):
            rt._workspace_for(hq)
        self.exchanges = [PeerExchange(hq, group) for _ in layers] if exchange else None
        if not exchange:
            self.gathered = [torch.empty((world, hq, _lib.PARTIAL_FLOATS), dtype=torch.float32, device=dev)
                             for _ in layers]
            # NCCL warm-up outside the capture.
            dist.all_gather_into_tensor(self.gathered[0], self.partials[0], group=group)
        torch.cuda.synchronize()
        self.graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(self.graph):
            for i, rt in enumerate(layers):
                s = rt.config.attention_scale
                if exchange:
                    x = self.exchanges[i]
                    if self.last:
                        graph.launch_decode_step(rt, k_in[i], v_in[i], q_in[i], out[i], s, exchange=x)
                    else:
                        graph.launch_attention(rt, q_in[i], out[i], s, exchange=x)
                    continue
                if self.last:
                    graph.launch_decode_step(rt, k_in[i], v_in[i], q_in[i], None, s, partial_out=self.partials[i])
                else:
                    graph.launch_attention(rt, q_in[i], None, s, partial_out=self.partials[i])
                dist.all_gather_into_tensor(self.gathered[i], self.partials[i], group=group)
                combine(self.gathered[i], out[i])
        torch.cuda.synchronize()

    def partial_buffer(self, i: int) -> torch.Tensor:
        return self.partials[i]

    def replay(self) -> None:
        if self.monitor is not None:
            self.monitor.step()
        if self.last:
            graph._check_room(self.layers)
        self.graph.replay()
        if self.last:
            for rt in self.layers:
                graph.advance_host(rt, 1)

    def release(self) -> None:
        torch.cuda.synchronize()
        self.graph = None
        if self.exchanges:
            for x in self.exchanges:
                x.close()
            self.exchanges = None
