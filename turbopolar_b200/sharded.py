"""Sequence-sharded decode attention over several GPUs (one process per GPU).

The reference is single-device (no collective exists in it).  For contexts too long for one
GPU's bandwidth, the pages of every KV head are split into contiguous ranges, one per rank;
the last rank also holds the dense tail and receives the new tokens.  Each rank computes, for
every query head, an unnormalised partial (m in log2 units, l, o[128]) over its range
(``tp_decode_attention`` with ``partial_out``), one NCCL all-gather per layer exchanges the
``H_q x 130`` floats, and every rank merges them with ``tp_combine_partials``:
``M = max m_r, L = sum l_r 2^(m_r-M), O = sum o_r 2^(m_r-M) / L``.
"""

from __future__ import annotations

import ctypes
from typing import List, Tuple

import torch
import torch.distributed as dist

from . import _lib, graph
from .cache import TurboPolarKVCacheRuntime
from .pages import PAGE


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


class ShardedDecodeStep:
    """One captured decode step over all layers: local attention partial (the last rank appends
    the new token in the same call, tp_decode_step), NCCL all-gather, combine.  The graph must
    be released (``release()``) before the process group is destroyed."""

    def __init__(self, layers: List[TurboPolarKVCacheRuntime], k_in, v_in, q_in, out, rank: int, world: int,
                 group=None):
        self.layers, self.rank, self.world, self.group = layers, rank, world, group
        self.last = rank == world - 1
        dev = q_in[0].device
        hq = q_in[0].shape[0] * q_in[0].shape[-2]
        self.partials = [torch.empty((hq, _lib.PARTIAL_FLOATS), dtype=torch.float32, device=dev) for _ in layers]
        self.gathered = [torch.empty((world, hq, _lib.PARTIAL_FLOATS), dtype=torch.float32, device=dev)
                         for _ in layers]
        for rt, q in zip(layers, q_in):
            rt._workspace_for(hq)
        # NCCL warm-up outside the capture.
        dist.all_gather_into_tensor(self.gathered[0], self.partials[0], group=group)
        torch.cuda.synchronize()
        self.graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(self.graph):
            for i, rt in enumerate(layers):
                if self.last:
                    graph.launch_decode_step(rt, k_in[i], v_in[i], q_in[i], None, rt.config.attention_scale,
                                             partial_out=self.partials[i])
                else:
                    graph.launch_attention(rt, q_in[i], None, rt.config.attention_scale, partial_out=self.partials[i])
                dist.all_gather_into_tensor(self.gathered[i], self.partials[i], group=group)
                combine(self.gathered[i], out[i])
        torch.cuda.synchronize()

    def partial_buffer(self, i: int) -> torch.Tensor:
        return self.partials[i]

    def replay(self) -> None:
        if self.last:
            graph._check_room(self.layers)
        self.graph.replay()
        if self.last:
            for rt in self.layers:
                graph.advance_host(rt, 1)

    def release(self) -> None:
        torch.cuda.synchronize()
        self.graph = None
