"""One decode step of a Hugging Face Llama model as a CUDA graph, on the TurboPolar cache or on a
dense float16 cache: the end-to-end configuration of the measurement plan on the device path.

The reference's end-to-end benchmark (``benchmarks/run_fast_attention_bench.py:104-121``)
decodes through mlx_lm with the patched attention call (``benchmarks/
turbopolar_fast_attention.py:247-278``): per layer the q/k/v projections, RoPE at the cache
offset, the fused compressed-cache attention (append the new token, attend), o_proj.  Here the
same arithmetic runs as one captured step over all layers, on the model's own weights (the
q/k/v and gate/up projections concatenated into one GEMV each): RMSNorm, the projections (cuBLAS
GEMVs), RoPE (Hugging Face's rotate-half form, applied to the query and key heads in one
pass), per layer one ``tp_decode_step`` call (TurboPolar) or flash-attention's decode with an
in-place cache append (``flash_attn_with_kvcache``; dense), o_proj, the SiLU MLP, the final
norm, the logits and their argmax.  The cache counters and the position of the new token are
device tensors advanced inside the graph, so one capture replays at every position.

A third attention, ``decompressed`` (eager, not captured), appends the token to the TurboPolar
cache and attends in float32 over the cache decoded by ``tp_decode_pages`` plus the dense tail:
the key and value formats' error alone, without the fused kernel's arithmetic.
"""

from __future__ import annotations

from typing import Optional

import torch
import torch.nn.functional as F

from . import graph as tpgraph
from .llama import TurboPolarCache


class LlamaDecodeGraph:
    """Decode steps of ``model`` after a prefill into ``cache``.

    ``cache`` is a :class:`~turbopolar_b200.llama.TurboPolarCache` whose runtimes were created
    with ``max_seq_len`` (``make_turbo_caches(..., max_seq_len=...)``), or a transformers cache
    holding the prompt's keys and values (copied into static ``[layers, 1, max_seq_len, H_kv,
    128]`` buffers).  ``attention`` is ``"fused"`` (TurboPolar, captured), ``"dense"`` (captured)
    or ``"decompressed"`` (TurboPolar, eager).  ``token`` holds the input token of the next
    step; after a step ``logits`` (float32) and ``next`` (argmax) hold its outputs.
    """

    def __init__(self, model, cache, max_seq_len: int, attention: Optional[str] = None):
        c = model.config
        self.model = model
        self.L, self.hq, self.hkv, self.d = c.num_hidden_layers, c.num_attention_heads, c.num_key_value_heads, \
            c.head_dim
        self.eps = c.rms_norm_eps
        self.max_seq_len = int(max_seq_len)
        self.dev = model.lm_head.weight.device
        self.turbo = isinstance(cache, TurboPolarCache)
        self.attention = attention or ("fused" if self.turbo else "dense")
        if self.attention not in ("fused", "dense", "decompressed"):
            raise ValueError(f"unknown attention {self.attention!r}")
        if (self.attention != "dense") != self.turbo:
            raise ValueError("fused / decompressed attention needs a TurboPolarCache, dense a dense cache")
        layers = model.model.layers
        with torch.no_grad():
            self.wqkv = [torch.cat([m.self_attn.q_proj.weight, m.self_attn.k_proj.weight, m.self_attn.v_proj.weight])
                         for m in layers]
            self.wgu = [torch.cat([m.mlp.gate_proj.weight, m.mlp.up_proj.weight]) for m in layers]
        self.wo = [m.self_attn.o_proj.weight for m in layers]
        self.wd = [m.mlp.down_proj.weight for m in layers]
        self.n_in = [m.input_layernorm.weight for m in layers]
        self.n_post = [m.post_attention_layernorm.weight for m in layers]
        self.scale = float(layers[0].self_attn.scaling)
        if self.turbo:
            self.rts = [layer.runtime for layer in cache.layers]
            for rt in self.rts:
                if not rt._initialized or rt.pool is None or not rt.max_seq_len:
                    raise ValueError("the TurboPolar caches need a prefill and a max_seq_len")
            offset = self.rts[0].actual_seq_len
            self.attn_out = torch.empty((self.L, 1, self.hq, self.d), dtype=torch.float16, device=self.dev)
        else:
            from flash_attn import flash_attn_with_kvcache
            self._flash = flash_attn_with_kvcache
            offset = cache.get_seq_length()
            shape = (self.L, 1, self.max_seq_len, self.hkv, self.d)  # flash-attention's cache layout
            self.kb = torch.zeros(shape, dtype=torch.float16, device=self.dev)
            self.vb = torch.zeros_like(self.kb)
            for i in range(self.L):
                self.kb[i, :, :offset] = cache.layers[i].keys.transpose(1, 2)
                self.vb[i, :, :offset] = cache.layers[i].values.transpose(1, 2)
            self.seqlens = torch.zeros((1,), dtype=torch.int32, device=self.dev)
        self.token = torch.zeros((1, 1), dtype=torch.long, device=self.dev)
        self.pos = torch.full((1, 1), offset, dtype=torch.long, device=self.dev)
        self.logits = torch.empty((1, c.vocab_size), dtype=torch.float32, device=self.dev)
        self.next = torch.empty((1, 1), dtype=torch.long, device=self.dev)
        self.offset = offset
        self.graph = None

    # ------------------------------------------------------------------ the step
    def _rmsnorm(self, x, w):
        # LlamaRMSNorm: normalise in float32, round to the input dtype, scale by the weight.
        return w * F.rms_norm(x.float(), (x.shape[-1],), eps=self.eps).to(x.dtype)

    def _attend(self, i, q, k, v):
        """Attention of layer i for the new token: q (1, H_q, 1, 128), k, v (1, H_kv, 1, 128)
        after RoPE; returns (1, H_q, 128) float16."""
        if self.attention == "fused":
            out = self.attn_out[i]
            tpgraph.launch_decode_step(self.rts[i], k, v, q.reshape(1, self.hq, self.d), out, self.scale)
            return out
        if self.attention == "dense":
            # Appends k, v at position seqlens and attends over seqlens + 1 tokens.
            self.seqlens.copy_(self.pos.view(1))
            o = self._flash(q.transpose(1, 2), self.kb[i], self.vb[i], k=k.transpose(1, 2), v=v.transpose(1, 2),
                            cache_seqlens=self.seqlens, softmax_scale=self.scale, causal=True)
            return o.view(1, self.hq, self.d)
        rt = self.rts[i]
        rt.append(k.contiguous(), v.contiguous())
        kd, vd = rt.decompress(padded_tail=False)
        o = F.scaled_dot_product_attention(q.float(), kd.float(), vd.float(), scale=self.scale, enable_gqa=True)
        return o.to(torch.float16).view(1, self.hq, self.d)

    def _step(self, attend) -> None:
        m = self.model.model
        h = F.embedding(self.token, m.embed_tokens.weight)  # (1, 1, hidden)
        cos, sin = m.rotary_emb(h, self.pos)
        cos, sin = cos.unsqueeze(1), sin.unsqueeze(1)
        nq, nkv, half = self.hq * self.d, self.hkv * self.d, self.d // 2
        for i in range(self.L):
            x = self._rmsnorm(h, self.n_in[i])
            qkv = F.linear(x, self.wqkv[i])
            # apply_rotary_pos_emb of the query and key heads together: x * cos + rotate_half(x) * sin.
            qk = qkv[..., :nq + nkv].view(1, 1, self.hq + self.hkv, self.d).transpose(1, 2)
            qk = qk * cos + torch.cat((-qk[..., half:], qk[..., :half]), dim=-1) * sin
            q, k = qk[:, :self.hq], qk[:, self.hq:]
            v = qkv[..., nq + nkv:].view(1, 1, self.hkv, self.d).transpose(1, 2)
            o = attend(i, q, k, v)
            h = h + F.linear(o.reshape(1, 1, nq), self.wo[i])
            x = self._rmsnorm(h, self.n_post[i])
            g, u = F.linear(x, self.wgu[i]).chunk(2, dim=-1)
            h = h + F.linear(F.silu(g) * u, self.wd[i])
        h = self._rmsnorm(h, m.norm.weight)
        self.logits.copy_(F.linear(h, self.model.lm_head.weight)[:, 0].float())
        self.next.copy_(self.logits.argmax(-1, keepdim=True))
        self.pos.add_(1)

    # ------------------------------------------------------------------ capture / replay
    def capture(self) -> None:
        """Capture one decode step (``fused`` and ``dense`` attention).  The step's non-attention
        kernels are warmed first on a side stream with the attention left out, so the caches and
        the position are unchanged."""
        if self.attention == "decompressed":
            raise ValueError("the decompressed attention runs eagerly")
        with torch.no_grad():
            if self.turbo:
                q = torch.zeros((1, self.hq, self.d), dtype=torch.float16, device=self.dev)
                for rt, out in zip(self.rts, self.attn_out):
                    rt._workspace_for(self.hq)
                    tpgraph.launch_attention(rt, q, out, self.scale)  # kernel attributes; reads only
            saved = self.pos.clone()
            side = torch.cuda.Stream(self.dev)
            side.wait_stream(torch.cuda.current_stream(self.dev))
            with torch.cuda.stream(side):
                for _ in range(2):
                    self._step(lambda i, q, k, v: q.reshape(1, self.hq, self.d))
            torch.cuda.current_stream(self.dev).wait_stream(side)
            self.pos.copy_(saved)
            torch.cuda.synchronize(self.dev)
            self.graph = torch.cuda.CUDAGraph()
            with torch.cuda.graph(self.graph):
                self._step(self._attend)

    def step(self) -> None:
        """One decode step on ``token``: a graph replay, or the eager decompressed step."""
        if self.attention == "decompressed":
            with torch.no_grad():
                self._step(self._attend)
            return
        if self.graph is None:
            self.capture()
        if self.turbo:
            tpgraph._check_room(self.rts)
        if int(self.offset) + 1 > self.max_seq_len:
            raise RuntimeError("decode past max_seq_len")
        self.graph.replay()
        self.offset += 1
        if self.turbo:
            for rt in self.rts:
                tpgraph.advance_host(rt, 1)

    def decode(self, first_token: torch.Tensor, steps: int, forced: Optional[torch.Tensor] = None,
               logits_out: Optional[torch.Tensor] = None) -> float:
        """``steps`` decode steps from ``first_token`` ((1, 1) long): greedy, or fed ``forced``
        ((1, steps) long; forced[:, 0] must equal first_token).  Row t of ``logits_out`` receives
        the logits step t computes.  Returns the device seconds of the loop (CUDA events)."""
        self.token.copy_(first_token)
        start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        start.record()
        for t in range(steps):
            self.step()
            if logits_out is not None:
                logits_out[t].copy_(self.logits[0])
            if t + 1 < steps:
                self.token.copy_(forced[:, t + 1:t + 2] if forced is not None else self.next)
        end.record()
        torch.cuda.synchronize(self.dev)
        return start.elapsed_time(end) / 1e3

    def release(self) -> None:
        self.graph = None
