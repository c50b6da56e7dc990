"""PyTorch Llama adapter: the TurboPolar compressed KV cache inside Hugging Face Llama models.

Replaces the reference's mlx_lm adapter (``benchmarks/turbopolar_fast_attention.py:20-298``)
with the same names and behaviour:

* ``TurboPolarFastCache`` -- one layer's cache (``:20-204``): ``offset``, ``update_and_fetch``
  (prefill: append, then decompress-on-read of the whole history, the tail padded, encoded
  and decoded like the stored blocks, ``:56-86``), ``decode_attention`` (append one token
  and run the fused CUDA decode attention over pages + dense tail, ``:106-188``), ``size``,
  ``nbytes``, ``empty``.  It is also a ``transformers`` cache layer, so a list of them is a
  ``past_key_values`` object (``TurboPolarCache``).
* ``make_turbo_caches`` (``:207-229``): the adapter key format (int8 log radii, 8-bit deep
  angles, ``split_dim=0``).
* ``patch_llama_attention`` / ``unpatch_llama_attention`` (``:281-298``): swap
  ``LlamaAttention.forward`` so single-token steps with a TurboPolar cache take the fused
  path (``_turbo_attention_call``, ``:247-278``) and everything else runs the stock forward.

Where the reference runs its dense MLX attention for a cache with no full block yet
(``:149-159``), the CUDA kernel handles that case itself (tail-only attention).
"""

from __future__ import annotations

from typing import Any, List, Optional, Tuple

import torch
from transformers.cache_utils import Cache, CacheLayerMixin

from .bridge import CudaKernelBridge
from .cache import TurboPolarKVCacheRuntime
from .codec import GroupedVQuantizer, PolarQuantDecoder
from .config import TurboPolarConfig


class TurboPolarFastCache(CacheLayerMixin):
    """One decoder layer's TurboPolar cache: fused CUDA attention for decode steps,
    decompress-on-read for prefill."""

    is_compileable = False
    is_sliding = False

    def __init__(self, config: TurboPolarConfig, device=None, max_seq_len: Optional[int] = None,
                 check_finite: bool = True):
        super().__init__()
        self.config = config
        # check_finite keeps the reference's finiteness check on every append
        # (turbo_polar_cache.py:69-70), one host synchronisation per layer and token; without it
        # nothing on the decode path synchronises (runtime.read_device_error() reads the
        # device's error word when the caller chooses to).
        self.runtime = TurboPolarKVCacheRuntime(config, device=device, max_seq_len=max_seq_len,
                                                check_finite=check_finite)
        self.bridge = CudaKernelBridge()
        self.decoder = PolarQuantDecoder()
        self.v_dequantizer = GroupedVQuantizer(group_size=32)
        self.qjl_encoder = None  # QJL is rejected by the configuration contract

    # ------------------------------------------------------------------ reference API
    @property
    def offset(self) -> int:
        """Sequence length; the RoPE position of the next token."""
        return self.runtime.actual_seq_len

    def update_and_fetch(self, keys: torch.Tensor, values: torch.Tensor) -> Tuple[torch.Tensor, torch.Tensor]:
        """Prefill path: append ``(B, H_kv, T, 128)`` keys/values and return the decompressed
        history ``(B, H_kv, offset, 128)`` in the input dtype."""
        original_dtype = keys.dtype
        if keys.dtype != torch.float16:
            keys = keys.to(torch.float16)
        if values.dtype != torch.float16:
            values = values.to(torch.float16)
        self.runtime.append(keys, values)
        if self.runtime.actual_seq_len == 0:
            raise RuntimeError("TurboPolar cache returned no blocks after append")
        k_dense, v_dense = self.runtime.decompress(padded_tail=True)
        if original_dtype != k_dense.dtype:
            k_dense = k_dense.to(original_dtype)
            v_dense = v_dense.to(original_dtype)
        return k_dense, v_dense

    @staticmethod
    def _validate_decode_shape(q: torch.Tensor, k_new: torch.Tensor, v_new: torch.Tensor, config: TurboPolarConfig):
        if q.dim() != 4 or k_new.dim() != 4 or v_new.dim() != 4:
            raise ValueError("decode_attention inputs must be 4-D (B, H, T, D)")
        B, H_q, T, D = q.shape
        _, H_kv, T_k, _ = k_new.shape
        _, _, T_v, _ = v_new.shape
        if B != 1:
            raise NotImplementedError("TurboPolar fused decode only supports batch size 1.")
        if T != 1 or T_k != 1 or T_v != 1:
            raise ValueError("decode_attention only supports a single query/key/value token")
        if D != 128:
            raise NotImplementedError("TurboPolar fused decode only supports head_dim == 128.")
        if D != config.head_dim:
            raise ValueError(f"decode_attention head_dim {D} does not match config {config.head_dim}")
        if H_q % H_kv != 0:
            raise ValueError(f"decode_attention requires GQA ratio to divide evenly, got {H_q} and {H_kv}")

    def decode_attention(self, q: torch.Tensor, k_new: torch.Tensor, v_new: torch.Tensor,
                         scale: float) -> torch.Tensor:
        """Decode path: append one token and run fused attention.

        ``q`` ``(B, H_q, 1, D)`` and ``k_new, v_new`` ``(B, H_kv, 1, D)`` are RoPE'd; returns
        ``(B, H_q, D)`` float16 attention output."""
        self._validate_decode_shape(q, k_new, v_new, self.config)
        if k_new.dtype != torch.float16:
            k_new = k_new.to(torch.float16)
        if v_new.dtype != torch.float16:
            v_new = v_new.to(torch.float16)
        q_squeezed = q.squeeze(2)
        if q_squeezed.dtype not in (torch.float16, torch.float32):
            q_squeezed = q_squeezed.to(torch.float16)
        # Append and attention in one tp_decode_step call.
        return self.runtime.decode_step(k_new, v_new, q_squeezed, scale=scale)

    def size(self) -> int:
        return self.offset

    @property
    def nbytes(self) -> int:
        telem = self.runtime.get_io_telemetry()
        return int(telem.get("actual_cache_bytes", 0))

    def empty(self) -> bool:
        return self.offset == 0

    # ------------------------------------------------------------------ transformers cache layer
    def lazy_initialization(self, key_states: torch.Tensor, value_states: torch.Tensor) -> None:
        self.is_initialized = True

    def update(self, key_states: torch.Tensor, value_states: torch.Tensor, *args, **kwargs):
        self.is_initialized = True
        return self.update_and_fetch(key_states, value_states)

    def get_seq_length(self) -> int:
        return self.offset

    def get_mask_sizes(self, query_length: int) -> Tuple[int, int]:
        return self.offset + query_length, 0

    def get_max_cache_shape(self) -> int:
        return -1

    def reset(self) -> None:
        self.runtime.reset()

    def offload(self):
        raise NotImplementedError("TurboPolar caches stay on the GPU")

    def prefetch(self):
        pass


class TurboPolarCache(Cache):
    """``past_key_values`` for a Hugging Face model: one ``TurboPolarFastCache`` per layer.
    Indexing and iteration give the layers, as the reference's list of caches does."""

    def __init__(self, layers: List[TurboPolarFastCache]):
        super().__init__(layers=list(layers))

    def __getitem__(self, i):
        return self.layers[i]

    def __iter__(self):
        return iter(self.layers)


def make_turbo_caches(num_layers: int, num_q_heads: int, num_kv_heads: int, head_dim: int, use_qjl: bool = False,
                      device=None, max_seq_len: Optional[int] = None, check_finite: bool = True) -> TurboPolarCache:
    """Per-layer caches with the adapter's benchmark format (int8 log radii, 8-bit deep
    angles, every pair in the deep level)."""
    if head_dim not in (64, 128):
        raise ValueError(f"TurboPolar only supports head_dim 64 or 128, got {head_dim}")
    config = TurboPolarConfig(
        num_q_heads=num_q_heads,
        num_kv_heads=num_kv_heads,
        head_dim=head_dim,
        block_size=64,
        qjl_proj_dim=32 if head_dim == 64 else 64,
        use_qjl=use_qjl,
        storage_mode="kv_quant",
        use_int8_radii=True,
        k_angle_bits_deep=8,
        split_dim=0,
    )
    return TurboPolarCache([TurboPolarFastCache(config, device=device, max_seq_len=max_seq_len,
                                                check_finite=check_finite) for _ in range(num_layers)])


def _is_standard_causal_mask(mask: Optional[torch.Tensor], seq_len: int, cache_len: int) -> bool:
    """True for no mask or the full-history causal mask of shape ``(1, 1, seq_len, cache_len)``:
    query row i may see keys ``[0, cache_len - seq_len + i]``.  Boolean masks mark visible
    keys True; additive float masks hold 0 where visible and a large negative value elsewhere.

    The reference states the same rule (``turbopolar_fast_attention.py:235-244``) but builds
    its expected mask with an unshifted ``tril``, which for one query row over a longer cache
    admits only key 0; the diagonal here is shifted by ``cache_len - seq_len`` so that the
    documented full-history mask is the one accepted."""
    if mask is None:
        return True
    if tuple(mask.shape) != (1, 1, seq_len, cache_len):
        return False
    expected = torch.ones((seq_len, cache_len), dtype=torch.bool, device=mask.device).tril(cache_len - seq_len)
    if mask.dtype == torch.bool:
        visible = mask[0, 0]
    else:
        m = mask[0, 0]
        if bool(((m != 0) & (m > torch.finfo(m.dtype).min / 2)).any()):
            return False
        visible = m == 0
    return bool(torch.equal(visible, expected))


_orig_llama_attention_forward: Optional[Any] = None


def _turbo_attention_forward(self, hidden_states: torch.Tensor, position_embeddings=None, attention_mask=None,
                             past_key_values=None, **kwargs):
    layer = None
    if isinstance(past_key_values, TurboPolarCache) and self.layer_idx < len(past_key_values.layers):
        layer = past_key_values.layers[self.layer_idx]
    if isinstance(layer, TurboPolarFastCache) and hidden_states.shape[1] == 1:
        from transformers.models.llama.modeling_llama import apply_rotary_pos_emb
        n_heads = self.config.num_attention_heads
        n_kv_heads = self.config.num_key_value_heads
        if n_heads % n_kv_heads != 0:
            raise ValueError("TurboPolar fused decode requires GQA ratio to divide evenly.")
        if not _is_standard_causal_mask(attention_mask, hidden_states.shape[1], layer.offset + hidden_states.shape[1]):
            raise NotImplementedError("TurboPolar fused decode only supports standard causal full-history masks.")
        B, L, _ = hidden_states.shape
        hidden_shape = (B, L, -1, self.head_dim)
        queries = self.q_proj(hidden_states).view(hidden_shape).transpose(1, 2)
        keys = self.k_proj(hidden_states).view(hidden_shape).transpose(1, 2)
        values = self.v_proj(hidden_states).view(hidden_shape).transpose(1, 2)
        cos, sin = position_embeddings
        queries, keys = apply_rotary_pos_emb(queries, keys, cos, sin)
        output = layer.decode_attention(queries, keys, values, self.scaling)  # (B, H_q, D)
        output = output.to(hidden_states.dtype).reshape(B, L, -1)
        return self.o_proj(output), None
    return _orig_llama_attention_forward(self, hidden_states, position_embeddings, attention_mask, past_key_values,
                                         **kwargs)


def patch_llama_attention(model=None) -> None:
    """Route ``LlamaAttention.forward`` through the TurboPolar decode path when the layer's
    cache is a ``TurboPolarFastCache`` and one token is decoded."""
    from transformers.models.llama import modeling_llama
    global _orig_llama_attention_forward
    if _orig_llama_attention_forward is None:
        _orig_llama_attention_forward = modeling_llama.LlamaAttention.forward
    modeling_llama.LlamaAttention.forward = _turbo_attention_forward


def unpatch_llama_attention(model=None) -> None:
    """Restore the stock ``LlamaAttention.forward``."""
    from transformers.models.llama import modeling_llama
    global _orig_llama_attention_forward
    if _orig_llama_attention_forward is not None:
        modeling_llama.LlamaAttention.forward = _orig_llama_attention_forward
        _orig_llama_attention_forward = None
