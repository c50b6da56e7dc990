"""``TurboPolarKVCacheRuntime`` with the page store, tail and counters on the device.

Mirrors ``rfsn_v11/generation/turbo_polar_cache.py``: same constructor, ``append``
validation (types, ranks, persistent invariants, finiteness; same exception types and
messages), tail / flush semantics, ``get_fused_attention_inputs``,
``get_blocks_for_attention``, ``fetch_blocks``, ``get_io_telemetry`` and ``reset``.  Adds
``attention(q, scale=None)``: fused decode attention over everything appended so far, the
read half of ``TurboPolarFastCache.decode_attention``
(``benchmarks/turbopolar_fast_attention.py:133-188``).

Device layout: a :class:`~turbopolar_b200.pages.PagePool` of ``batch * H_kv`` heads, a dense
tail ``[batch*H_kv, 64, 128]`` in the input dtype, and six int32 state words (pages, tail
length, sequence length, first page, error, ticket) that the append kernel advances on the
device, so a decode step can be replayed from a CUDA graph.  The host keeps a mirror of the
counters (the append semantics are deterministic in the input shapes), which is what the
Python API and the telemetry read; nothing here synchronises with the device except the
optional finiteness check the reference performs (``turbo_polar_cache.py:69-70``).

Batch: the reference runtime stores any batch size; here batch and KV heads are flattened
into one head axis, which every kernel handles unchanged.
"""

from __future__ import annotations

import ctypes
import math
from typing import Any, Dict, Optional, Tuple

import torch

from . import _lib, guard
from .codec import encode_pages, _stream
from .config import TurboPolarConfig
from .pages import PAGE, PagePool, page_bytes
from .payload import PolarKeyBlock, QuantizedVBlock, block_metadata


class TurboPolarKVCacheRuntime:
    """Stateful incremental KV cache with polar-coded keys and grouped int8 values in HBM.

    ``max_seq_len`` preallocates the page pool (no growth copies; required before capturing
    decode steps in a CUDA graph).  Without it the pool starts at 4 pages at the first flush
    and doubles when full, as the reference's storage does (``storage.py:57-87``).
    ``check_finite`` keeps the reference's host-synchronising finiteness check on appends.
    """

    def __init__(self, config: TurboPolarConfig, device=None, max_seq_len: Optional[int] = None,
                 check_finite: bool = True, first_page: int = 0):
        self.config = config
        self.fmt = config.format_fields()
        self.max_seq_len = max_seq_len
        self.check_finite = check_finite
        self._device_arg = device
        # Sequence shard: absolute index of local page 0 (tokens before it live on other ranks).
        self.first_page = int(first_page)
        self.reset()

    # ------------------------------------------------------------------ state
    def reset(self):
        """Clear all cache state and persistent invariants (``turbo_polar_cache.py:379-395``)."""
        self.pool: Optional[PagePool] = None
        self.tail_k: Optional[torch.Tensor] = None
        self.tail_v: Optional[torch.Tensor] = None
        self.d_state: Optional[torch.Tensor] = None
        self._workspace: Optional[torch.Tensor] = None
        self.n_pages = 0
        self.tail_len = 0
        self.qjl_blocks: list = []
        self.actual_seq_len = 0
        self.total_blocks = 0
        self.bytes_written = 0
        self.bytes_read = 0
        self.compression_time_ns = 0
        self.capacity = 0
        self.reallocation_count = 0
        self._initialized = False
        self._batch_size: Optional[int] = None
        self._num_kv_heads: Optional[int] = None
        self._head_dim: Optional[int] = None
        self._input_dtype = None
        self.device = torch.device(self._device_arg) if self._device_arg is not None else None

    @property
    def heads(self) -> int:
        return self._batch_size * self._num_kv_heads

    # ------------------------------------------------------------------ validation
    def _validate_append_inputs(self, k_new, v_new):
        if not isinstance(k_new, torch.Tensor) or not isinstance(v_new, torch.Tensor):
            raise TypeError("append() expects torch.Tensor inputs")
        if k_new.dim() != 4 or v_new.dim() != 4:
            raise ValueError(f"append() expects 4-D inputs (B, H_kv, T, D), got {tuple(k_new.shape)} and {tuple(v_new.shape)}")
        if k_new.shape != v_new.shape:
            raise ValueError(f"k_new shape {tuple(k_new.shape)} must match v_new shape {tuple(v_new.shape)}")
        B, H_kv, T_new, D = k_new.shape
        if T_new < 1:
            raise ValueError(f"input must have at least one token, got T={T_new}")
        if k_new.dtype != v_new.dtype:
            raise ValueError(f"k_new dtype {k_new.dtype} must match v_new dtype {v_new.dtype}")
        if k_new.dtype not in (torch.float16, torch.float32):
            raise ValueError(f"only float16 and float32 inputs are supported, got {k_new.dtype}")
        if not (k_new.is_cuda and v_new.is_cuda):
            raise ValueError("TurboPolar B200 cache inputs must be CUDA tensors")
        if self.check_finite and not bool(torch.isfinite(k_new).all() and torch.isfinite(v_new).all()):
            raise ValueError("append() inputs must contain finite values")
        if self._initialized:
            if B != self._batch_size:
                raise ValueError(f"batch size changed from {self._batch_size} to {B}; "
                                 "TurboPolar cache does not support varying batch size.")
            if H_kv != self._num_kv_heads:
                raise ValueError(f"KV head count changed from {self._num_kv_heads} to {H_kv}; "
                                 "TurboPolar cache does not support varying head counts.")
            if D != self._head_dim:
                raise ValueError(f"head_dim changed from {self._head_dim} to {D}; "
                                 "TurboPolar cache does not support varying head dimension.")
            if k_new.dtype != self._input_dtype:
                raise ValueError(f"input dtype changed from {self._input_dtype} to {k_new.dtype}; "
                                 "TurboPolar cache does not support varying dtype.")
            if k_new.device != self.device:
                raise ValueError(f"input device changed from {self.device} to {k_new.device}")
        else:
            if H_kv != self.config.num_kv_heads:
                raise ValueError(f"input has {H_kv} KV heads but config expects {self.config.num_kv_heads}")
            if D != self.config.head_dim:
                raise ValueError(f"input head_dim {D} does not match config {self.config.head_dim}")
            self._batch_size, self._num_kv_heads, self._head_dim = B, H_kv, D
            self._input_dtype = k_new.dtype
            self.device = k_new.device
            self._initialized = True
            self._allocate_tail()

    def _allocate_tail(self):
        dev = self.device
        self.tail_k = guard.zeros((self.heads, PAGE, 128), self._input_dtype, dev, "dense tail (K)")
        self.tail_v = guard.zeros((self.heads, PAGE, 128), self._input_dtype, dev, "dense tail (V)")
        self.d_state = guard.zeros((_lib.STATE_WORDS,), torch.int32, dev, "state words")
        if self.first_page:
            self.d_state[2] = self.first_page * PAGE
            self.d_state[3] = self.first_page
        if self.max_seq_len:
            self._ensure_capacity(max(1, math.ceil(self.max_seq_len / PAGE)))

    def _ensure_capacity(self, pages: int):
        if self.pool is not None and pages <= self.capacity:
            return
        if self.pool is None:
            cap = 4
            if self.max_seq_len:
                cap = max(cap, math.ceil(self.max_seq_len / PAGE))
            while cap < pages:
                # The reference allocates 4 blocks at the first flush and doubles one block
                # at a time; a bulk first append counts the same doublings.
                cap *= 2
                self.reallocation_count += 1
            self.pool = PagePool(self.heads, cap, self.fmt, self.device)
        else:
            cap = self.capacity
            while cap < pages:
                cap *= 2
                self.reallocation_count += 1
            self.pool = self.pool.grown(cap, self.n_pages)
        self.capacity = cap

    # ------------------------------------------------------------------ append
    def append(self, k_new: torch.Tensor, v_new: torch.Tensor):
        """Append ``(B, H_kv, T, 128)`` keys/values (``turbo_polar_cache.py:106-126``)."""
        self._validate_append_inputs(k_new, v_new)
        B, H, T, D = k_new.shape
        k = k_new.reshape(B * H, T, D)
        v = v_new.reshape(B * H, T, D)
        if k.stride(-1) != 1 or v.stride(-1) != 1 or k.stride() != v.stride():
            k, v = k.contiguous(), v.contiguous()
        lib = _lib.lib()
        stream = _stream(self.device)
        tail = _lib.Tail(self.tail_k.data_ptr(), self.tail_v.data_ptr(),
                         _lib.TP_F16 if self._input_dtype == torch.float16 else _lib.TP_F32)
        dcode = tail.dtype
        pos = 0
        while pos < T:
            left = T - pos
            if self.tail_len == 0 and left >= PAGE:
                # Whole blocks go straight from the input into the pool.
                n = left // PAGE
                self._ensure_capacity(self.n_pages + n)
                encode_pages(self.pool, k, v, n, self.n_pages, src_token0=pos, d_state=self.d_state)
                self._flushed(n)
                self.actual_seq_len += n * PAGE
                pos += n * PAGE
                continue
            n = min(PAGE - self.tail_len, left)
            fills = self.tail_len + n == PAGE
            if fills:
                self._ensure_capacity(self.n_pages + 1)
            pool_struct = self.pool.struct() if self.pool is not None else _lib.empty_pool(self.heads, self.fmt)
            src_k = k[:, pos:pos + n]
            src_v = v[:, pos:pos + n]
            _lib.check(lib.tp_append(ctypes.byref(pool_struct), ctypes.byref(tail), self.d_state.data_ptr(),
                                     src_k.data_ptr(), src_v.data_ptr(), dcode, k.stride(0), k.stride(1), n, stream))
            self.actual_seq_len += n
            if fills:
                self.tail_len = 0
                self._flushed(1)
            else:
                self.tail_len += n
            pos += n

    def _flushed(self, n: int):
        """Account ``n`` newly stored blocks (``turbo_polar_cache.py:133-161``)."""
        self.n_pages += n
        self.total_blocks += n
        self.bytes_written += n * self.pool.nbytes_valid(1)

    # ------------------------------------------------------------------ attention
    def _workspace_for(self, num_q_heads: int) -> torch.Tensor:
        need = _lib.lib().tp_decode_attention_workspace_size(self.heads, num_q_heads)
        if need == 0:
            raise ValueError("num_q_heads must be divisible by num_kv_heads for GQA")
        if self._workspace is None or self._workspace.numel() < need:
            self._workspace = torch.zeros(need, dtype=torch.uint8, device=self.device)
        return self._workspace

    def state(self) -> _lib.State:
        """Host mirror of the device state words; positions are absolute over the sequence."""
        return _lib.State(self.n_pages, self.tail_len,
                          self.first_page * PAGE + self.actual_seq_len + self.later_tokens, self.first_page)

    later_tokens = 0  # tokens held by shards after this one (sequence sharding)

    def set_global_length(self, total_tokens: int) -> None:
        """Declare the whole sequence's length when this runtime holds one shard of it, so no
        local position is masked (positions >= the sequence length are excluded)."""
        local_end = self.first_page * PAGE + self.actual_seq_len
        self.later_tokens = max(0, int(total_tokens) - local_end)
        if self.d_state is not None:
            self.d_state[2] = local_end + self.later_tokens

    def tail_struct(self) -> _lib.Tail:
        return _lib.Tail(self.tail_k.data_ptr(), self.tail_v.data_ptr(),
                         _lib.TP_F16 if self._input_dtype == torch.float16 else _lib.TP_F32)

    def pool_struct(self) -> _lib.PagePool:
        if self.pool is not None:
            return self.pool.struct()
        return _lib.empty_pool(self.heads, self.fmt)

    def attention(self, q: torch.Tensor, scale: Optional[float] = None, out: Optional[torch.Tensor] = None,
                  partial_out: Optional[torch.Tensor] = None, use_device_state: bool = False) -> torch.Tensor:
        """Decode attention of one query token over every appended token.

        ``q`` is ``(B, H_q, 128)`` or ``(B, H_q, 1, 128)``, float16 or float32; returns float16
        ``(B, H_q, 128)``.  ``partial_out`` (float32 ``[B*H_q, 130]``) receives unnormalised
        (max, sum, output) records instead, for a cross-shard merge.  ``use_device_state`` reads
        the counters from device memory (CUDA-graph replay) instead of the host mirror.
        """
        if not self._initialized or (self.n_pages == 0 and self.tail_len == 0):
            raise RuntimeError("TurboPolar cache returned no blocks after append")
        if q.dim() == 4:
            if q.shape[2] != 1:
                raise ValueError("decode attention only supports a single query token")
            q = q.squeeze(2)
        if q.dim() != 3 or q.shape[0] != self._batch_size or q.shape[-1] != self._head_dim:
            raise ValueError(f"query shape {tuple(q.shape)} does not match the cache (B={self._batch_size}, D=128)")
        if q.dtype not in (torch.float16, torch.float32):
            raise ValueError(f"query dtype must be float16 or float32, got {q.dtype}")
        if q.device != self.device:
            raise ValueError("query must be on the cache's device")
        B, Hq, D = q.shape
        if Hq % self._num_kv_heads:
            raise ValueError(f"decode_attention requires GQA ratio to divide evenly, got {Hq} and {self._num_kv_heads}")
        qf = q.reshape(B * Hq, D)
        if not qf.is_contiguous():
            qf = qf.contiguous()
        if out is None and partial_out is None:
            out = torch.empty((B, Hq, D), dtype=torch.float16, device=self.device)
        ws = self._workspace_for(B * Hq)
        scale = float(self.config.attention_scale if scale is None else scale)
        _lib.check(_lib.lib().tp_decode_attention(
            ctypes.byref(self.pool_struct()), ctypes.byref(self.tail_struct()), self.state(),
            self.d_state.data_ptr() if use_device_state else None, qf.data_ptr(),
            _lib.TP_F16 if qf.dtype == torch.float16 else _lib.TP_F32, B * Hq, scale,
            out.data_ptr() if out is not None else None,
            partial_out.data_ptr() if partial_out is not None else None,
            ws.data_ptr(), ws.numel(), _stream(self.device)))
        return out if out is not None else partial_out

    def decode_step(self, k_new: torch.Tensor, v_new: torch.Tensor, q: torch.Tensor, scale: Optional[float] = None,
                    out: Optional[torch.Tensor] = None, partial_out: Optional[torch.Tensor] = None) -> torch.Tensor:
        """``append(k_new, v_new)`` of one token then ``attention(q)``, as one tp_decode_step
        call (two kernels, no separate append kernel).  Same validation, results and host
        counters as the two calls; inputs of more than one token take that two-call path."""
        if k_new.dim() != 4 or k_new.shape[2] != 1 or not self._initialized or k_new.shape != v_new.shape:
            self.append(k_new, v_new)
            return self.attention(q, scale=scale, out=out, partial_out=partial_out)
        self._validate_append_inputs(k_new, v_new)
        if q.dim() == 4:
            if q.shape[2] != 1:
                raise ValueError("decode attention only supports a single query token")
            q = q.squeeze(2)
        if q.dim() != 3 or q.shape[0] != self._batch_size or q.shape[-1] != self._head_dim:
            raise ValueError(f"query shape {tuple(q.shape)} does not match the cache (B={self._batch_size}, D=128)")
        if q.dtype not in (torch.float16, torch.float32):
            raise ValueError(f"query dtype must be float16 or float32, got {q.dtype}")
        if q.device != self.device:
            raise ValueError("query must be on the cache's device")
        B, Hq, D = q.shape
        if Hq % self._num_kv_heads:
            raise ValueError(f"decode_attention requires GQA ratio to divide evenly, got {Hq} and {self._num_kv_heads}")
        fills = self.tail_len == PAGE - 1
        if fills:
            self._ensure_capacity(self.n_pages + 1)
        kf = k_new.reshape(self.heads, D)
        vf = v_new.reshape(self.heads, D)
        if kf.stride() != vf.stride() or kf.stride(-1) != 1 or kf.stride(0) % 8 or kf.data_ptr() % 16 \
                or vf.data_ptr() % 16:
            kf, vf = kf.contiguous(), vf.contiguous()
        qf = q.reshape(B * Hq, D)
        if not qf.is_contiguous():
            qf = qf.contiguous()
        if out is None and partial_out is None:
            out = torch.empty((B, Hq, D), dtype=torch.float16, device=self.device)
        ws = self._workspace_for(B * Hq)
        scale = float(self.config.attention_scale if scale is None else scale)
        _lib.check(_lib.lib().tp_decode_step(
            ctypes.byref(self.pool_struct()), ctypes.byref(self.tail_struct()), self.d_state.data_ptr(),
            kf.data_ptr(), vf.data_ptr(), _lib.TP_F16 if kf.dtype == torch.float16 else _lib.TP_F32, kf.stride(0),
            qf.data_ptr(), _lib.TP_F16 if qf.dtype == torch.float16 else _lib.TP_F32, B * Hq, scale,
            out.data_ptr() if out is not None else None,
            partial_out.data_ptr() if partial_out is not None else None,
            ws.data_ptr(), ws.numel(), _stream(self.device)))
        self.actual_seq_len += 1
        if fills:
            self.tail_len = 0
            self._flushed(1)
        else:
            self.tail_len += 1
        return out if out is not None else partial_out

    # ------------------------------------------------------------------ reference views
    def _views(self, n: int):
        """Reference-layout copies of pages [0, n) (``storage.py:89-102, :160-169``)."""
        B, H = self._batch_size, self._num_kv_heads
        ref = self.pool.export(0, n)
        k = PolarKeyBlock(
            radii=ref.radii.view(B, H, n, PAGE, 64),
            angle_codes_l1=ref.angle_codes_l1.view(B, H, n, PAGE, ref.l1_row),
            angle_codes_deep=ref.angle_codes_deep.view(B, H, n, PAGE, ref.deep_row),
            radii_scales=ref.radii_scales.view(B, H, n, 1, 1) if ref.radii_scales is not None else None,
            shape=(B, H, n * PAGE, self._head_dim), block_size=PAGE, head_dim=self._head_dim,
            metadata=block_metadata(self.fmt))
        v = QuantizedVBlock(codes=ref.v_codes.view(B, H, n, PAGE, 128), scales=ref.v_scales.view(B, H, n, PAGE, 4),
                            group_size=32)
        return k, v

    def _tail_views(self):
        if self.tail_len == 0:
            return None, None
        B, H, t = self._batch_size, self._num_kv_heads, self.tail_len
        return self.tail_k[:, :t].view(B, H, t, 128), self.tail_v[:, :t].view(B, H, t, 128)

    @property
    def partial_k(self):
        return self._tail_views()[0] if self._initialized else None

    @property
    def partial_v(self):
        return self._tail_views()[1] if self._initialized else None

    def get_fused_attention_inputs(self) -> Tuple[Optional[PolarKeyBlock], Optional[QuantizedVBlock],
                                                  Optional[torch.Tensor], Optional[torch.Tensor], None, int]:
        """Fused-attention inputs without re-encoding the tail (``turbo_polar_cache.py:163-198``):
        the stored blocks as reference-layout copies and the tail as views of the live buffer."""
        k = v = None
        if self.n_pages > 0:
            k, v = self._views(self.n_pages)
        tk, tv = self._tail_views() if self._initialized else (None, None)
        return k, v, tk, tv, None, self.actual_seq_len

    def _encode_padded_tail(self) -> Optional[PagePool]:
        """The tail zero-padded to one block and encoded (``turbo_polar_cache.py:276-319``)."""
        if not self._initialized or self.tail_len == 0:
            return None
        padded_k = torch.zeros_like(self.tail_k)
        padded_v = torch.zeros_like(self.tail_v)
        padded_k[:, :self.tail_len] = self.tail_k[:, :self.tail_len]
        padded_v[:, :self.tail_len] = self.tail_v[:, :self.tail_len]
        tmp = PagePool(self.heads, 1, self.fmt, self.device)
        encode_pages(tmp, padded_k, padded_v, 1, 0)
        return tmp

    def get_blocks_for_attention(self):
        """Decompress-on-read inputs: stored blocks plus the padded, encoded tail
        (``turbo_polar_cache.py:200-274``).  Returns (block, quant_v, None, None, actual_seq_len)."""
        part = self._encode_padded_tail()
        if self.n_pages == 0 and part is None:
            return None, None, None, None, self.actual_seq_len
        B, H = self._batch_size, self._num_kv_heads
        refs = []
        if self.n_pages:
            refs.append(self.pool.export(0, self.n_pages))
        if part is not None:
            refs.append(part.export(0, 1))
        cat = lambda name: torch.cat([getattr(r, name) for r in refs], dim=1)
        n = sum(r.capacity for r in refs)
        l1, deep = cat("angle_codes_l1"), cat("angle_codes_deep")
        k = PolarKeyBlock(
            radii=cat("radii").view(B, H, n, PAGE, 64),
            angle_codes_l1=l1.view(B, H, n, PAGE, l1.shape[-1]),
            angle_codes_deep=deep.view(B, H, n, PAGE, deep.shape[-1]),
            radii_scales=cat("radii_scales").view(B, H, n, 1, 1) if self.fmt["int8_radii"] else None,
            shape=(B, H, n * PAGE, self._head_dim), block_size=PAGE, head_dim=self._head_dim,
            metadata=block_metadata(self.fmt))
        v = QuantizedVBlock(codes=cat("v_codes").view(B, H, n, PAGE, 128),
                            scales=cat("v_scales").view(B, H, n, PAGE, 4), group_size=32)
        return k, v, None, None, self.actual_seq_len

    def decompress(self, padded_tail: bool = True) -> Tuple[torch.Tensor, torch.Tensor]:
        """Dense float16 K and V ``(B, H, actual_seq_len, 128)`` as the decompress-on-read path
        sees them: stored blocks plus, with ``padded_tail``, the tail encoded and decoded too
        (``benchmarks/turbopolar_fast_attention.py:56-86``)."""
        B, H = self._batch_size, self._num_kv_heads
        part = self._encode_padded_tail() if padded_tail else None
        lib = _lib.lib()
        s = _stream(self.device)

        def decode(pool: PagePool, n: int):
            # tp_decode_pages writes [heads][n * 64][128].
            kk = torch.empty((self.heads, n * PAGE, 128), dtype=torch.float16, device=self.device)
            vv = torch.empty_like(kk)
            _lib.check(lib.tp_decode_pages(ctypes.byref(pool.struct()), 0, n, kk.data_ptr(), vv.data_ptr(), s))
            return kk, vv

        parts = []
        if self.n_pages:
            parts.append(decode(self.pool, self.n_pages))
        if part is not None:
            parts.append(decode(part, 1))
        if not parts:
            k = torch.empty((self.heads, 0, 128), dtype=torch.float16, device=self.device)
            v = torch.empty_like(k)
        elif len(parts) == 1:
            k, v = parts[0]
        else:
            k = torch.cat([p_[0] for p_ in parts], dim=1)
            v = torch.cat([p_[1] for p_ in parts], dim=1)
        if not padded_tail and self.tail_len:
            k = torch.cat([k, self.tail_k[:, :self.tail_len].to(torch.float16)], dim=1)
            v = torch.cat([v, self.tail_v[:, :self.tail_len].to(torch.float16)], dim=1)
        L = self.actual_seq_len
        return k[:, :L].view(B, H, L, 128), v[:, :L].view(B, H, L, 128)

    def fetch_blocks(self, indices: Optional[list] = None) -> torch.Tensor:
        """Decode stored blocks to dense keys (``turbo_polar_cache.py:321-346``)."""
        if self.n_pages == 0:
            return torch.empty(0, device=self.device)
        if indices is None:
            indices = list(range(self.n_pages))
        B, H = self._batch_size, self._num_kv_heads
        out = torch.empty((self.heads, len(indices) * PAGE, 128), dtype=torch.float16, device=self.device)
        scratch_v = torch.empty_like(out[:, :PAGE])
        kb = PAGE * 64 * (1 if self.fmt["int8_radii"] else 2) + PAGE * (self.pool.l1_row + self.pool.deep_row)
        kb += 2 if self.fmt["int8_radii"] else 0
        for i, idx in enumerate(indices):
            if not 0 <= idx < self.n_pages:
                raise IndexError(f"block index {idx} out of range")
            dst = out[:, i * PAGE:(i + 1) * PAGE]
            tmp = torch.empty((self.heads, PAGE, 128), dtype=torch.float16, device=self.device)
            _lib.check(_lib.lib().tp_decode_pages(ctypes.byref(self.pool.struct()), idx, 1, tmp.data_ptr(),
                                                  scratch_v.data_ptr(), _stream(self.device)))
            dst.copy_(tmp)
            self.bytes_read += self.heads * kb
        return out.view(B, H, len(indices) * PAGE, 128)

    # ------------------------------------------------------------------ telemetry
    @property
    def k_storage_capacity(self) -> int:
        return self.capacity

    def get_io_telemetry(self) -> Dict[str, Any]:
        """Byte accounting with the reference's keys and arithmetic (``turbo_polar_cache.py:348-377``)."""
        if self.n_pages == 0 and self.tail_len == 0:
            return {}
        D = self.config.head_dim
        B, H = self._batch_size, self._num_kv_heads
        dense = B * H * self.actual_seq_len * D * 2 * 2
        comp = self.bytes_written
        if self.tail_len:
            comp += 2 * B * H * self.tail_len * D * self.tail_k.element_size()
        return {
            "dense_kv_bytes": dense,
            "actual_cache_bytes": comp,
            "compression_ratio": float(dense / comp) if comp > 0 else 0.0,
            "total_blocks": self.total_blocks,
            "partial_tokens": self.tail_len,
            "k_storage_capacity": self.capacity,
            "v_storage_capacity": self.capacity,
            "k_storage_reallocs": self.reallocation_count,
            "v_storage_reallocs": self.reallocation_count,
        }

    def read_device_error(self) -> int:
        """The append kernel's error word (0 ok, 1 tail overflow, 2 pool full); synchronises."""
        return int(self.d_state[4].item()) if self.d_state is not None else 0

    def compressed_bytes_per_token(self) -> int:
        """Page bytes per token summed over heads (algorithmic bytes the attention streams)."""
        return self.heads * page_bytes(self.fmt) // PAGE if self._initialized else 0
