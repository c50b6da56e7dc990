"""Cache-runtime bookkeeping restated in NumPy (oracle; test infrastructure only).

Follows ``rfsn_v11/generation/turbo_polar_cache.py``:

* ``append`` / ``_flush_block`` (``:106-161``): tokens accumulate in a dense tail; every
  full 64-token block is encoded (polar K, grouped int8 V) and appended to block storage;
  ``bytes_written`` adds the payload bytes of each flushed block;
* ``get_fused_attention_inputs`` (``:163-198``): stored blocks plus the raw tail;
* ``get_blocks_for_attention`` / ``_maybe_encode_partial`` (``:200-319``): the tail
  zero-padded to 64 tokens and encoded as one more block (decompress-on-read path);
* ``get_io_telemetry`` (``:348-377``) with the capacity growth of
  ``rfsn_v11/generation/storage.py:57-87`` (initial capacity 4, doubling).

Arrays carry the batch dimension (B=1) exactly like the reference's.
"""

from __future__ import annotations

import numpy as np

from . import polar, vquant

BLOCK = 64


class CacheModel:
    def __init__(self, num_kv_heads: int, l1_bits=4, deep_bits=4, split_dim=64, int8_radii=False):
        self.h = num_kv_heads
        self.fmt = dict(l1_bits=l1_bits, deep_bits=deep_bits, split_dim=split_dim)
        self.int8_radii = int8_radii
        self.blocks = []          # list of dicts (encoded block payloads, batch dim kept)
        self.partial_k = None
        self.partial_v = None
        self.actual_seq_len = 0
        self.bytes_written = 0
        self.capacity = 0
        self.reallocs = 0

    def _encode(self, k_block, v_block):
        enc = polar.encode_block(k_block, int8_radii=self.int8_radii, **self.fmt)
        codes, scales = vquant.quantize(v_block)
        return {
            "radii": enc["radii"], "angle_codes_l1": enc["angle_codes_l1"],
            "angle_codes_deep": enc["angle_codes_deep"], "radii_scales": enc["radii_scales"],
            "v_codes": codes, "v_scales": scales,
        }

    def append(self, k_new: np.ndarray, v_new: np.ndarray):
        t = k_new.shape[2]
        self.actual_seq_len += t
        if self.partial_k is None:
            self.partial_k, self.partial_v = k_new, v_new
        else:
            self.partial_k = np.concatenate([self.partial_k, k_new], axis=2)
            self.partial_v = np.concatenate([self.partial_v, v_new], axis=2)
        while self.partial_k is not None and self.partial_k.shape[2] >= BLOCK:
            blk = self._encode(self.partial_k[:, :, :BLOCK], self.partial_v[:, :, :BLOCK])
            self.blocks.append(blk)
            # storage.py:75-87 -- lazy init at capacity 4, doubling when full.
            if self.capacity == 0:
                self.capacity = 4
            elif len(self.blocks) > self.capacity:
                self.capacity *= 2
                self.reallocs += 1
            self.bytes_written += sum(int(np.asarray(blk[f]).nbytes) for f in
                                      ("radii", "angle_codes_l1", "angle_codes_deep", "v_codes", "v_scales"))
            if blk["radii_scales"] is not None:
                self.bytes_written += int(blk["radii_scales"].nbytes)
            self.partial_k = self.partial_k[:, :, BLOCK:]
            self.partial_v = self.partial_v[:, :, BLOCK:]
            if self.partial_k.shape[2] == 0:
                self.partial_k = self.partial_v = None

    @property
    def total_blocks(self) -> int:
        return len(self.blocks)

    def pages(self) -> dict | None:
        """Stored blocks stacked on a block axis, reference unified shapes without B:
        ``radii (H,S,64,64)``, ``radii_scales (H,S)``, ``v_scales (H,S,64,4)`` ..."""
        if not self.blocks:
            return None
        out = {}
        for f in ("radii", "angle_codes_l1", "angle_codes_deep", "v_codes", "v_scales"):
            out[f] = np.stack([b[f][0] for b in self.blocks], axis=1)
        if self.blocks[0]["radii_scales"] is not None:
            out["radii_scales"] = np.stack([b["radii_scales"][0, :, 0, 0] for b in self.blocks], axis=1)
        else:
            out["radii_scales"] = None
        return out

    def padded_partial(self) -> dict | None:
        """The tail zero-padded to one block and encoded (``turbo_polar_cache.py:276-319``)."""
        if self.partial_k is None:
            return None
        pad = BLOCK - self.partial_k.shape[2]
        widths = [(0, 0), (0, 0), (0, pad), (0, 0)]
        return self._encode(np.pad(self.partial_k, widths), np.pad(self.partial_v, widths))

    def telemetry(self) -> dict:
        if not self.blocks and self.partial_k is None:
            return {}
        b = 1
        dense = b * self.h * self.actual_seq_len * polar.HEAD_DIM * 2 * 2
        comp = self.bytes_written
        if self.partial_k is not None:
            comp += int(self.partial_k.nbytes) + int(self.partial_v.nbytes)
        return {
            "dense_kv_bytes": dense,
            "actual_cache_bytes": comp,
            "compression_ratio": float(dense / comp) if comp > 0 else 0.0,
            "total_blocks": self.total_blocks,
            "partial_tokens": self.partial_k.shape[2] if self.partial_k is not None else 0,
            "k_storage_capacity": self.capacity,
            "v_storage_capacity": self.capacity,
            "k_storage_reallocs": self.reallocs,
            "v_storage_reallocs": self.reallocs,
        }
