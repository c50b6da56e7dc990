"""Device page pool: the block store, resident in HBM.

Replaces ``PolarKBlockStorage`` / ``QuantVBlockStorage``
(``rfsn_v11/generation/storage.py:17-169``).  :class:`PagePool` holds every page of every head
as one contiguous page block of two units (half pages); a unit is radii | value codes | angle
codes | value scales (``include/turbopolar.h``), so the decode kernel streams a half page with
one bulk copy.  The codes are the reference's bit for bit.  :class:`BlockStore` is the
reference's own layout, one array per field (``storage.py:89-102, :160-169``);
:meth:`PagePool.export` produces one and :meth:`PagePool.from_reference` loads one.  ``heads``
is batch x KV heads.
"""

from __future__ import annotations

import ctypes

import torch

from . import _lib, guard

PAGE = 64
HEAD_DIM = 128


def row_bytes(fmt: dict):
    l1 = ctypes.c_int32()
    deep = ctypes.c_int32()
    _lib.check(_lib.lib().tp_row_bytes(ctypes.byref(_lib.fmt_struct(fmt)), ctypes.byref(l1), ctypes.byref(deep)))
    return l1.value, deep.value


def unit_bytes(fmt: dict) -> int:
    """Bytes of one unit (half page of one head) in the kernel layout."""
    u = ctypes.c_int32()
    _lib.check(_lib.lib().tp_unit_bytes(ctypes.byref(_lib.fmt_struct(fmt)), ctypes.byref(u)))
    return u.value


def page_bytes(fmt: dict) -> int:
    """Compressed bytes per page per head (K and V payload, radius scale included), the
    reference's accounting (``turbo_polar_cache.py:154-161``)."""
    l1, deep = row_bytes(fmt)
    radii = PAGE * 64 * (1 if fmt["int8_radii"] else 2)
    return radii + PAGE * (l1 + deep) + PAGE * HEAD_DIM + PAGE * 4 * 2 + (2 if fmt["int8_radii"] else 0)


def _stream(device) -> int:
    return torch.cuda.current_stream(device).cuda_stream


def _ptr(t):
    return t.data_ptr() if (t is not None and t.numel() > 0) else None


class BlockStore:
    """Pages in the reference's block-storage layout: ``radii [heads, cap, 64, 64]``,
    ``angle_codes_l1 / _deep [heads, cap, 64, row]``, ``radii_scales [heads, cap]`` (int8 radii),
    ``v_codes`` int8 ``[heads, cap, 64, 128]``, ``v_scales [heads, cap, 64, 4]``.  Without
    ``keys`` the key fields are ``None`` (values only)."""

    def __init__(self, heads: int, capacity: int, fmt: dict, device, keys: bool = True):
        self.heads, self.capacity, self.fmt, self.device = heads, capacity, dict(fmt), torch.device(device)
        self.l1_row, self.deep_row = row_bytes(self.fmt)
        dev = self.device
        if keys:
            rdt = torch.int8 if fmt["int8_radii"] else torch.float16
            self.radii = torch.zeros((heads, capacity, PAGE, 64), dtype=rdt, device=dev)
            self.radii_scales = (torch.zeros((heads, capacity), dtype=torch.float16, device=dev)
                                 if fmt["int8_radii"] else None)
            self.angle_codes_l1 = torch.zeros((heads, capacity, PAGE, self.l1_row), dtype=torch.uint8, device=dev)
            self.angle_codes_deep = torch.zeros((heads, capacity, PAGE, self.deep_row), dtype=torch.uint8, device=dev)
        else:
            self.radii = self.radii_scales = self.angle_codes_l1 = self.angle_codes_deep = None
        self.v_codes = torch.zeros((heads, capacity, PAGE, HEAD_DIM), dtype=torch.int8, device=dev)
        self.v_scales = torch.zeros((heads, capacity, PAGE, 4), dtype=torch.float16, device=dev)
        self._struct = None

    @classmethod
    def wrap(cls, radii, angle_codes_l1, angle_codes_deep, radii_scales, v_codes, v_scales, fmt: dict):
        """Wrap caller tensors in the reference layout, shaped ``[heads, S, 64, .]`` (contiguous)."""
        self = cls.__new__(cls)
        ref = v_codes if v_codes is not None else radii
        self.heads, self.capacity = int(ref.shape[0]), int(ref.shape[1])
        self.fmt, self.device = dict(fmt), ref.device
        self.l1_row, self.deep_row = row_bytes(self.fmt)
        self.radii, self.angle_codes_l1, self.angle_codes_deep = radii, angle_codes_l1, angle_codes_deep
        self.radii_scales, self.v_codes, self.v_scales = radii_scales, v_codes, v_scales
        self._struct = None
        return self

    def struct(self) -> _lib.BlockStore:
        if self._struct is None:
            self._struct = _lib.BlockStore(_ptr(self.radii), _ptr(self.radii_scales), _ptr(self.angle_codes_l1),
                                           _ptr(self.angle_codes_deep), _ptr(self.v_codes), _ptr(self.v_scales),
                                           self.heads, self.capacity, _lib.fmt_struct(self.fmt))
        return self._struct


class PagePool:
    """``pages`` uint8 ``[heads, capacity, 2 * unit_bytes]`` plus ``radii_scales``
    ``[heads, capacity]`` float16 for int8 radii."""

    def __init__(self, heads: int, capacity: int, fmt: dict, device):
        self.heads, self.capacity, self.fmt, self.device = heads, capacity, dict(fmt), torch.device(device)
        self.l1_row, self.deep_row = row_bytes(self.fmt)
        self.unit_bytes = unit_bytes(self.fmt)
        self.pages = guard.zeros((heads, capacity, 2 * self.unit_bytes), torch.uint8, self.device, "page pool")
        self.radii_scales = (guard.zeros((heads, capacity), torch.float16, self.device, "radius scales")
                             if fmt["int8_radii"] else None)
        self._struct = None

    @classmethod
    def from_reference(cls, ref: BlockStore) -> "PagePool":
        """A pool holding the pages of a reference-layout block store."""
        pool = cls(ref.heads, ref.capacity, ref.fmt, ref.device)
        if ref.capacity:
            _lib.check(_lib.lib().tp_import_pages(ctypes.byref(pool.struct()), 0, ref.capacity,
                                                  ctypes.byref(ref.struct()), _stream(ref.device)))
        return pool

    def export(self, first: int, n: int, keys: bool = True) -> BlockStore:
        """Pages ``[first, first + n)`` in the reference layout (a new store of capacity ``n``)."""
        ref = BlockStore(self.heads, n, self.fmt, self.device, keys=keys)
        if n:
            _lib.check(_lib.lib().tp_export_pages(ctypes.byref(self.struct()), first, n, ctypes.byref(ref.struct()),
                                                  _stream(self.device)))
        return ref

    def struct(self) -> _lib.PagePool:
        if self._struct is None:
            self._struct = _lib.PagePool(_ptr(self.pages), _ptr(self.radii_scales), self.heads, self.capacity,
                                         _lib.fmt_struct(self.fmt))
        return self._struct

    def grown(self, new_capacity: int, n_valid: int) -> "PagePool":
        """A larger pool holding a device copy of the first ``n_valid`` pages of every head."""
        new = PagePool(self.heads, new_capacity, self.fmt, self.device)
        if guard.enabled():  # this pool is dropped once the copy is taken
            guard.check_tensor(self.pages)
            if self.radii_scales is not None:
                guard.check_tensor(self.radii_scales)
        if n_valid:
            new.pages[:, :n_valid].copy_(self.pages[:, :n_valid])
            if self.radii_scales is not None:
                new.radii_scales[:, :n_valid].copy_(self.radii_scales[:, :n_valid])
        return new

    def nbytes_valid(self, n_pages: int) -> int:
        return self.heads * n_pages * page_bytes(self.fmt)
