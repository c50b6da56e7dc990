"""Device page pool: the structure-of-arrays block store, resident in HBM.

Replaces ``PolarKBlockStorage`` / ``QuantVBlockStorage``
(``rfsn_v11/generation/storage.py:17-169``).  One tensor per field, shaped
``[heads, capacity, 64, row]`` with every page of a head contiguous, so the kernels stream a
head's pages as five contiguous byte ranges and the reference's unified views
(``storage.py:89-102, :160-169``) are zero-copy slices.  ``heads`` is batch x KV heads.
"""

from __future__ import annotations

import ctypes

import torch

from . import _lib

PAGE = 64
HEAD_DIM = 128


def row_bytes(fmt: dict):
    f = _lib.Format(fmt["l1_bits"], fmt["deep_bits"], fmt["split_dim"], fmt["int8_radii"])
    l1 = ctypes.c_int32()
    deep = ctypes.c_int32()
    _lib.check(_lib.lib().tp_row_bytes(ctypes.byref(f), ctypes.byref(l1), ctypes.byref(deep)))
    return l1.value, deep.value


def page_bytes(fmt: dict) -> int:
    """Compressed bytes per page per head (K and V payload, radius scale included)."""
    l1, deep = row_bytes(fmt)
    radii = PAGE * 64 * (1 if fmt["int8_radii"] else 2)
    return radii + PAGE * (l1 + deep) + PAGE * HEAD_DIM + PAGE * 4 * 2 + (2 if fmt["int8_radii"] else 0)


class PagePool:
    def __init__(self, heads: int, capacity: int, fmt: dict, device, keys: bool = True):
        self.heads, self.capacity, self.fmt, self.device = heads, capacity, dict(fmt), torch.device(device)
        l1, deep = row_bytes(self.fmt)
        self.l1_row, self.deep_row = l1, deep
        dev = self.device
        if keys:
            rdt = torch.int8 if fmt["int8_radii"] else torch.float16
            self.radii = torch.zeros((heads, capacity, PAGE, 64), dtype=rdt, device=dev)
            self.radii_scales = (torch.zeros((heads, capacity), dtype=torch.float16, device=dev)
                                 if fmt["int8_radii"] else None)
            self.angle_codes_l1 = torch.zeros((heads, capacity, PAGE, l1), dtype=torch.uint8, device=dev)
            self.angle_codes_deep = torch.zeros((heads, capacity, PAGE, deep), dtype=torch.uint8, device=dev)
        else:
            self.radii = self.radii_scales = self.angle_codes_l1 = self.angle_codes_deep = None
        self.v_codes = torch.zeros((heads, capacity, PAGE, HEAD_DIM), dtype=torch.int8, device=dev)
        self.v_scales = torch.zeros((heads, capacity, PAGE, 4), dtype=torch.float16, device=dev)
        self._struct = None

    @classmethod
    def from_tensors(cls, radii, angle_codes_l1, angle_codes_deep, radii_scales, v_codes, v_scales, fmt: dict):
        """Wrap caller tensors shaped ``[heads, S, 64, .]`` (contiguous) without copying."""
        self = cls.__new__(cls)
        ref = v_codes if v_codes is not None else radii
        self.heads, self.capacity = int(ref.shape[0]), int(ref.shape[1])
        self.fmt, self.device = dict(fmt), ref.device
        self.l1_row, self.deep_row = row_bytes(self.fmt)
        self.radii, self.angle_codes_l1, self.angle_codes_deep = radii, angle_codes_l1, angle_codes_deep
        self.radii_scales, self.v_codes, self.v_scales = radii_scales, v_codes, v_scales
        self._struct = None
        return self

    def struct(self) -> _lib.PagePool:
        if self._struct is None:
            ptr = lambda t: (t.data_ptr() if (t is not None and t.numel() > 0) else None)
            f = _lib.Format(self.fmt["l1_bits"], self.fmt["deep_bits"], self.fmt["split_dim"], self.fmt["int8_radii"])
            self._struct = _lib.PagePool(ptr(self.radii), ptr(self.radii_scales), ptr(self.angle_codes_l1),
                                         ptr(self.angle_codes_deep), ptr(self.v_codes), ptr(self.v_scales),
                                         self.heads, self.capacity, f)
        return self._struct

    def grown(self, new_capacity: int, n_valid: int) -> "PagePool":
        """A larger pool holding a device copy of the first ``n_valid`` pages of every head."""
        new = PagePool(self.heads, new_capacity, self.fmt, self.device, keys=self.radii is not None)
        for name in ("radii", "angle_codes_l1", "angle_codes_deep", "v_codes", "v_scales"):
            src = getattr(self, name)
            if src is not None and n_valid:
                getattr(new, name)[:, :n_valid].copy_(src[:, :n_valid])
        if self.radii_scales is not None and n_valid:
            new.radii_scales[:, :n_valid].copy_(self.radii_scales[:, :n_valid])
        return new

    def nbytes_valid(self, n_pages: int) -> int:
        return self.heads * n_pages * page_bytes(self.fmt)
