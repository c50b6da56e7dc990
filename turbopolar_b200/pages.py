"""Device page pool: the structure-of-arrays block store, resident in HBM.

Replaces ``PolarKBlockStorage`` / ``QuantVBlockStorage``
(``rfsn_v11/generation/storage.py:17-169``).  One tensor per field with every page of a head
contiguous, so a kernel streams a head's pages as five contiguous byte ranges.  The codes are
the reference's bit for bit; inside a page they are ordered for the decode kernel (swizzled
fp16 radii rows, value codes biased and in mma fragment order, value scales in fragment
order -- ``include/turbopolar.h``).  :meth:`PagePool.export` produces the reference layout
(``storage.py:89-102, :160-169``) and :meth:`PagePool.from_reference` loads it.  ``heads`` is
batch x KV heads.
"""

from __future__ import annotations

import ctypes

import torch

from . import _lib

PAGE = 64
HEAD_DIM = 128
V_PAGE_BYTES = PAGE * HEAD_DIM
V_SCALES_PER_PAGE = PAGE * 4


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


def _stream(device) -> int:
    return torch.cuda.current_stream(device).cuda_stream


class PagePool:
    """``kernel_layout=False`` builds a pool in the reference's block-storage layout instead
    (``v_codes`` int8 ``[heads, cap, 64, 128]``, ``v_scales`` ``[heads, cap, 64, 4]``)."""

    def __init__(self, heads: int, capacity: int, fmt: dict, device, keys: bool = True, kernel_layout: bool = True):
        self.heads, self.capacity, self.fmt, self.device = heads, capacity, dict(fmt), torch.device(device)
        self.kernel_layout = kernel_layout
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
        if kernel_layout:
            self.v_codes = torch.zeros((heads, capacity, V_PAGE_BYTES), dtype=torch.uint8, device=dev)
            self.v_scales = torch.zeros((heads, capacity, V_SCALES_PER_PAGE), dtype=torch.float16, device=dev)
        else:
            self.v_codes = torch.zeros((heads, capacity, PAGE, HEAD_DIM), dtype=torch.int8, device=dev)
            self.v_scales = torch.zeros((heads, capacity, PAGE, 4), dtype=torch.float16, device=dev)
        self._struct = None

    @classmethod
    def wrap_reference(cls, radii, angle_codes_l1, angle_codes_deep, radii_scales, v_codes, v_scales, fmt: dict):
        """Wrap caller tensors in the reference layout, shaped ``[heads, S, 64, .]`` (contiguous)."""
        self = cls.__new__(cls)
        ref = v_codes if v_codes is not None else radii
        self.heads, self.capacity = int(ref.shape[0]), int(ref.shape[1])
        self.fmt, self.device, self.kernel_layout = dict(fmt), ref.device, False
        self.l1_row, self.deep_row = row_bytes(self.fmt)
        self.radii, self.angle_codes_l1, self.angle_codes_deep = radii, angle_codes_l1, angle_codes_deep
        self.radii_scales, self.v_codes, self.v_scales = radii_scales, v_codes, v_scales
        self._struct = None
        return self

    @classmethod
    def from_reference(cls, ref: "PagePool") -> "PagePool":
        """A kernel-layout pool holding the pages of a reference-layout pool."""
        pool = cls(ref.heads, ref.capacity, ref.fmt, ref.device, keys=ref.radii is not None)
        if ref.capacity:
            _lib.check(_lib.lib().tp_import_pages(ctypes.byref(pool.struct()), 0, ref.capacity,
                                                  ctypes.byref(ref.struct()), _stream(ref.device)))
        return pool

    def export(self, first: int, n: int) -> "PagePool":
        """Pages ``[first, first + n)`` in the reference layout (a new pool of capacity ``n``)."""
        ref = PagePool(self.heads, n, self.fmt, self.device, keys=self.radii is not None, kernel_layout=False)
        if n:
            _lib.check(_lib.lib().tp_export_pages(ctypes.byref(self.struct()), first, n, ctypes.byref(ref.struct()),
                                                  _stream(self.device)))
        return ref

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
        new = PagePool(self.heads, new_capacity, self.fmt, self.device, keys=self.radii is not None,
                       kernel_layout=self.kernel_layout)
        for name in ("radii", "angle_codes_l1", "angle_codes_deep", "v_codes", "v_scales", "radii_scales"):
            src = getattr(self, name)
            if src is not None and n_valid:
                getattr(new, name)[:, :n_valid].copy_(src[:, :n_valid])
        return new

    def nbytes_valid(self, n_pages: int) -> int:
        return self.heads * n_pages * page_bytes(self.fmt)
