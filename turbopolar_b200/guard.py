"""Canary guard bytes around the runtime's device buffers (a debug aid; off unless enabled).

The kernels write into runtime-owned buffers: the page pool and its radius scales (page encode,
the flush of a decode step), the dense tail (appends) and the state words.  A write past the end
of one of them would silently corrupt whatever the allocator placed next.  With ``enable(n)``,
each of those buffers is allocated as a view into a larger buffer whose bytes outside the view
hold a fixed pattern (``n`` bytes before, at least ``n`` after); ``check()`` reads every guard
back and raises ``AssertionError`` naming the buffer and the first changed byte.  A record keeps
its whole buffer alive until the first check after the runtime has dropped the buffer's view, so
buffers replaced during a test (a pool that grew) are checked too.  The GPU tests run with guards
on and check after each test.  Payload views start ``n`` bytes into a 256-byte-aligned
allocation, so with ``n`` a multiple of 256 their alignment is unchanged.
"""

from __future__ import annotations

import math
import weakref
from typing import List, Tuple

import torch

PATTERN = 0xA5
_bytes = 0
# (whole buffer, weak reference to the payload view, payload offset, payload bytes, label)
_live: List[Tuple[torch.Tensor, "weakref.ref[torch.Tensor]", int, int, str]] = []


def enable(nbytes: int = 4096) -> None:
    global _bytes
    if nbytes <= 0 or nbytes % 256:
        raise ValueError("guard size must be a positive multiple of 256 bytes")
    _bytes = int(nbytes)


def disable() -> None:
    global _bytes
    _bytes = 0
    _live.clear()


def enabled() -> bool:
    return _bytes > 0


def zeros(shape, dtype: torch.dtype, device, label: str) -> torch.Tensor:
    """A zero-filled tensor of ``shape``; with guards enabled, a view inside a guarded buffer."""
    if not _bytes:
        return torch.zeros(shape, dtype=dtype, device=device)
    size = math.prod(shape) * torch.empty((), dtype=dtype).element_size()
    total = 2 * _bytes + (size + 255) // 256 * 256
    base = torch.full((total,), PATTERN, dtype=torch.uint8, device=device)
    base[_bytes:_bytes + size].zero_()
    view = base[_bytes:_bytes + size].view(dtype).view(shape)
    _live.append((base, weakref.ref(view), _bytes, size, label))
    return view


def _check_one(base: torch.Tensor, off: int, size: int, label: str) -> None:
    bad = torch.cat([base[:off], base[off + size:]]) != PATTERN
    if bool(bad.any()):
        i = int(torch.nonzero(bad)[0])
        where = f"{off - i} bytes before" if i < off else f"{i - off + 1} bytes past the end"
        raise AssertionError(f"guard bytes of {label} changed: first at {where} ({size}-byte buffer)")


def check_tensor(t: torch.Tensor) -> None:
    """Check the guards of the buffer whose payload view is ``t`` (one about to be dropped)."""
    for base, view, off, size, label in _live:
        if view() is t:
            _check_one(base, off, size, label)


def check() -> int:
    """Check every recorded buffer, then forget those whose view the runtime has dropped;
    returns how many were checked."""
    for base, _view, off, size, label in _live:
        _check_one(base, off, size, label)
    n = len(_live)
    _live[:] = [rec for rec in _live if rec[1]() is not None]
    return n
