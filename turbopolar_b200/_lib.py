"""ctypes binding of ``libturbopolar.so`` (declared in ``include/turbopolar.h``).

The library is loaded from this package folder.  There is no CPU fallback: a missing library
or a machine without CUDA raises on first use.
"""

from __future__ import annotations

import ctypes
import os
import threading

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "libturbopolar.so")

TP_OK, TP_ERR_INVALID, TP_ERR_UNSUPPORTED, TP_ERR_CUDA = 0, 1, 2, 3
TP_F16, TP_F32 = 0, 1
PARTIAL_FLOATS = 130
STATE_WORDS = 6

EXPORTED = (
    "tp_row_bytes", "tp_unit_bytes", "tp_encode_pages", "tp_append", "tp_decode_attention_workspace_size",
    "tp_decode_attention", "tp_decode_attention_dense_v", "tp_decode_step", "tp_decode_attention_noalloc", "tp_noalloc_error", "tp_combine_partials", "tp_fused_scores", "tp_decode_pages",
    "tp_export_pages", "tp_import_pages", "tp_last_error", "tp_version",
    "tp_exchange_bytes", "tp_ipc_alloc", "tp_ipc_open", "tp_ipc_close", "tp_ipc_free",
    "tp_decode_attention_sharded", "tp_decode_step_sharded",
)
MAX_RANKS = 8


class Format(ctypes.Structure):
    _fields_ = [("l1_bits", ctypes.c_int32), ("deep_bits", ctypes.c_int32),
                ("split_dim", ctypes.c_int32), ("int8_radii", ctypes.c_int32)]


class PagePool(ctypes.Structure):
    """tp_page_pool: page blocks in the kernels' layout."""
    _fields_ = [("pages", ctypes.c_void_p), ("radii_scales", ctypes.c_void_p),
                ("num_kv_heads", ctypes.c_int32), ("page_capacity", ctypes.c_int32),
                ("fmt", Format)]


class BlockStore(ctypes.Structure):
    """tp_block_store: pages in the reference's block-storage layout."""
    _fields_ = [("radii", ctypes.c_void_p), ("radii_scales", ctypes.c_void_p),
                ("angle_codes_l1", ctypes.c_void_p), ("angle_codes_deep", ctypes.c_void_p),
                ("v_codes", ctypes.c_void_p), ("v_scales", ctypes.c_void_p),
                ("num_kv_heads", ctypes.c_int32), ("page_capacity", ctypes.c_int32),
                ("fmt", Format)]


def fmt_struct(fmt: dict) -> Format:
    return Format(fmt["l1_bits"], fmt["deep_bits"], fmt["split_dim"], fmt["int8_radii"])


def empty_pool(heads: int, fmt: dict) -> PagePool:
    """A pool of capacity 0 (attention over the dense tail only)."""
    return PagePool(None, None, heads, 0, fmt_struct(fmt))


class Tail(ctypes.Structure):
    _fields_ = [("k", ctypes.c_void_p), ("v", ctypes.c_void_p), ("dtype", ctypes.c_int32)]


class State(ctypes.Structure):
    _fields_ = [("n_pages", ctypes.c_int32), ("tail_len", ctypes.c_int32),
                ("seq_len", ctypes.c_int32), ("first_page", ctypes.c_int32)]


class Exchange(ctypes.Structure):
    _fields_ = [("world", ctypes.c_int32), ("rank", ctypes.c_int32), ("buffers", ctypes.c_void_p * 8)]


_lib = None
_lock = threading.Lock()


def _declare(lib):
    P, I32, I64, SZ, F = ctypes.c_void_p, ctypes.c_int32, ctypes.c_int64, ctypes.c_size_t, ctypes.c_float
    sig = {
        "tp_row_bytes": (ctypes.c_int, [ctypes.POINTER(Format), ctypes.POINTER(I32), ctypes.POINTER(I32)]),
        "tp_unit_bytes": (ctypes.c_int, [ctypes.POINTER(Format), ctypes.POINTER(I32)]),
        "tp_encode_pages": (ctypes.c_int, [ctypes.POINTER(PagePool), P, P, I32, I64, I64, I64, I32, I32, P, P]),
        "tp_append": (ctypes.c_int, [ctypes.POINTER(PagePool), ctypes.POINTER(Tail), P, P, P, I32, I64, I64, I32, P]),
        "tp_decode_attention_workspace_size": (SZ, [I32, I32]),
        "tp_decode_attention": (ctypes.c_int, [ctypes.POINTER(PagePool), ctypes.POINTER(Tail), State, P, P, I32, I32,
                                               F, P, P, P, SZ, P]),
        "tp_decode_attention_dense_v": (ctypes.c_int, [ctypes.POINTER(PagePool), State, P, I64, I64, P, I32, I32, F,
                                                       P, P, P, SZ, P]),
        "tp_decode_step": (ctypes.c_int, [ctypes.POINTER(PagePool), ctypes.POINTER(Tail), P, P, P, I32, I64, P, I32,
                                          I32, F, P, P, P, SZ, P]),
        "tp_decode_attention_noalloc": (ctypes.c_int, [ctypes.POINTER(PagePool), ctypes.POINTER(Tail), State, P, P,
                                                       I32, I32, F, P, P, P]),
        "tp_noalloc_error": (ctypes.c_int, [ctypes.POINTER(I32), P]),
        "tp_combine_partials": (ctypes.c_int, [P, I32, I32, P, P]),
        "tp_fused_scores": (ctypes.c_int, [ctypes.POINTER(PagePool), I32, P, I32, I32, F, P, P]),
        "tp_decode_pages": (ctypes.c_int, [ctypes.POINTER(PagePool), I32, I32, P, P, P]),
        "tp_export_pages": (ctypes.c_int, [ctypes.POINTER(PagePool), I32, I32, ctypes.POINTER(BlockStore), P]),
        "tp_import_pages": (ctypes.c_int, [ctypes.POINTER(PagePool), I32, I32, ctypes.POINTER(BlockStore), P]),
        "tp_exchange_bytes": (SZ, [I32, I32]),
        "tp_ipc_alloc": (ctypes.c_int, [SZ, ctypes.POINTER(ctypes.c_void_p), P]),
        "tp_ipc_open": (ctypes.c_int, [P, ctypes.POINTER(ctypes.c_void_p)]),
        "tp_ipc_close": (ctypes.c_int, [P]),
        "tp_ipc_free": (ctypes.c_int, [P]),
        "tp_decode_attention_sharded": (ctypes.c_int, [ctypes.POINTER(PagePool), ctypes.POINTER(Tail), State, P, P,
                                                       I32, I32, F, P, ctypes.POINTER(Exchange), P, SZ, P]),
        "tp_decode_step_sharded": (ctypes.c_int, [ctypes.POINTER(PagePool), ctypes.POINTER(Tail), P, P, P, I32, I64, P,
                                                  I32, I32, F, P, ctypes.POINTER(Exchange), P, SZ, P]),
        "tp_last_error": (ctypes.c_char_p, []),
        "tp_version": (ctypes.c_int, []),
    }
    for name, (res, args) in sig.items():
        fn = getattr(lib, name)
        fn.restype = res
        fn.argtypes = args


def lib():
    """The loaded library (loaded once).  Raises RuntimeError when it has not been built."""
    global _lib
    if _lib is None:
        with _lock:
            if _lib is None:
                if not os.path.exists(LIB_PATH):
                    raise RuntimeError(
                        f"libturbopolar.so not found at {LIB_PATH}; build it with "
                        "`python -m turbopolar_b200.build` (CUDA 12.9 nvcc, sm_100a)")
                handle = ctypes.CDLL(LIB_PATH)
                _declare(handle)
                _lib = handle
    return _lib


def check(status: int) -> None:
    """Map a tp_status to the reference's exception types."""
    if status == TP_OK:
        return
    msg = lib().tp_last_error().decode(errors="replace")
    if status == TP_ERR_INVALID:
        raise ValueError(msg)
    if status == TP_ERR_UNSUPPORTED:
        raise NotImplementedError(msg)
    raise RuntimeError(msg)
