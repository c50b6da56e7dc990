"""Codec classes with the reference's names and methods, executed by the CUDA library.

* ``PolarQuantEncoder.encode_block`` -- ``rfsn_v11/quant/polar/encoder.py:24-98``
* ``PolarQuantDecoder.decode_block`` -- ``rfsn_v11/quant/polar/decoder.py:7-67``
* ``GroupedVQuantizer.quantize_block / dequantize_block`` -- ``rfsn_v11/quant/v_quant/encoder.py:16-38``

Payloads are in the reference's layout (the kernels' own page layout is converted on the
way in and out); blocks are 64 tokens (the supported ``block_size``); tensors must live on a
CUDA device.
"""

from __future__ import annotations

import ctypes

import torch

from . import _lib
from .pages import PAGE, BlockStore, PagePool
from .payload import PolarKeyBlock, QuantizedVBlock, block_metadata, format_of_metadata

_VALUE_ONLY_FMT = dict(l1_bits=4, deep_bits=4, split_dim=64, int8_radii=0)


def _dtype_code(t: torch.Tensor) -> int:
    if t.dtype == torch.float16:
        return _lib.TP_F16
    if t.dtype == torch.float32:
        return _lib.TP_F32
    raise ValueError(f"only float16 and float32 inputs are supported, got {t.dtype}")


def _stream(device) -> int:
    return torch.cuda.current_stream(device).cuda_stream


def _require_cuda(*ts):
    for t in ts:
        if not (isinstance(t, torch.Tensor) and t.is_cuda):
            raise ValueError("TurboPolar B200 kernels need CUDA tensors")


def encode_pages(pool: PagePool, k: torch.Tensor, v: torch.Tensor, n_pages: int, dst_page: int,
                 src_token0: int = 0, d_state: torch.Tensor | None = None) -> None:
    """Encode ``n_pages`` 64-token blocks of ``k, v`` ``[heads, T, 128]`` (innermost contiguous)."""
    _require_cuda(k, v)
    if k.stride(-1) != 1 or v.stride(-1) != 1 or k.stride() != v.stride():
        k, v = k.contiguous(), v.contiguous()
    st = pool.struct()
    _lib.check(_lib.lib().tp_encode_pages(
        ctypes.byref(st), k.data_ptr(), v.data_ptr(), _dtype_code(k), k.stride(0), k.stride(1), src_token0,
        n_pages, dst_page, d_state.data_ptr() if d_state is not None else None, _stream(k.device)))


class PolarQuantEncoder:
    def __init__(self, config):
        self.config = config
        self.fmt = config.format_fields()

    def encode_block(self, k_block: torch.Tensor) -> PolarKeyBlock:
        _require_cuda(k_block)
        B, H, L, D = k_block.shape
        if D != self.config.head_dim:
            raise ValueError(f"encode_block head_dim {D} does not match config {self.config.head_dim}")
        if L != PAGE:
            raise NotImplementedError("encode_block encodes 64-token blocks")
        pool = PagePool(B * H, 1, self.fmt, k_block.device)
        flat = k_block.reshape(B * H, L, D)
        encode_pages(pool, flat, flat, 1, 0)
        ref = pool.export(0, 1)
        return PolarKeyBlock(
            radii=ref.radii.view(B, H, L, 64),
            angle_codes_l1=ref.angle_codes_l1.view(B, H, L, ref.l1_row),
            angle_codes_deep=ref.angle_codes_deep.view(B, H, L, ref.deep_row),
            shape=(B, H, L, D), block_size=L, head_dim=D, metadata=block_metadata(self.fmt),
            radii_scales=ref.radii_scales.view(B, H, 1, 1) if ref.radii_scales is not None else None)


def pool_of_block(block: PolarKeyBlock, quant_v: QuantizedVBlock | None = None):
    """A kernel-layout pool ``[B*H, S, ...]`` holding a 4-D or 5-D reference key payload and,
    when given, its values.  Returns ``(pool, B, H, S)``."""
    radii = block.radii
    five = radii.dim() == 5
    if not five:
        radii = radii.unsqueeze(2)
    B, H, S = radii.shape[:3]
    ex = (lambda t: t if five else t.unsqueeze(2))
    fmt = format_of_metadata(block.metadata, radii)
    rs = None
    if block.radii_scales is not None:
        rs = ex(block.radii_scales).reshape(B * H, S).contiguous()
    if quant_v is not None:
        vc = quant_v.codes.reshape(B * H, S, PAGE, -1).contiguous()
        vs = quant_v.scales.reshape(B * H, S, PAGE, -1).contiguous()
    else:
        vc = torch.zeros((B * H, S, PAGE, 128), dtype=torch.int8, device=radii.device)
        vs = torch.zeros((B * H, S, PAGE, 4), dtype=torch.float16, device=radii.device)
    ref = BlockStore.wrap(
        radii.reshape(B * H, S, PAGE, 64).contiguous(),
        ex(block.angle_codes_l1).reshape(B * H, S, PAGE, -1).contiguous(),
        ex(block.angle_codes_deep).reshape(B * H, S, PAGE, -1).contiguous(), rs, vc, vs, fmt)
    return PagePool.from_reference(ref), B, H, S


class PolarQuantDecoder:
    def decode_block(self, block: PolarKeyBlock) -> torch.Tensor:
        _require_cuda(block.radii)
        if block.radii.dtype == torch.int8 and block.radii_scales is None:
            raise ValueError("int8 radii require radii_scales")
        pool, B, H, S = pool_of_block(block)
        k = torch.empty((B * H, S * PAGE, 128), dtype=torch.float16, device=block.radii.device)
        v = torch.empty_like(k)
        _lib.check(_lib.lib().tp_decode_pages(ctypes.byref(pool.struct()), 0, S, k.data_ptr(), v.data_ptr(),
                                              _stream(k.device)))
        return k.view(B, H, S * PAGE, 128)


class GroupedVQuantizer:
    def __init__(self, group_size: int = 32):
        if group_size != 32:
            raise NotImplementedError("TurboPolar value groups are 32 channels")
        self.group_size = group_size

    def quantize_block(self, v_block: torch.Tensor) -> QuantizedVBlock:
        _require_cuda(v_block)
        B, H, S, L, D = v_block.shape
        if L != PAGE or D != 128:
            raise NotImplementedError("quantize_block expects (B, H, S, 64, 128) values")
        pool = PagePool(B * H, S, _VALUE_ONLY_FMT, v_block.device)
        flat = v_block.reshape(B * H, S * L, D)
        encode_pages(pool, flat, flat, S, 0)
        ref = pool.export(0, S, keys=False)
        return QuantizedVBlock(codes=ref.v_codes.view(B, H, S, L, D), scales=ref.v_scales.view(B, H, S, L, 4),
                               group_size=self.group_size)

    def dequantize_block(self, block: QuantizedVBlock) -> torch.Tensor:
        _require_cuda(block.codes)
        B, H, S, L, D = block.codes.shape
        ref = BlockStore.wrap(None, None, None, None, block.codes.reshape(B * H, S, L, D).contiguous(),
                              block.scales.reshape(B * H, S, L, 4).contiguous(), _VALUE_ONLY_FMT)
        pool = PagePool.from_reference(ref)
        out = torch.empty((B * H, S * L, D), dtype=torch.float16, device=block.codes.device)
        _lib.check(_lib.lib().tp_decode_pages(ctypes.byref(pool.struct()), 0, S, None, out.data_ptr(),
                                              _stream(out.device)))
        return out.view(B, H, S, L, D)
