"""Compressed keys with dense float16 values (B200): ``execute_online_attention_dense_v``
(``rfsn_v11/kernels/turbo_polar/metal.py:587-649``) through ``tp_decode_attention_dense_v``,
against the float64 oracle of its CPU fallback (``metal.py:267-291``) over the same encoded
keys and the values as given.

Cases: every key-format path of the page pass (the table-driven default format, the adapter
format, the general path with 8-bit level-1 / 2-bit deep codes and with int8 radii), GQA groups
1 to 8, masking of the last tokens, a 5-D value block, batch 2, a value array shorter than the
pages (read as zeros past its end), 32K tokens at the Llama-3 head layout, and the outputs of
the reference's own code (``tests/golden/dense_v.npz``).
"""

import ctypes

import numpy as np
import pytest
import torch

from _util import ATOL, fmt_of, kv_inputs, oracle_cache
from oracle import attention as oatt

pytestmark = pytest.mark.gpu

DEV = "cuda:0"
ADAPTER = dict(use_int8_radii=True, k_angle_bits_deep=8, split_dim=0)


@pytest.fixture(scope="module", autouse=True)
def _built():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    from turbopolar_b200 import build
    build.build()


def T(x):
    return torch.from_numpy(np.ascontiguousarray(x)).to(DEV)


def _cfg(**kw):
    from turbopolar_b200 import TurboPolarConfig
    return TurboPolarConfig(**kw)


def _cache(cfg, k, v):
    from turbopolar_b200 import TurboPolarKVCacheRuntime
    rt = TurboPolarKVCacheRuntime(cfg)
    rt.append(T(k), T(v))
    blk, _, tk, _, _, seq = rt.get_fused_attention_inputs()
    assert tk is None and seq == k.shape[2]
    return rt, blk


CASES = [
    (4, 2, 192, {}),
    (32, 8, 64 * 6, {}),
    (8, 1, 320, ADAPTER),
    (4, 4, 256, dict(k_angle_bits_level1=8, k_angle_bits_deep=2, split_dim=32)),
    (12, 2, 128, dict(use_int8_radii=True)),
]


@pytest.mark.parametrize("hq,hkv,t,fmt", CASES)
def test_dense_v_vs_oracle(hq, hkv, t, fmt):
    from turbopolar_b200 import CudaKernelBridge
    cfg = _cfg(num_q_heads=hq, num_kv_heads=hkv, **fmt)
    k, v = kv_inputs(600 + t + hq, hkv, t, np.float16)
    _, blk = _cache(cfg, k, v)
    pages, _, _ = oracle_cache(k, v, fmt_of(cfg), cfg.use_int8_radii)
    q = np.random.default_rng(601 + t).standard_normal((1, hq, 128)).astype(np.float16)
    for L in (t, t - 37, 65, 1):
        out, tr = CudaKernelBridge().execute_online_attention_dense_v(T(q), blk, T(v), None, None, cfg, L)
        want = oatt.attention_dense_v(q[0].astype(np.float64), pages, fmt_of(cfg), v[0], L, cfg.attention_scale)
        err = float(np.max(np.abs(out.float().cpu().numpy()[0] - want)))
        assert err < ATOL, (L, err)
    assert tr["kernel_name"] == "tp_decode_attention_dense_v" and tr["quant_v_used"] is False
    assert tr["num_queries_per_kv"] == hq // hkv


def test_dense_v_five_d_block_and_batch_two():
    """Values as (B, H_kv, S, 64, 128) with batch 2 (heads flattened batch-major, as the pages)."""
    from turbopolar_b200 import CudaKernelBridge
    cfg = _cfg(num_q_heads=8, num_kv_heads=2)
    k, v = kv_inputs(610, 4, 256, np.float16)  # batch 2 x 2 KV heads, stored as 4 heads
    _, blk = _cache(cfg, k.reshape(2, 2, 256, 128), v.reshape(2, 2, 256, 128))
    pages, _, _ = oracle_cache(k, v, fmt_of(cfg), False)
    q = np.random.default_rng(611).standard_normal((2, 8, 128)).astype(np.float16)
    v5 = T(v.reshape(2, 2, 4, 64, 128))
    out, _ = CudaKernelBridge().execute_online_attention_dense_v(T(q), blk, v5, None, None, cfg, 200)
    got = out.float().cpu().numpy()
    kd, _ = oatt.decode_pages(pages, fmt_of(cfg))
    for b in range(2):
        want = oatt.attention(q[b].astype(np.float64), kd[2 * b:2 * b + 2], v[0, 2 * b:2 * b + 2], 200,
                              cfg.attention_scale)
        assert np.max(np.abs(got[b] - want)) < ATOL, b


def test_dense_v_short_value_array_reads_zeros_past_its_end():
    """A value array of seq_len tokens per head (not a whole number of half pages): the tensor
    copies fill the rest of the last half page with zeros, whose weights are zero."""
    from turbopolar_b200 import _lib
    cfg = _cfg(num_q_heads=8, num_kv_heads=2)
    t, L = 256, 211
    k, v = kv_inputs(620, 2, t, np.float16)
    rt, _ = _cache(cfg, k, v)
    pages, _, _ = oracle_cache(k, v, fmt_of(cfg), False)
    q = np.random.default_rng(621).standard_normal((1, 8, 128)).astype(np.float16)
    vs = T(v[0, :, :L])  # (2, 211, 128), heads 211 * 128 elements apart
    out = torch.full((1, 8, 128), float("nan"), dtype=torch.float16, device=DEV)
    lib = _lib.lib()
    ws = torch.zeros(lib.tp_decode_attention_workspace_size(2, 8), dtype=torch.uint8, device=DEV)
    qd = T(q)
    _lib.check(lib.tp_decode_attention_dense_v(
        ctypes.byref(rt.pool_struct()), _lib.State(t // 64, 0, L, 0), vs.data_ptr(), L * 128, L, qd.data_ptr(),
        _lib.TP_F16, 8, float(cfg.attention_scale), out.data_ptr(), None, ws.data_ptr(), ws.numel(),
        torch.cuda.current_stream().cuda_stream))
    torch.cuda.synchronize()
    assert int(ws[:4].view(torch.int32).item()) == 0
    want = oatt.attention_dense_v(q[0].astype(np.float64), pages, fmt_of(cfg), v[0], L, cfg.attention_scale)
    assert np.max(np.abs(out.float().cpu().numpy()[0] - want)) < ATOL


@pytest.mark.parametrize("fmt", [{}, ADAPTER])
def test_dense_v_32k_vs_float64(fmt):
    """32K tokens, 32 query / 8 KV heads: every CTA's ring wraps many times.  The reference
    formula in float64 on the device over the keys tp_decode_pages decodes."""
    from turbopolar_b200 import CudaKernelBridge, TurboPolarKVCacheRuntime
    cfg = _cfg(num_q_heads=32, num_kv_heads=8, **fmt)
    t = 32768
    gen = torch.Generator(device=DEV)
    gen.manual_seed(630)
    chan = torch.from_numpy(np.random.default_rng(1).uniform(0.5, 4.0, size=128).astype(np.float32)).to(DEV)
    k = (torch.randn((1, 8, t, 128), generator=gen, device=DEV) * chan).half()
    v = torch.randn((1, 8, t, 128), generator=gen, device=DEV).half()
    rt = TurboPolarKVCacheRuntime(cfg, check_finite=False)
    rt.append(k, v)
    blk, _, _, _, _, _ = rt.get_fused_attention_inputs()
    kd, _ = rt.decompress(padded_tail=False)
    q = torch.randn((1, 32, 128), generator=gen, device=DEV).half()
    for L in (t, t - 1000):
        out, _ = CudaKernelBridge().execute_online_attention_dense_v(q, blk, v, None, None, cfg, L)
        want = torch.empty((32, 128), dtype=torch.float64, device=DEV)
        for h in range(8):
            s = (q[0, 4 * h:4 * h + 4].double() @ kd[0, h, :L].double().T) * cfg.attention_scale
            want[4 * h:4 * h + 4] = torch.softmax(s, dim=-1) @ v[0, h, :L].double()
        err = float((out[0].double() - want).abs().max())
        assert err < ATOL, (L, err)


@pytest.mark.parametrize("name", ["default", "adapter_fmt"])
def test_dense_v_vs_reference_fixture(name):
    """Against the reference's own execute_online_attention_dense_v (tests/golden/dense_v.npz, its
    CPU fallback in float16): the kernel is within ATOL of the float64 oracle, and within the
    reference's float16 error (4e-3, the bound the oracle itself needs) of the fixture."""
    import os

    import inputs
    from turbopolar_b200 import CudaKernelBridge
    g = np.load(os.path.join(os.path.dirname(inputs.__file__), "dense_v.npz"))
    overrides, _ = inputs.DENSE_V_CASES[name]
    cfg = _cfg(num_q_heads=8, num_kv_heads=2, **overrides)
    k, v, q = inputs.dense_v_inputs(name)
    _, blk = _cache(cfg, k, v)
    # The pages hold the reference runtime's codes.
    for f in ("radii", "angle_codes_l1", "angle_codes_deep"):
        np.testing.assert_array_equal(getattr(blk, f).cpu().numpy(), g[f"{name}/{f}"])
    pages, _, _ = oracle_cache(k, v, fmt_of(cfg), cfg.use_int8_radii)
    for length in inputs.DENSE_V_LENGTHS:
        out, _ = CudaKernelBridge().execute_online_attention_dense_v(T(q), blk, T(v), None, None, cfg, length)
        got = out.float().cpu().numpy()[0].astype(np.float64)
        want = oatt.attention_dense_v(q[0].astype(np.float64), pages, fmt_of(cfg), v[0], length, cfg.attention_scale)
        assert np.max(np.abs(got - want)) < ATOL, length
        assert np.max(np.abs(got - g[f"{name}/out_L{length}"][0].astype(np.float64))) < 4e-3, length


@pytest.mark.parametrize("B", [40, 64])
def test_dense_v_large_batches(B):
    """40 and 64 sequences x 4 KV heads: 160 segments (two waves of the flat partition) and 256
    (whole segments per CTA), more than the SMs; every sequence against the oracle."""
    from turbopolar_b200 import CudaKernelBridge
    cfg = _cfg(num_q_heads=8, num_kv_heads=4)
    t = 192
    k, v = kv_inputs(640, 4 * B, t, np.float16)
    kb, vb = k.reshape(B, 4, t, 128), v.reshape(B, 4, t, 128)
    _, blk = _cache(cfg, kb, vb)
    pages, _, _ = oracle_cache(k, v, fmt_of(cfg), False)
    kd, _ = oatt.decode_pages(pages, fmt_of(cfg))
    q = np.random.default_rng(641).standard_normal((B, 8, 128)).astype(np.float16)
    out, _ = CudaKernelBridge().execute_online_attention_dense_v(T(q), blk, T(vb), None, None, cfg, 150)
    got = out.float().cpu().numpy()
    for b in range(B):
        want = oatt.attention(q[b].astype(np.float64), kd[4 * b:4 * b + 4], vb[b], 150, cfg.attention_scale)
        assert np.max(np.abs(got[b] - want)) < ATOL, b
