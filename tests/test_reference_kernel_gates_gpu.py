"""The reference's own kernel tests, run on this build's kernels (B200).

``tests/benchmarks/test_turbo_polar_kernel_qk.py`` (``test_phase_6_fused_qk_precision``) and
``tests/benchmarks/test_turbo_polar_online_attention.py`` (``test_phase_8_dense_v_gate``,
``test_phase_9_quant_v_gate``, ``test_long_context_float_accumulator_stability``), and
``tests/benchmarks/test_turbopolar_fast_attention.py`` (the Llama adapter's three decode cases): the same
configurations, shapes, reference formula (scores over the decoded keys, softmax, weighted sum
of the values) and gates (max error and cosine).  The QJL variants are left out (QJL is rejected
by the configuration contract).  Inputs: seeded NumPy float32 normals in place of
``mx.random.normal`` (MLX's streams cannot be reproduced); the reference formula in float64.
"""

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu

DEV = "cuda:0"


@pytest.fixture(scope="module", autouse=True)
def _built():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    from turbopolar_b200 import build
    build.build()


def _cfg(num_heads, seed):
    from turbopolar_b200 import TurboPolarConfig
    return TurboPolarConfig(head_dim=128, qjl_proj_dim=64, block_size=64, split_dim=64, num_q_heads=num_heads,
                            num_kv_heads=num_heads, seed=seed)


def _normal(rng, shape):
    return torch.from_numpy(rng.standard_normal(shape).astype(np.float32)).to(DEV)


def _encode_unified(cfg, k):
    """test_turbo_polar_online_attention.py:27-38: encode every 64-token block and stack them."""
    from turbopolar_b200 import PolarKeyBlock, PolarQuantEncoder
    B, H, T, D = k.shape
    S = T // cfg.block_size
    kb = k.reshape(B, H, S, cfg.block_size, D)
    blocks = [PolarQuantEncoder(cfg).encode_block(kb[:, :, s].contiguous()) for s in range(S)]
    return PolarKeyBlock(radii=torch.stack([b.radii for b in blocks], 2),
                         angle_codes_l1=torch.stack([b.angle_codes_l1 for b in blocks], 2),
                         angle_codes_deep=torch.stack([b.angle_codes_deep for b in blocks], 2),
                         shape=(B, H, T, D), block_size=cfg.block_size, head_dim=D, metadata=blocks[0].metadata)


def _reference_attention(cfg, q, unified, v):
    from turbopolar_b200 import PolarQuantDecoder
    k_recon = PolarQuantDecoder().decode_block(unified).double()
    scores = (q.double()[:, :, None, :] * k_recon).sum(-1) * cfg.attention_scale
    w = torch.softmax(scores, dim=-1)
    return (w[:, :, :, None] * v.double().reshape(k_recon.shape)).sum(-2)


def _gates(ref, got):
    ref, got = ref.double().flatten(), got.double().flatten()
    cosine = float(ref @ got / (ref.norm() * got.norm() + 1e-12))
    return float((ref - got).abs().max()), cosine


def test_phase_6_fused_qk_precision():
    """test_turbo_polar_kernel_qk.py:39-59: scores within 1e-2, cosine >= 0.999."""
    from turbopolar_b200 import CudaKernelBridge, PolarQuantDecoder
    cfg = _cfg(4, 42)
    rng = np.random.default_rng(cfg.seed)
    k = _normal(rng, (1, 4, 128, 128))
    q = _normal(rng, (1, 4, 128))
    unified = _encode_unified(cfg, k)
    k_recon = PolarQuantDecoder().decode_block(unified).double()
    ref = (q.double()[:, :, None, :] * k_recon).sum(-1) * cfg.attention_scale
    got = CudaKernelBridge().execute_fused_qk(q, unified, cfg)
    err, cosine = _gates(ref, got)
    assert err <= 1e-2 and cosine >= 0.999, (err, cosine)


def test_phase_8_dense_v_gate():
    """test_turbo_polar_online_attention.py:40-63: within 1e-3, cosine >= 0.999."""
    from turbopolar_b200 import CudaKernelBridge
    cfg = _cfg(2, 2026)
    rng = np.random.default_rng(cfg.seed)
    q = _normal(rng, (1, 2, 128))
    k = _normal(rng, (1, 2, 128, 128))
    v = _normal(rng, (1, 2, 2, 64, 128))
    unified = _encode_unified(cfg, k)
    got, _ = CudaKernelBridge().execute_online_attention_dense_v(q, unified, v, None, None, cfg, actual_seq_len=128)
    err, cosine = _gates(_reference_attention(cfg, q, unified, v), got)
    assert err <= 1e-3 and cosine >= 0.999, (err, cosine)


def test_phase_9_quant_v_gate():
    """test_turbo_polar_online_attention.py:88-111: int8 values, within 1e-3 of the attention
    over the dequantised values, cosine >= 0.999."""
    from turbopolar_b200 import CudaKernelBridge, GroupedVQuantizer
    cfg = _cfg(2, 2026)
    rng = np.random.default_rng(cfg.seed + 1)
    q = _normal(rng, (1, 2, 128))
    k = _normal(rng, (1, 2, 128, 128))
    v = _normal(rng, (1, 2, 2, 64, 128))
    quant_v = GroupedVQuantizer(group_size=32).quantize_block(v)
    v_deq = GroupedVQuantizer(group_size=32).dequantize_block(quant_v)
    unified = _encode_unified(cfg, k)
    got, _ = CudaKernelBridge().execute_online_attention_quant_v(q, unified, quant_v, None, None, cfg,
                                                                 actual_seq_len=128)
    err, cosine = _gates(_reference_attention(cfg, q, unified, v_deq), got)
    assert err <= 1e-3 and cosine >= 0.999, (err, cosine)


@pytest.mark.parametrize("t", [4096, 8192])
def test_long_context_float_accumulator_stability(t):
    """test_turbo_polar_online_attention.py:113-141: dense values at 4K and 8K, within
    2e-3 * sqrt(T / 64), cosine >= 0.999 (this build also meets the flat 2e-3 bar)."""
    from turbopolar_b200 import CudaKernelBridge
    cfg = _cfg(2, 2026)
    rng = np.random.default_rng(cfg.seed + t)
    q = _normal(rng, (1, 2, 128))
    k = _normal(rng, (1, 2, t, 128))
    v = _normal(rng, (1, 2, t // 64, 64, 128))
    unified = _encode_unified(cfg, k)
    got, _ = CudaKernelBridge().execute_online_attention_dense_v(q, unified, v, None, None, cfg, actual_seq_len=t)
    err, cosine = _gates(_reference_attention(cfg, q, unified, v), got)
    assert err <= 2e-3 * np.sqrt(t / 64.0) and cosine >= 0.999, (err, cosine)
    assert err <= 2e-3, err


# tests/benchmarks/test_turbopolar_fast_attention.py: the Llama adapter's decode_attention.  As
# in the reference, the ground truth is dense attention over the tokens appended before the last
# call (which appends one more), with its cosine gates.
@pytest.mark.parametrize("tokens,seed,gate", [(37, 2026, 0.99), (100, 2027, 0.95), (64, 2028, 0.95)])
def test_fast_attention_decode_vs_dense_history(tokens, seed, gate):
    """:21-61 (all tokens in the dense tail), :63-103 (one compressed block and a tail),
    :105-141 (ending on a block boundary)."""
    from turbopolar_b200 import TurboPolarConfig
    from turbopolar_b200.llama import TurboPolarFastCache
    cfg = TurboPolarConfig(head_dim=128, block_size=64, num_q_heads=4, num_kv_heads=2, storage_mode="kv_quant",
                           use_int8_radii=True)
    cache = TurboPolarFastCache(cfg)
    scale = cfg.attention_scale
    rng = np.random.default_rng(seed)
    ks, vs = [], []
    for _ in range(tokens):
        q = _normal(rng, (1, 4, 1, 128))
        k_new = _normal(rng, (1, 2, 1, 128))
        v_new = _normal(rng, (1, 2, 1, 128))
        ks.append(k_new)
        vs.append(v_new)
        out = cache.decode_attention(q, k_new, v_new, scale)
        assert out.shape == (1, 4, 128) and not bool(torch.isnan(out).any())
    full_k = torch.repeat_interleave(torch.cat(ks, 2), 2, dim=1).double()
    full_v = torch.repeat_interleave(torch.cat(vs, 2), 2, dim=1).double()
    q_last = _normal(rng, (1, 4, 1, 128))
    w = torch.softmax((q_last.double() * full_k).sum(-1) * scale, dim=-1)
    ref = (w[:, :, :, None] * full_v).sum(-2)
    got = cache.decode_attention(q_last, _normal(rng, (1, 2, 1, 128)), _normal(rng, (1, 2, 1, 128)), scale)
    _, cosine = _gates(ref, got)
    assert cosine >= gate, cosine
