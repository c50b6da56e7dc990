"""The reference's own codec and runtime unit tests, run on this build (B200).

* ``tests/benchmarks/test_turbo_polar_offline.py:19-73`` -- packed shapes of the encoder's
  blocks, the unified 5-D payload, and the reconstruction gate (cosine >= 0.90, MSE <= 0.5,
  score cosine >= 0.92).
* ``tests/unit/test_int8_radius_standalone_decode.py:29-50`` -- a 4-D int8-radius block decodes
  like its 5-D unified form, finite, radius scales kept.
* ``tests/test_turbo_polar_cache_runtime.py:90-115`` -- no QJL payload is stored; the GQA
  payload keeps the KV head count.
* ``tests/unit/test_cache_invariants.py:53-61`` -- a head_dim change after the first append is
  rejected.

Seeded NumPy normals replace ``mx.random`` (its streams cannot be reproduced).
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


def _normal(rng, shape):
    return torch.from_numpy(rng.standard_normal(shape).astype(np.float32)).to(DEV)


def _cos(a, b):
    a, b = a.double().flatten(), b.double().flatten()
    return float(a @ b / (a.norm() * b.norm() + 1e-12))


def test_offline_reconstruction_gate():
    from turbopolar_b200 import PolarKeyBlock, PolarQuantDecoder, PolarQuantEncoder, TurboPolarConfig
    cfg = TurboPolarConfig(head_dim=128, qjl_proj_dim=64, block_size=64, split_dim=64, num_q_heads=4,
                           num_kv_heads=4, seed=42)
    B, H, S, L, D = 1, 4, 2, 64, 128
    rng = np.random.default_rng(cfg.seed)
    k = _normal(rng, (B, H, S * L, D))
    kb = k.reshape(B, H, S, L, D)
    blocks = [PolarQuantEncoder(cfg).encode_block(kb[:, :, s].contiguous()) for s in range(S)]
    split_half = cfg.split_dim // 2
    l1_len = (split_half + 1) // 2
    per = 8 // cfg.k_angle_bits_deep
    deep_len = (D // 2 - split_half + per - 1) // per
    assert tuple(blocks[0].radii.shape) == (B, H, L, D // 2)
    assert tuple(blocks[0].angle_codes_l1.shape) == (B, H, L, l1_len)
    assert tuple(blocks[0].angle_codes_deep.shape) == (B, H, L, deep_len)
    unified = PolarKeyBlock(radii=torch.stack([b.radii for b in blocks], 2),
                            angle_codes_l1=torch.stack([b.angle_codes_l1 for b in blocks], 2),
                            angle_codes_deep=torch.stack([b.angle_codes_deep for b in blocks], 2),
                            shape=(B, H, S * L, D), block_size=L, head_dim=D, metadata=blocks[0].metadata)
    assert tuple(unified.radii.shape) == (B, H, S, L, D // 2)
    assert tuple(unified.angle_codes_l1.shape) == (B, H, S, L, l1_len)
    k_recon = PolarQuantDecoder().decode_block(unified)
    assert tuple(k_recon.shape) == (B, H, S * L, D)
    mse = float(((k.double() - k_recon.double()) ** 2).mean())
    assert _cos(k, k_recon) >= 0.90 and mse <= 0.5, (_cos(k, k_recon), mse)
    q = _normal(rng, (B, H, D))
    s_ref = (q.double()[:, :, None, :] * k.double()).sum(-1)
    s_rec = (q.double()[:, :, None, :] * k_recon.double()).sum(-1)
    assert _cos(s_ref, s_rec) >= 0.92


def test_int8_radius_4d_decode_preserves_radii_scales():
    from turbopolar_b200 import PolarKeyBlock, PolarQuantDecoder, PolarQuantEncoder, TurboPolarConfig
    cfg = TurboPolarConfig(head_dim=128, block_size=64, split_dim=0, num_q_heads=4, num_kv_heads=4,
                           use_int8_radii=True, k_angle_bits_deep=8)
    rng = np.random.default_rng(42)
    k = _normal(rng, (1, 4, 64, 128))
    block = PolarQuantEncoder(cfg).encode_block(k)
    assert block.radii.dtype == torch.int8 and block.radii_scales is not None
    d4 = PolarQuantDecoder().decode_block(block)
    assert bool(torch.isfinite(d4).all()) and tuple(d4.shape) == (1, 4, 64, 128)
    unified = PolarKeyBlock(radii=block.radii.unsqueeze(2), angle_codes_l1=block.angle_codes_l1.unsqueeze(2),
                            angle_codes_deep=block.angle_codes_deep.unsqueeze(2),
                            radii_scales=block.radii_scales.unsqueeze(2), shape=(1, 4, 64, 128), block_size=64,
                            head_dim=128, metadata=block.metadata)
    d5 = PolarQuantDecoder().decode_block(unified)
    assert torch.equal(d4.reshape(d5.shape).view(torch.int16), d5.view(torch.int16))


def test_no_qjl_payload_and_gqa_payload_heads():
    from turbopolar_b200 import TurboPolarConfig, TurboPolarKVCacheRuntime
    rng = np.random.default_rng(3)
    rt = TurboPolarKVCacheRuntime(TurboPolarConfig(head_dim=128, block_size=64, num_q_heads=4, num_kv_heads=4,
                                                   use_qjl=False, storage_mode="kv_quant"))
    rt.append(_normal(rng, (1, 4, 64, 128)), _normal(rng, (1, 4, 64, 128)))
    _, _, _, qjl, _ = rt.get_blocks_for_attention()
    assert qjl is None and len(rt.qjl_blocks) == 0
    rt = TurboPolarKVCacheRuntime(TurboPolarConfig(head_dim=128, block_size=64, num_q_heads=8, num_kv_heads=2,
                                                   use_qjl=False, storage_mode="kv_quant"))
    rt.append(_normal(rng, (1, 2, 64, 128)), _normal(rng, (1, 2, 64, 128)))
    block, quant_v, _, _, actual_len = rt.get_blocks_for_attention()
    assert actual_len == 64 and block.radii.shape[1] == 2 and quant_v.codes.shape[1] == 2


def test_head_dim_change_after_first_append_rejected():
    from turbopolar_b200 import TurboPolarConfig, TurboPolarKVCacheRuntime
    rt = TurboPolarKVCacheRuntime(TurboPolarConfig(num_q_heads=4, num_kv_heads=4))
    k = torch.zeros((1, 4, 1, 128), dtype=torch.float16, device=DEV)
    rt.append(k, k)
    k2 = torch.zeros((1, 4, 1, 64), dtype=torch.float16, device=DEV)
    with pytest.raises(ValueError):
        rt.append(k2, k2)
