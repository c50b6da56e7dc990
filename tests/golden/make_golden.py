"""Generate the golden fixtures in this folder by running the reference's own code.

Run once, in a container that has the reference checkout (it never runs on the GPU box):

    python tests/golden/make_golden.py /path/to/Turbopolar

MLX cannot be installed here, so ``mlx_standin/`` (a NumPy stand-in for the part of
``mlx.core`` the reference's CPU path touches) is put first on ``sys.path`` and the
reference's modules are imported unmodified from the checkout.  The Metal bridge's dispatch
probe fails on the stand-in, so every bridge call takes the reference's CPU fallback.
Inputs come from ``inputs.py`` (seeded PCG64) and are rebuilt by the tests, so only outputs
are stored: ``golden.npz`` (arrays) and ``golden_meta.json`` (telemetry dicts, traces).
"""

from __future__ import annotations

import json
import os
import sys
import warnings

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, HERE)
import inputs  # noqa: E402


def main(ref_root: str) -> None:
    sys.path.insert(0, os.path.join(HERE, "mlx_standin"))
    sys.path.insert(0, ref_root)
    sys.path.insert(0, os.path.join(ref_root, "benchmarks"))
    warnings.simplefilter("ignore", RuntimeWarning)
    import mlx.core as mx
    from rfsn_v11.candidates.turbo_polar_config import TurboPolarConfig
    from rfsn_v11.generation.turbo_polar_cache import TurboPolarKVCacheRuntime
    from rfsn_v11.kernels.turbo_polar.metal import MetalKernelBridge
    from rfsn_v11.quant.polar.decoder import PolarQuantDecoder
    from rfsn_v11.quant.polar.encoder import PolarQuantEncoder
    from rfsn_v11.quant.v_quant.encoder import GroupedVQuantizer
    from turbopolar_fast_attention import TurboPolarFastCache

    arrays: dict[str, np.ndarray] = {}
    meta: dict = {}

    def put(prefix, **kw):
        for k, v in kw.items():
            if v is not None:
                arrays[f"{prefix}/{k}"] = np.asarray(v)

    # ---------------------------------------------------------------- codec cases
    for name, (overrides, _dtype, _seed) in inputs.CODEC_CASES.items():
        cfg = TurboPolarConfig(num_q_heads=8, num_kv_heads=4, **overrides)
        k, v = inputs.codec_inputs(name)
        blk = PolarQuantEncoder(cfg).encode_block(mx.array(k))
        qv = GroupedVQuantizer(32).quantize_block(mx.array(v).reshape(1, 4, 1, 64, 128))
        unified = blk.__class__(
            radii=mx.expand_dims(blk.radii, 2), angle_codes_l1=mx.expand_dims(blk.angle_codes_l1, 2),
            angle_codes_deep=mx.expand_dims(blk.angle_codes_deep, 2),
            radii_scales=mx.expand_dims(blk.radii_scales, 2) if blk.radii_scales is not None else None,
            shape=(1, 4, 1, 64, 128), block_size=64, head_dim=128, metadata=blk.metadata)
        k_dec = PolarQuantDecoder().decode_block(unified)
        put(f"codec/{name}", radii=blk.radii, angle_codes_l1=blk.angle_codes_l1,
            angle_codes_deep=blk.angle_codes_deep,
            radii_scales=None if blk.radii_scales is None else np.asarray(blk.radii_scales),
            v_codes=qv.codes, v_scales=qv.scales, k_decoded=k_dec)
        if name == "default_f16":
            put(f"codec/{name}", v_dequant=GroupedVQuantizer(32).dequantize_block(qv))
        md = {a: (b.item() if isinstance(b, np.generic) else b) for a, b in blk.metadata.items()}
        meta[f"codec/{name}"] = {"cfg": overrides, "metadata": md}

    # ---------------------------------------------------------------- README case (config 1)
    cfg = TurboPolarConfig(num_q_heads=8, num_kv_heads=4, head_dim=128, block_size=64)
    rt = TurboPolarKVCacheRuntime(cfg)
    ks, vs, q = inputs.c1_inputs()
    for i in range(ks.shape[0]):
        rt.append(mx.array(ks[i]), mx.array(vs[i]))
    blk, qv, tk, tv, _qjl, seq = rt.get_fused_attention_inputs()
    bridge = MetalKernelBridge()
    out, trace = bridge.execute_online_attention_quant_v_dense_tail(
        q=mx.array(q), block=blk, quant_v=qv, tail_k=tk, tail_v=tv, qjl_payload=None,
        q_proj_signs=None, config=cfg, actual_seq_len=seq)
    scores = bridge.execute_fused_qk(mx.array(q), blk, cfg)
    put("c1", radii=blk.radii, angle_codes_l1=blk.angle_codes_l1, angle_codes_deep=blk.angle_codes_deep,
        v_codes=qv.codes, v_scales=qv.scales, tail_k=tk, tail_v=tv, out=out, scores=scores)
    meta["c1"] = {"telemetry": rt.get_io_telemetry(), "trace": trace, "actual_seq_len": seq}

    # ---------------------------------------------------------------- runtime shape matrix
    # tests/test_turbo_polar_cache_runtime.py:42-56 (T x GQA) with split_dim=0; the padded
    # partial block of get_blocks_for_attention is stored for the single-KV-head cases.
    for t in inputs.SHAPE_TS:
        for gqa in (1, 4):
            cfg = TurboPolarConfig(head_dim=128, qjl_proj_dim=64, block_size=64, split_dim=0,
                                   num_q_heads=4, num_kv_heads=4 // gqa, seed=7)
            rt = TurboPolarKVCacheRuntime(cfg)
            k, v = inputs.shape_inputs(t, gqa)
            rt.append(mx.array(k), mx.array(v))
            blk, qv, _dense_v, _qjl, seq = rt.get_blocks_for_attention()
            tag = f"shape/T{t}_g{gqa}"
            if gqa == 4:
                put(tag, radii=blk.radii, angle_codes_l1=blk.angle_codes_l1, angle_codes_deep=blk.angle_codes_deep,
                    v_codes=qv.codes, v_scales=qv.scales, k_decoded=PolarQuantDecoder().decode_block(blk))
            meta[tag] = {"telemetry": rt.get_io_telemetry(), "actual_seq_len": seq,
                         "blocks_shape": list(blk.radii.shape)}

    # ---------------------------------------------------------------- incremental telemetry (growth)
    cfg = TurboPolarConfig(num_q_heads=4, num_kv_heads=2)
    rt = TurboPolarKVCacheRuntime(cfg)
    tele = []
    for k, v in inputs.growth_inputs():
        rt.append(mx.array(k), mx.array(v))
        tele.append(rt.get_io_telemetry())
    meta["growth"] = {"telemetry": tele}

    # ---------------------------------------------------------------- Llama adapter decode sequence
    # tests/benchmarks/test_turbopolar_fast_attention.py: 4q/2kv, one token per decode step.
    qs, ks, vs = inputs.adapter_inputs()
    for name, overrides in inputs.ADAPTER_CASES.items():
        cfg = TurboPolarConfig(head_dim=128, block_size=64, num_q_heads=4, num_kv_heads=2,
                               storage_mode="kv_quant", **overrides)
        cache = TurboPolarFastCache(cfg)
        outs = [np.asarray(cache.decode_attention(mx.array(qs[i]), mx.array(ks[i]), mx.array(vs[i]),
                                                  cfg.attention_scale)) for i in range(qs.shape[0])]
        put(f"adapter/{name}", out=np.stack(outs))
        meta[f"adapter/{name}"] = {"cfg": overrides, "telemetry": cache.runtime.get_io_telemetry()}

    # ---------------------------------------------------------------- prefill decompress-on-read
    cfg = TurboPolarConfig(head_dim=128, block_size=64, num_q_heads=4, num_kv_heads=2,
                           use_int8_radii=True, k_angle_bits_deep=8, split_dim=0)
    cache = TurboPolarFastCache(cfg)
    kp, vp, kp2, vp2 = inputs.prefill_inputs()
    kd, vd = cache.update_and_fetch(mx.array(kp), mx.array(vp))
    kd2, vd2 = cache.update_and_fetch(mx.array(kp2), mx.array(vp2))
    put("prefill", k_out=kd, v_out=vd, k_out2=kd2, v_out2=vd2)

    np.savez_compressed(os.path.join(HERE, "golden.npz"), **arrays)
    with open(os.path.join(HERE, "golden_meta.json"), "w") as f:
        json.dump(meta, f, indent=1, sort_keys=True,
                  default=lambda o: o.item() if isinstance(o, np.generic) else str(o))
    print(f"wrote {len(arrays)} arrays, {os.path.getsize(os.path.join(HERE, 'golden.npz'))} bytes")


if __name__ == "__main__":
    if len(sys.argv) != 2:
        sys.exit("usage: python tests/golden/make_golden.py <reference checkout>")
    main(sys.argv[1])
