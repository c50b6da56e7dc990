"""Generate ``dense_v.npz``: the reference's ``execute_online_attention_dense_v`` on the inputs of
``inputs.DENSE_V_CASES``, run by the reference's own code (compressed keys, dense values).

Run once, in a container that has the reference checkout (it never runs on the GPU box):

    python tests/golden/make_golden_dense_v.py /path/to/Turbopolar

As for ``make_golden.py``, ``mlx_standin/`` stands in for ``mlx.core`` and the reference's
modules are imported unmodified; the Metal dispatch probe fails on the stand-in, so the bridge
takes its CPU fallback (``rfsn_v11/kernels/turbo_polar/metal.py:597-603`` into
``_cpu_online_attention``, ``:267-291``).  Stored per case: the page codes the reference's
runtime encoded and the output at each of ``inputs.DENSE_V_LENGTHS``.
"""

from __future__ import annotations

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
    warnings.simplefilter("ignore", RuntimeWarning)
    import mlx.core as mx
    from rfsn_v11.candidates.turbo_polar_config import TurboPolarConfig
    from rfsn_v11.generation.turbo_polar_cache import TurboPolarKVCacheRuntime
    from rfsn_v11.kernels.turbo_polar.metal import MetalKernelBridge

    arrays: dict[str, np.ndarray] = {}
    for name, (overrides, _seed) in inputs.DENSE_V_CASES.items():
        cfg = TurboPolarConfig(num_q_heads=8, num_kv_heads=2, **overrides)
        k, v, q = inputs.dense_v_inputs(name)
        rt = TurboPolarKVCacheRuntime(cfg)
        rt.append(mx.array(k), mx.array(v))
        blk, _qv, _tk, _tv, _qjl, seq = rt.get_fused_attention_inputs()
        assert seq == k.shape[2]
        for f in ("radii", "angle_codes_l1", "angle_codes_deep", "radii_scales"):
            a = getattr(blk, f)
            if a is not None:
                arrays[f"{name}/{f}"] = np.asarray(a)
        bridge = MetalKernelBridge()
        for length in inputs.DENSE_V_LENGTHS:
            out, trace = bridge.execute_online_attention_dense_v(
                q=mx.array(q), block=blk, v_dense=mx.array(v), qjl_payload=None, q_proj_signs=None,
                config=cfg, actual_seq_len=length)
            assert trace["fallback_used"] and not trace["quant_v_used"]
            arrays[f"{name}/out_L{length}"] = np.asarray(out)
    path = os.path.join(HERE, "dense_v.npz")
    np.savez_compressed(path, **arrays)
    print(f"wrote {len(arrays)} arrays, {os.path.getsize(path)} bytes")


if __name__ == "__main__":
    if len(sys.argv) != 2:
        sys.exit("usage: python tests/golden/make_golden_dense_v.py <reference checkout>")
    main(sys.argv[1])
