"""Time the decode-attention kernel on synthetic layers (also the small case for ncu captures).

    python -m turbopolar_b200.profile_attention --ctx 32768 --hq 32 --hkv 8

Builds enough independent layers that their pages exceed 4x the 126 MB L2 (so every launch
reads cold data), captures one launch per layer in a CUDA graph and replays it; the per-launch
device time comes from CUDA events around the replays on the launching stream.  Prints the
time and the achieved GB/s of algorithmic bytes (compressed pages + dense tail + q + out), for
independent launches (every layer reads the same query) and for a dependent chain (each
layer's query is the previous layer's output).
``--batch B`` times calls over B sequences each (B x H_kv flattened KV heads).  ``--launches N``
instead issues N plain launches over the layers (for ncu: one kernel per
launch, no graph).  ``--dense-v`` times tp_decode_attention_dense_v instead (the keys of the
same pages, float16 values from a separate array; no dense tail: ``--ctx`` a multiple of 64).
"""

from __future__ import annotations

import argparse
import ctypes
import json
import math

import numpy as np
import torch

from . import TurboPolarConfig, TurboPolarKVCacheRuntime, _lib, build
from .pages import page_bytes, row_bytes

FORMATS = {
    "default": {},
    "adapter": dict(use_int8_radii=True, k_angle_bits_deep=8, split_dim=0),
}
L2_BYTES = 126 * 2 ** 20


def make_layers(a, dev):
    cfg = TurboPolarConfig(num_q_heads=a.hq, num_kv_heads=a.hkv, **FORMATS[a.format])
    per_layer = a.batch * ((a.ctx // 64) * a.hkv * page_bytes(cfg.format_fields()) + (a.ctx * a.hkv * 256 if a.dense_v else 0))
    n = a.layers or max(1, math.ceil(4 * L2_BYTES / max(per_layer, 1)))
    gen = torch.Generator(device=dev)
    chan = torch.from_numpy(np.random.default_rng(1).uniform(0.5, 4.0, size=128).astype(np.float32)).to(dev)
    layers, values = [], []
    for i in range(n):
        gen.manual_seed(a.seed + i)
        k = (torch.randn((a.batch, a.hkv, a.ctx, 128), generator=gen, device=dev) * chan).half()
        v = torch.randn((a.batch, a.hkv, a.ctx, 128), generator=gen, device=dev).half()
        rt = TurboPolarKVCacheRuntime(cfg, max_seq_len=a.ctx, check_finite=False)
        rt.append(k, v)
        if a.dense_v:
            values.append(v.reshape(a.batch * a.hkv, a.ctx, 128).contiguous())
        del k, v
        layers.append(rt)
    q = torch.randn((a.batch, a.hq, 128), generator=gen, device=dev).half()
    return cfg, layers, values, q


def dense_v_caller(a, layers, values, dev):
    """attend(i, q, out): tp_decode_attention_dense_v over layer i's pages and values."""
    if a.ctx % 64:
        raise SystemExit("--dense-v needs --ctx a multiple of 64")
    lib = _lib.lib()
    heads, q_heads = a.batch * a.hkv, a.batch * a.hq
    ws = [torch.zeros(lib.tp_decode_attention_workspace_size(heads, q_heads), dtype=torch.uint8, device=dev)
          for _ in layers]
    scale = float(layers[0].config.attention_scale)

    def attend(i, q, out):
        rt = layers[i]
        _lib.check(lib.tp_decode_attention_dense_v(
            ctypes.byref(rt.pool_struct()), _lib.State(rt.n_pages, 0, a.ctx, 0), values[i].data_ptr(), a.ctx * 128,
            a.ctx, q.data_ptr(), _lib.TP_F16, q_heads, scale, out.data_ptr(), None, ws[i].data_ptr(), ws[i].numel(),
            torch.cuda.current_stream(dev).cuda_stream))
    return attend


def main(argv=None):
    ap = argparse.ArgumentParser()
    ap.add_argument("--ctx", type=int, default=32768)
    ap.add_argument("--hq", type=int, default=32)
    ap.add_argument("--hkv", type=int, default=8)
    ap.add_argument("--batch", type=int, default=1, help="sequences per call (KV heads flattened batch-major)")
    ap.add_argument("--layers", type=int, default=0, help="0: enough layers to exceed 4x L2")
    ap.add_argument("--reps", type=int, default=20)
    ap.add_argument("--launches", type=int, default=0, help="plain launches instead of graph replays")
    ap.add_argument("--format", default="default", choices=sorted(FORMATS))
    ap.add_argument("--seed", type=int, default=0)
    ap.add_argument("--dense-v", action="store_true", help="time tp_decode_attention_dense_v")
    a = ap.parse_args(argv)
    build.build()
    dev = torch.device("cuda:0")
    cfg, layers, values, q = make_layers(a, dev)
    outs = [torch.empty((a.batch, a.hq, 128), dtype=torch.float16, device=dev) for _ in layers]
    if a.dense_v:
        attend = dense_v_caller(a, layers, values, dev)
    else:
        def attend(i, q, out):
            layers[i].attention(q, out=out)
    for i, o in enumerate(outs):
        attend(i, q, o)
    torch.cuda.synchronize()
    rt0 = layers[0]
    if a.dense_v:  # keys (radii + angle codes) of every page, float16 values, q, out
        fmt = rt0.fmt
        l1, deep = row_bytes(fmt)
        k_row = (64 if fmt["int8_radii"] else 128) + l1 + deep
        nbytes = a.batch * (rt0.n_pages * 64 * a.hkv * (k_row + 256) + a.hq * 128 * 4)
    else:
        nbytes = a.batch * (rt0.n_pages * a.hkv * page_bytes(rt0.fmt) + rt0.tail_len * a.hkv * 128 * 4 + a.hq * 128 * 4)
    if a.launches:
        for i in range(a.launches):
            attend(i % len(layers), q, outs[i % len(layers)])
        torch.cuda.synchronize()
        print(json.dumps({"plain_launches": a.launches}))
        return

    def per_launch_us(chain: bool) -> float:
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g):
            for i, o in enumerate(outs):
                attend(i, outs[i - 1] if chain and i > 0 else q, o)
        for _ in range(3):
            g.replay()
        torch.cuda.synchronize()
        s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        s.record()
        for _ in range(a.reps):
            g.replay()
        e.record()
        torch.cuda.synchronize()
        del g
        return s.elapsed_time(e) * 1e3 / (a.reps * len(layers))

    # Independent calls (each layer reads the same query), then a dependent chain (each layer's
    # query is the previous layer's output, so no call may start streaming before the previous
    # one has completed).
    us = per_launch_us(False)
    dep = per_launch_us(True)
    print(json.dumps({"ctx": a.ctx, "batch": a.batch, "hq": a.hq, "hkv": a.hkv, "format": a.format, "dense_v": a.dense_v,
                      "layers": len(layers),
                      "us_per_launch": us, "bytes_per_launch": nbytes, "gbs": nbytes / us / 1e3,
                      "us_per_launch_dependent": dep, "gbs_dependent": nbytes / dep / 1e3}))


if __name__ == "__main__":
    main()
