"""Parity at the benchmark configurations' full sizes (B200): the fused kernels against a float64
softmax over the cache decoded by tp_decode_pages (bit-exact with the reference decoder; the
CPU oracle's formula, metal.py:293-332, evaluated on the device because NumPy would take minutes
at these sizes).

* 128K tokens with a ragged dense tail (config 4 on one GPU), several queries.
* Decode steps at 128K that complete a page (the flush inside the split combine) and keep going.
* The adapter key format at 4K with many queries (its P.V is computed exactly).
"""

import numpy as np
import pytest
import torch

from _util import ATOL

pytestmark = pytest.mark.gpu

DEV = "cuda:0"
ADAPTER = dict(use_int8_radii=True, k_angle_bits_deep=8, split_dim=0)


@pytest.fixture(scope="module", autouse=True)
def _built():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    from turbopolar_b200 import build
    build.build()


def _kv(seed, heads, t):
    gen = torch.Generator(device=DEV)
    gen.manual_seed(seed)
    chan = torch.from_numpy(np.random.default_rng(1).uniform(0.5, 4.0, size=128).astype(np.float32)).to(DEV)
    k = (torch.randn((1, heads, t, 128), generator=gen, device=DEV) * chan).half()
    v = torch.randn((1, heads, t, 128), generator=gen, device=DEV).half()
    return k, v, gen


def _fp64(q, kd, vd, scale):
    """float64 attention of q [n, H_q, 128] over dense kd, vd [H_kv, T, 128], one KV head at a time."""
    n, hq = q.shape[0], q.shape[1]
    g = hq // kd.shape[0]
    out = torch.empty((n, hq, 128), dtype=torch.float64, device=q.device)
    for h in range(kd.shape[0]):
        kk, vv = kd[h].double(), vd[h].double()
        s = torch.einsum("ngd,td->ngt", q[:, h * g:(h + 1) * g].double(), kk) * scale
        out[:, h * g:(h + 1) * g] = torch.einsum("ngt,td->ngd", torch.softmax(s, dim=-1), vv)
    return out


def test_128k_ragged_tail_vs_float64():
    from turbopolar_b200 import TurboPolarConfig, TurboPolarKVCacheRuntime
    cfg = TurboPolarConfig(num_q_heads=32, num_kv_heads=8)
    t = 131072 + 37
    k, v, gen = _kv(131, 8, t)
    rt = TurboPolarKVCacheRuntime(cfg, check_finite=False)
    rt.append(k, v)
    assert rt.n_pages == 2048 and rt.tail_len == 37
    kd, vd = rt.decompress(padded_tail=False)
    del k, v
    qs = torch.randn((4, 1, 32, 128), generator=gen, device=DEV).half()
    got = torch.stack([rt.attention(qs[i]) for i in range(4)])[:, 0]
    want = _fp64(qs[:, 0], kd[0], vd[0], cfg.attention_scale)
    err = float((got.double() - want).abs().max())
    assert err < ATOL, err


def test_decode_steps_at_128k_across_a_page_flush():
    from turbopolar_b200 import TurboPolarConfig, TurboPolarKVCacheRuntime
    cfg = TurboPolarConfig(num_q_heads=32, num_kv_heads=8)
    t0, steps = 131072 + 60, 8  # the 4th step completes page 2048
    k, v, gen = _kv(132, 8, t0 + steps)
    rt = TurboPolarKVCacheRuntime(cfg, max_seq_len=t0 + steps + 64, check_finite=False)
    rt.append(k[:, :, :t0].contiguous(), v[:, :, :t0].contiguous())
    qs = torch.randn((steps, 1, 32, 128), generator=gen, device=DEV).half()
    outs = []
    err = 0.0
    for s in range(steps):
        outs.append(rt.decode_step(k[:, :, t0 + s:t0 + s + 1].contiguous(), v[:, :, t0 + s:t0 + s + 1].contiguous(),
                                   qs[s]).clone())
        if s == 0:  # before the flush the last 61 tokens are the dense tail
            kd, vd = rt.decompress(padded_tail=False)
            want = _fp64(qs[0], kd[0], vd[0], cfg.attention_scale)
            err = max(err, float((outs[0].double() - want).abs().max()))
            del kd, vd
    assert rt.n_pages == 2049 and rt.tail_len == 4 and rt.read_device_error() == 0
    kd, vd = rt.decompress(padded_tail=False)  # pages (the flushed one included) + the dense tail
    del k, v
    for s in (3, 4, steps - 1):  # at and after the flush
        n = t0 + s + 1
        want = _fp64(qs[s], kd[0, :, :n], vd[0, :, :n], cfg.attention_scale)
        err = max(err, float((outs[s].double() - want).abs().max()))
    assert err < ATOL, err


def test_adapter_format_many_queries_vs_float64():
    from turbopolar_b200 import TurboPolarConfig, TurboPolarKVCacheRuntime
    cfg = TurboPolarConfig(num_q_heads=32, num_kv_heads=8, **ADAPTER)
    k, v, gen = _kv(133, 8, 4096)
    rt = TurboPolarKVCacheRuntime(cfg, check_finite=False)
    rt.append(k, v)
    kd, vd = rt.decompress(padded_tail=False)
    qs = torch.randn((300, 1, 32, 128), generator=gen, device=DEV).half()
    got = torch.stack([rt.attention(qs[i]) for i in range(300)])[:, 0]
    want = _fp64(qs[:, 0], kd[0], vd[0], cfg.attention_scale)
    err = float((got.double() - want).abs().max())
    assert err < ATOL, err
