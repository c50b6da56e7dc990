"""tp_decode_step: append one token and attend, in one call (two kernels).

The reference appends and then attends (TurboPolarFastCache.decode_attention,
benchmarks/turbopolar_fast_attention.py:106-188); the fused step must leave the same cache
(pages bit-exact, tail, counters, telemetry) and give the same outputs as the two calls,
including on the steps where the new token completes a page and that page is encoded inside
the attention launch.
"""

import ctypes

import numpy as np
import pytest
import torch

from _util import ATOL, fmt_of, kv_inputs, oracle_attention

pytestmark = pytest.mark.gpu
DEV = "cuda:0"


@pytest.fixture(scope="module", autouse=True)
def _built():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    from turbopolar_b200 import build
    build.build()


def T(x):
    return torch.from_numpy(np.ascontiguousarray(x)).to(DEV)


CASES = [
    # (q heads, kv heads, format overrides, dtype)
    (8, 4, {}, np.float16),
    (32, 8, {}, np.float16),
    (8, 4, dict(use_int8_radii=True, k_angle_bits_deep=8, split_dim=0), np.float16),
    (8, 4, {}, np.float32),
    (16, 1, dict(k_angle_bits_deep=2, split_dim=32), np.float16),  # 16 query heads a KV head: two chunks
]


@pytest.mark.parametrize("hq,hkv,fmt,dtype", CASES)
def test_decode_step_matches_append_then_attention(hq, hkv, fmt, dtype):
    from turbopolar_b200 import TurboPolarConfig, TurboPolarKVCacheRuntime
    cfg = TurboPolarConfig(num_q_heads=hq, num_kv_heads=hkv, **fmt)
    prefill, steps = 60, 72          # flushes on steps 4 and 68
    k, v = kv_inputs(7, hkv, prefill + steps, dtype)
    q = np.random.default_rng(8).standard_normal((steps, 1, hq, 128)).astype(np.float16)
    fused, split = TurboPolarKVCacheRuntime(cfg), TurboPolarKVCacheRuntime(cfg)
    for rt in (fused, split):
        rt.append(T(k[:, :, :prefill]), T(v[:, :, :prefill]))
    for i in range(steps):
        t = prefill + i
        kn, vn, qi = T(k[:, :, t:t + 1]), T(v[:, :, t:t + 1]), T(q[i])
        a = fused.decode_step(kn, vn, qi)
        split.append(kn, vn)
        b = split.attention(qi)
        torch.cuda.synchronize()
        err = (a.float() - b.float()).abs().max().item()
        if split.tail_len == 0:
            # The completed page: attended from the codes encoded in the step itself (float32
            # products) rather than by the page pass (float16 products); a rounding apart.
            assert err <= ATOL, (i, err)
        else:
            assert err == 0.0, (i, err)
        assert (fused.n_pages, fused.tail_len, fused.actual_seq_len) == (split.n_pages, split.tail_len,
                                                                         split.actual_seq_len)
        if i in (3, 4, 5, steps - 1):
            want = oracle_attention(q[i][0], k[:, :, :t + 1], v[:, :, :t + 1], fmt_of(cfg), cfg.use_int8_radii,
                                    cfg.attention_scale)
            assert np.max(np.abs(a[0].float().cpu().numpy() - want)) < ATOL, i
    # Device counters, stored pages and the tail agree bit for bit.
    assert torch.equal(fused.d_state[:5], split.d_state[:5])
    assert fused.read_device_error() == 0
    n = fused.n_pages
    ea, eb = fused.pool.export(0, n), split.pool.export(0, n)
    for name in ("radii", "angle_codes_l1", "angle_codes_deep", "v_codes", "v_scales"):
        assert torch.equal(getattr(ea, name), getattr(eb, name)), name
    if cfg.use_int8_radii:
        assert torch.equal(ea.radii_scales, eb.radii_scales)
    tl = fused.tail_len
    assert torch.equal(fused.tail_k[:, :tl], split.tail_k[:, :tl])
    assert fused.get_io_telemetry() == split.get_io_telemetry()


def test_decode_step_from_one_token_and_growth():
    """Starting from a single token: the pool is created and grown (capacity 4, doubling) by
    the host before the steps that flush, exactly as appends do."""
    from turbopolar_b200 import TurboPolarConfig, TurboPolarKVCacheRuntime
    cfg = TurboPolarConfig(num_q_heads=4, num_kv_heads=2)
    k, v = kv_inputs(17, 2, 64 * 5 + 3, np.float16)
    q = np.random.default_rng(18).standard_normal((1, 4, 128)).astype(np.float16)
    fused, split = TurboPolarKVCacheRuntime(cfg), TurboPolarKVCacheRuntime(cfg)
    for t in range(k.shape[2]):
        kn, vn = T(k[:, :, t:t + 1]), T(v[:, :, t:t + 1])
        a = fused.decode_step(kn, vn, T(q))
        split.append(kn, vn)
        b = split.attention(T(q))
        assert (a.float() - b.float()).abs().max().item() <= ATOL, t
    assert fused.get_io_telemetry() == split.get_io_telemetry()
    assert fused.reallocation_count == split.reallocation_count > 0


def test_decode_step_graph_replay_matches_eager():
    """A captured tp_decode_step replays at every position (the counters live on the device)."""
    from turbopolar_b200 import TurboPolarConfig, TurboPolarKVCacheRuntime, graph
    cfg = TurboPolarConfig(num_q_heads=8, num_kv_heads=4)
    prefill, steps = 100, 80
    k, v = kv_inputs(27, 4, prefill + steps, np.float16)
    q = np.random.default_rng(28).standard_normal((steps, 1, 8, 128)).astype(np.float16)
    g_rt = TurboPolarKVCacheRuntime(cfg, max_seq_len=prefill + steps)
    e_rt = TurboPolarKVCacheRuntime(cfg)
    for rt in (g_rt, e_rt):
        rt.append(T(k[:, :, :prefill]), T(v[:, :, :prefill]))
    k_in = torch.empty((1, 4, 1, 128), dtype=torch.float16, device=DEV)
    v_in, q_in = torch.empty_like(k_in), torch.empty((1, 8, 128), dtype=torch.float16, device=DEV)
    out = torch.empty((1, 8, 128), dtype=torch.float16, device=DEV)
    step = graph.DecodeStep(g_rt, k_in, v_in, q_in, out)
    for i in range(steps):
        t = prefill + i
        k_in.copy_(T(k[:, :, t:t + 1]))
        v_in.copy_(T(v[:, :, t:t + 1]))
        q_in.copy_(T(q[i]))
        step.replay()
        want = e_rt.decode_step(T(k[:, :, t:t + 1]), T(v[:, :, t:t + 1]), T(q[i]))
        torch.cuda.synchronize()
        assert torch.equal(out, want), i
    assert (g_rt.n_pages, g_rt.tail_len) == (e_rt.n_pages, e_rt.tail_len) == (2, 52)
    assert torch.equal(g_rt.d_state[:5], e_rt.d_state[:5])


@pytest.mark.parametrize("chained", [False, True])
def test_layers_back_to_back_match_one_at_a_time(chained):
    """Decode steps of several caches launched back to back, nothing else between them in the
    stream: a layer's page pass may then stream while the previous layer's kernels finish, which
    must change no result (bit for bit against the same steps run one at a time, flushes
    included).  With ``chained`` every layer's query is the previous layer's output, a
    dependency the library has to see and wait for."""
    from turbopolar_b200 import TurboPolarConfig, TurboPolarKVCacheRuntime
    cfg = TurboPolarConfig(num_q_heads=32, num_kv_heads=8)
    n_layers, prefill, steps = 4, 64 * 40 + 60, 8  # each cache completes a page on step 3
    kv = [kv_inputs(41 + i, 8, prefill + steps, np.float16) for i in range(n_layers)]
    q = T(np.random.default_rng(40).standard_normal((steps, n_layers, 1, 32, 128)).astype(np.float16))
    kin = [[T(kv[i][0][:, :, t:t + 1]) for t in range(prefill, prefill + steps)] for i in range(n_layers)]
    vin = [[T(kv[i][1][:, :, t:t + 1]) for t in range(prefill, prefill + steps)] for i in range(n_layers)]
    runs = []
    for serial in (False, True):
        rts = [TurboPolarKVCacheRuntime(cfg, max_seq_len=prefill + steps) for _ in range(n_layers)]
        for i, rt in enumerate(rts):
            rt.append(T(kv[i][0][:, :, :prefill]), T(kv[i][1][:, :, :prefill]))
        out = torch.empty((steps, n_layers, 1, 32, 128), dtype=torch.float16, device=DEV)
        torch.cuda.synchronize()
        for t in range(steps):
            for i, rt in enumerate(rts):
                qi = out[t, i - 1] if chained and i > 0 else q[t, i]
                rt.decode_step(kin[i][t], vin[i][t], qi, out=out[t, i])
                if serial:
                    torch.cuda.synchronize()
        torch.cuda.synchronize()
        runs.append((out, rts))
    (a, ra), (b, rb) = runs
    assert torch.equal(a, b)
    for x, y in zip(ra, rb):
        assert torch.equal(x.d_state[:5], y.d_state[:5])
        assert x.read_device_error() == 0
    last = prefill + steps
    want = oracle_attention(q[steps - 1, 0, 0].cpu().numpy(), kv[0][0][:, :, :last], kv[0][1][:, :, :last],
                            fmt_of(cfg), False, cfg.attention_scale)
    assert np.max(np.abs(a[steps - 1, 0, 0].float().cpu().numpy() - want)) < ATOL


def test_decode_step_c_abi_errors():
    from turbopolar_b200 import _lib
    lib = _lib.lib()
    f = _lib.Format(4, 4, 64, 0)
    pool = _lib.PagePool(None, None, 2, 0, f)
    tail = _lib.Tail(16, 16, _lib.TP_F16)
    st = lib.tp_decode_step(ctypes.byref(pool), ctypes.byref(tail), None, 16, 16, _lib.TP_F16, 128, 16, 0, 4, 0.1,
                            16, None, 16, 1 << 20, None)
    with pytest.raises(ValueError, match="state words are required"):
        _lib.check(st)
    st = lib.tp_decode_step(ctypes.byref(pool), ctypes.byref(tail), 16, 16, 16, _lib.TP_F32, 128, 16, 0, 4, 0.1,
                            16, None, 16, 1 << 20, None)
    with pytest.raises(ValueError, match="dtype must match"):
        _lib.check(st)
    st = lib.tp_decode_step(ctypes.byref(pool), ctypes.byref(tail), 16, 16, 16, _lib.TP_F16, 100, 16, 0, 4, 0.1,
                            16, None, 16, 1 << 20, None)
    with pytest.raises(ValueError, match="16-byte aligned"):
        _lib.check(st)
