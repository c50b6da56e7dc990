"""CUDA path against the oracle and the reference-generated fixtures (B200 only)."""

import numpy as np
import pytest
import torch

import inputs
from _util import ATOL, fmt_of, kv_inputs, oracle_attention, oracle_cache
from oracle import polar, vquant

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


def N(x):
    return x.detach().cpu().numpy()


def _cfg(**kw):
    from turbopolar_b200 import TurboPolarConfig
    return TurboPolarConfig(**kw)


# ---------------------------------------------------------------- codec: bit-exact
@pytest.mark.parametrize("name", list(inputs.CODEC_CASES))
def test_encode_bit_exact_vs_golden(name, golden):
    from turbopolar_b200 import GroupedVQuantizer, PolarQuantDecoder, PolarQuantEncoder
    overrides, _, _ = inputs.CODEC_CASES[name]
    cfg = _cfg(num_q_heads=8, num_kv_heads=4, **overrides)
    k, v = inputs.codec_inputs(name)
    blk = PolarQuantEncoder(cfg).encode_block(T(k))
    g = lambda f: golden[f"codec/{name}/{f}"]
    radii = N(blk.radii)
    assert radii.dtype == g("radii").dtype
    np.testing.assert_array_equal(radii.view(np.uint8), g("radii").view(np.uint8))
    # Angle codes: count bin disagreements (must be <= 1e-5 of codes; expected 0).
    fmt = fmt_of(cfg)
    n_l1, n_deep = fmt["split_dim"] // 2, 64 - fmt["split_dim"] // 2
    got = np.concatenate([polar._unpack(N(blk.angle_codes_l1), n_l1, fmt["l1_bits"]),
                          polar._unpack(N(blk.angle_codes_deep), n_deep, fmt["deep_bits"])], -1)
    want = np.concatenate([polar._unpack(g("angle_codes_l1"), n_l1, fmt["l1_bits"]),
                           polar._unpack(g("angle_codes_deep"), n_deep, fmt["deep_bits"])], -1)
    assert np.count_nonzero(got != want) <= 1e-5 * got.size
    np.testing.assert_array_equal(N(blk.angle_codes_l1), g("angle_codes_l1"))
    np.testing.assert_array_equal(N(blk.angle_codes_deep), g("angle_codes_deep"))
    if cfg.use_int8_radii:
        np.testing.assert_array_equal(N(blk.radii_scales).view(np.uint16), g("radii_scales").view(np.uint16))
    qv = GroupedVQuantizer(32).quantize_block(T(v).reshape(1, 4, 1, 64, 128))
    np.testing.assert_array_equal(N(qv.codes), g("v_codes"))
    np.testing.assert_array_equal(N(qv.scales).view(np.uint16), g("v_scales").view(np.uint16))
    dec = PolarQuantDecoder().decode_block(blk)
    np.testing.assert_array_equal(N(dec).view(np.uint16), g("k_decoded").reshape(N(dec).shape).view(np.uint16))
    if name == "default_f16":
        deq = GroupedVQuantizer(32).dequantize_block(qv)
        np.testing.assert_array_equal(N(deq).view(np.uint16), g("v_dequant").view(np.uint16))


@pytest.mark.parametrize("dtype", [np.float16, np.float32])
@pytest.mark.parametrize("fmt", [dict(), dict(use_int8_radii=True, k_angle_bits_deep=8, split_dim=0),
                                 dict(k_angle_bits_level1=8, k_angle_bits_deep=2, split_dim=46)])
def test_bulk_encode_bit_exact_vs_oracle(dtype, fmt):
    """Many pages at once (prefill path), random data; every code bit-exact."""
    from turbopolar_b200 import TurboPolarKVCacheRuntime
    cfg = _cfg(num_q_heads=8, num_kv_heads=2, **fmt)
    k, v = kv_inputs(3, 2, 64 * 40 + 17, dtype)
    rt = TurboPolarKVCacheRuntime(cfg)
    rt.append(T(k), T(v))
    blk, qv, tk, tv, _, seq = rt.get_fused_attention_inputs()
    pages, otk, otv = oracle_cache(k, v, fmt_of(cfg), cfg.use_int8_radii)
    assert seq == k.shape[2] and blk.radii.shape[2] == 40
    np.testing.assert_array_equal(N(blk.radii[0]).view(np.uint8), pages["radii"].view(np.uint8))
    np.testing.assert_array_equal(N(blk.angle_codes_l1[0]), pages["angle_codes_l1"])
    np.testing.assert_array_equal(N(blk.angle_codes_deep[0]), pages["angle_codes_deep"])
    np.testing.assert_array_equal(N(qv.codes[0]), pages["v_codes"])
    np.testing.assert_array_equal(N(qv.scales[0]).view(np.uint16), pages["v_scales"].view(np.uint16))
    if cfg.use_int8_radii:
        np.testing.assert_array_equal(N(blk.radii_scales[0, :, :, 0, 0]).view(np.uint16),
                                      pages["radii_scales"].view(np.uint16))
    np.testing.assert_array_equal(N(tk[0]), otk)


# ---------------------------------------------------------------- runtime: config 1 (README case)
def test_c1_runtime_contents_telemetry_attention(golden, golden_meta):
    from turbopolar_b200 import CudaKernelBridge, TurboPolarKVCacheRuntime
    cfg = _cfg(num_q_heads=8, num_kv_heads=4, head_dim=128, block_size=64)
    ks, vs, q = inputs.c1_inputs()
    rt = TurboPolarKVCacheRuntime(cfg)
    for i in range(ks.shape[0]):
        rt.append(T(ks[i]), T(vs[i]))
    assert rt.get_io_telemetry() == pytest.approx(golden_meta["c1"]["telemetry"])
    blk, qv, tk, tv, _, seq = rt.get_fused_attention_inputs()
    assert seq == 100
    for f, t_ in (("radii", blk.radii), ("angle_codes_l1", blk.angle_codes_l1),
                  ("angle_codes_deep", blk.angle_codes_deep), ("v_codes", qv.codes), ("v_scales", qv.scales)):
        np.testing.assert_array_equal(N(t_), golden[f"c1/{f}"])
    np.testing.assert_array_equal(N(tk), golden["c1/tail_k"])
    out = N(rt.attention(T(q))).astype(np.float64)
    want = oracle_attention(q[0], np.concatenate(list(ks), 2), np.concatenate(list(vs), 2), fmt_of(cfg), False,
                            cfg.attention_scale)
    assert np.max(np.abs(out[0] - want)) < ATOL
    assert np.max(np.abs(out[0] - golden["c1/out"][0].astype(np.float64))) < ATOL
    # Bridge form of the same call, and the scores kernel.
    bout, trace = CudaKernelBridge().execute_online_attention_quant_v_dense_tail(
        T(q), blk, qv, tk, tv, None, None, cfg, seq)
    assert trace["tail_length"] == 36 and trace["num_queries_per_kv"] == 2 and trace["cuda_used"]
    np.testing.assert_array_equal(N(bout), N(rt.attention(T(q))))
    sc = N(CudaKernelBridge().execute_fused_qk(T(q), blk, cfg)).astype(np.float64)
    assert np.max(np.abs(sc - golden["c1/scores"].astype(np.float64))) < 1e-2


# ---------------------------------------------------------------- attention sweep vs oracle
SWEEP = [
    # (H_q, H_kv, T, dtype, format overrides)
    (8, 4, 1, np.float16, {}),
    (8, 4, 37, np.float16, {}),
    (8, 4, 63, np.float16, {}),
    (8, 4, 64, np.float16, {}),
    (8, 4, 65, np.float16, {}),
    (8, 4, 129, np.float32, {}),
    (4, 4, 200, np.float16, {}),
    (32, 8, 4096, np.float16, {}),
    (32, 8, 4097 + 30, np.float16, {}),
    (16, 2, 1000, np.float16, {}),
    (64, 4, 700, np.float16, {}),
    (32, 8, 1500, np.float16, dict(use_int8_radii=True, k_angle_bits_deep=8, split_dim=0)),
    (8, 2, 777, np.float32, dict(k_angle_bits_level1=8, k_angle_bits_deep=2, split_dim=32)),
    (8, 8, 300, np.float16, dict(use_int8_radii=True)),
    (12, 4, 333, np.float16, dict(k_angle_bits_deep=8, split_dim=128)),
]


@pytest.mark.parametrize("hq,hkv,t,dtype,fmt", SWEEP)
def test_attention_vs_oracle(hq, hkv, t, dtype, fmt):
    from turbopolar_b200 import TurboPolarKVCacheRuntime
    cfg = _cfg(num_q_heads=hq, num_kv_heads=hkv, **fmt)
    k, v = kv_inputs(t * 7 + hq, hkv, t, dtype)
    q = np.random.default_rng(t).standard_normal((1, hq, 128)).astype(np.float16)
    rt = TurboPolarKVCacheRuntime(cfg)
    rt.append(T(k), T(v))
    out = N(rt.attention(T(q)))[0].astype(np.float64)
    want = oracle_attention(q[0], k, v, fmt_of(cfg), cfg.use_int8_radii, cfg.attention_scale)
    err = np.max(np.abs(out - want))
    assert err < ATOL, err


def test_incremental_decode_matches_bulk_and_oracle():
    """Token-by-token appends (tail fills, page flushes) give the same pages and outputs as one
    bulk append; attention after every step stays within tolerance of the oracle."""
    from turbopolar_b200 import TurboPolarKVCacheRuntime
    cfg = _cfg(num_q_heads=8, num_kv_heads=2)
    k, v = kv_inputs(11, 2, 150, np.float16)
    qs = np.random.default_rng(5).standard_normal((150, 1, 8, 128)).astype(np.float16)
    inc = TurboPolarKVCacheRuntime(cfg)
    for i in range(150):
        inc.append(T(k[:, :, i:i + 1]), T(v[:, :, i:i + 1]))
        if i % 13 == 0 or i in (62, 63, 64, 127, 128, 149):
            out = N(inc.attention(T(qs[i])))[0].astype(np.float64)
            want = oracle_attention(qs[i][0], k[:, :, :i + 1], v[:, :, :i + 1], fmt_of(cfg), False, cfg.attention_scale)
            assert np.max(np.abs(out - want)) < ATOL, i
    bulk = TurboPolarKVCacheRuntime(cfg)
    bulk.append(T(k), T(v))
    a, b = inc.get_fused_attention_inputs(), bulk.get_fused_attention_inputs()
    for x, y in ((a[0].radii, b[0].radii), (a[0].angle_codes_l1, b[0].angle_codes_l1),
                 (a[1].codes, b[1].codes), (a[2], b[2])):
        assert torch.equal(x, y)
    assert inc.get_io_telemetry() == bulk.get_io_telemetry()
    assert inc.read_device_error() == 0
    assert int(inc.d_state[0]) == 2 and int(inc.d_state[1]) == 22 and int(inc.d_state[2]) == 150


def test_device_state_path_matches_host_state():
    from turbopolar_b200 import TurboPolarKVCacheRuntime
    cfg = _cfg(num_q_heads=32, num_kv_heads=8)
    k, v = kv_inputs(2, 8, 2000, np.float16)
    rt = TurboPolarKVCacheRuntime(cfg, max_seq_len=4096)
    rt.append(T(k), T(v))
    q = T(np.random.default_rng(0).standard_normal((1, 32, 128)).astype(np.float16))
    assert torch.equal(rt.attention(q), rt.attention(q, use_device_state=True))


def test_cuda_graph_decode_steps_match_eager():
    """Capture a decode step (append 1 token + attention, one tp_decode_step) once; replay it
    for many steps (counters advance on the device) and compare with an eager runtime fed the
    same tokens through append + attention."""
    from turbopolar_b200 import TurboPolarKVCacheRuntime
    cfg = _cfg(num_q_heads=8, num_kv_heads=2)
    k, v = kv_inputs(21, 2, 60 + 80, np.float16)
    q = np.random.default_rng(9).standard_normal((1, 8, 128)).astype(np.float16)
    g_rt = TurboPolarKVCacheRuntime(cfg, max_seq_len=1024, check_finite=False)
    e_rt = TurboPolarKVCacheRuntime(cfg, max_seq_len=1024)
    g_rt.append(T(k[:, :, :60]), T(v[:, :, :60]))
    e_rt.append(T(k[:, :, :60]), T(v[:, :, :60]))
    kin = torch.zeros((1, 2, 1, 128), dtype=torch.float16, device=DEV)
    vin = torch.zeros_like(kin)
    qin = T(q)
    out = torch.zeros((1, 8, 128), dtype=torch.float16, device=DEV)
    from turbopolar_b200 import graph
    step = graph.DecodeStep(g_rt, kin, vin, qin, out)
    for i in range(60, 140):
        kin.copy_(T(k[:, :, i:i + 1]))
        vin.copy_(T(v[:, :, i:i + 1]))
        step.replay()
        e_rt.append(T(k[:, :, i:i + 1]), T(v[:, :, i:i + 1]))
        want = e_rt.attention(qin)
        if e_rt.tail_len == 0:
            # The step that completes a page attends it from the codes it just encoded
            # (float32 products) instead of through the page pass (float16 products).
            assert (out.float() - want.float()).abs().max().item() <= ATOL, i
        else:
            assert torch.equal(out, want), i
    assert g_rt.read_device_error() == 0
    assert g_rt.actual_seq_len == 140 and g_rt.n_pages == 2 and g_rt.tail_len == 12


# ---------------------------------------------------------------- reference fixtures
@pytest.mark.parametrize("t", inputs.SHAPE_TS)
@pytest.mark.parametrize("gqa", (1, 4))
def test_shape_matrix_vs_golden(t, gqa, golden, golden_meta):
    from turbopolar_b200 import TurboPolarKVCacheRuntime
    cfg = _cfg(head_dim=128, qjl_proj_dim=64, block_size=64, split_dim=0, num_q_heads=4, num_kv_heads=4 // gqa, seed=7)
    tag = f"shape/T{t}_g{gqa}"
    k, v = inputs.shape_inputs(t, gqa)
    rt = TurboPolarKVCacheRuntime(cfg)
    rt.append(T(k), T(v))
    assert rt.get_io_telemetry() == pytest.approx(golden_meta[tag]["telemetry"])
    blk, qv, _, _, seq = rt.get_blocks_for_attention()
    assert list(blk.radii.shape) == golden_meta[tag]["blocks_shape"] and seq == t
    if gqa == 4:
        for f, x in (("radii", blk.radii), ("angle_codes_l1", blk.angle_codes_l1),
                     ("angle_codes_deep", blk.angle_codes_deep), ("v_codes", qv.codes)):
            np.testing.assert_array_equal(N(x), golden[f"{tag}/{f}"])
        from turbopolar_b200 import PolarQuantDecoder
        np.testing.assert_array_equal(N(PolarQuantDecoder().decode_block(blk)).view(np.uint16),
                                      golden[f"{tag}/k_decoded"].view(np.uint16))


def test_growth_telemetry_vs_golden(golden_meta):
    from turbopolar_b200 import TurboPolarKVCacheRuntime
    rt = TurboPolarKVCacheRuntime(_cfg(num_q_heads=4, num_kv_heads=2))
    for (k, v), want in zip(inputs.growth_inputs(), golden_meta["growth"]["telemetry"]):
        rt.append(T(k), T(v))
        assert rt.get_io_telemetry() == pytest.approx(want)


@pytest.mark.parametrize("name", list(inputs.ADAPTER_CASES))
def test_decode_sequence_vs_reference_adapter(name, golden):
    """Per-step outputs of the reference adapter's decode_attention (dense-only, compressed +
    tail and block-boundary branches) against runtime append + attention."""
    from turbopolar_b200 import TurboPolarKVCacheRuntime
    cfg = _cfg(head_dim=128, block_size=64, num_q_heads=4, num_kv_heads=2, **inputs.ADAPTER_CASES[name])
    qs, ks, vs = inputs.adapter_inputs()
    want = golden[f"adapter/{name}/out"]
    rt = TurboPolarKVCacheRuntime(cfg)
    k_all = np.concatenate(list(ks), 2)[0:1]
    v_all = np.concatenate(list(vs), 2)[0:1]
    err_ref = err_oracle = 0.0
    for i in range(qs.shape[0]):
        rt.append(T(ks[i]), T(vs[i]))
        out = N(rt.attention(T(qs[i])))[0].astype(np.float64)
        # Against the float64 oracle on the same tokens: the 2e-3 bar.
        exact = oracle_attention(qs[i][0, :, 0], k_all[:, :, :i + 1], v_all[:, :, :i + 1], fmt_of(cfg),
                                 cfg.use_int8_radii, cfg.attention_scale)
        err_oracle = max(err_oracle, float(np.max(np.abs(out - exact))))
        # Against the reference adapter's own outputs, which it reduces in float16.
        err_ref = max(err_ref, float(np.max(np.abs(out - want[i][0].astype(np.float64)))))
    assert err_oracle < ATOL, err_oracle
    assert err_ref < 3e-3, (err_ref, err_oracle)


@pytest.mark.parametrize("fmt", [{}, dict(use_int8_radii=True, k_angle_bits_deep=8, split_dim=0)])
def test_scores_32q_8kv_vs_oracle(fmt):
    """tp_fused_scores (execute_fused_qk) at the Llama-3 head layout against the float64
    oracle scores over the decoded keys; the reference's kernel test bound is 1e-2
    (tests/benchmarks/test_turbo_polar_kernel_qk.py:57)."""
    from turbopolar_b200 import CudaKernelBridge, TurboPolarKVCacheRuntime
    from oracle import attention as oatt
    cfg = _cfg(num_q_heads=32, num_kv_heads=8, **fmt)
    k, v = kv_inputs(404, 8, 64 * 20, np.float16)
    q = np.random.default_rng(405).standard_normal((1, 32, 128)).astype(np.float16)
    rt = TurboPolarKVCacheRuntime(cfg)
    rt.append(T(k), T(v))
    blk, _, _, _, _, _ = rt.get_fused_attention_inputs()
    got = N(CudaKernelBridge().execute_fused_qk(T(q), blk, cfg))[0].astype(np.float64)
    pages, _, _ = oracle_cache(k, v, fmt_of(cfg), cfg.use_int8_radii)
    kd, _ = oatt.decode_pages(pages, fmt_of(cfg))
    want = oatt.fused_scores(q[0].astype(np.float64), kd, cfg.attention_scale)
    assert got.shape == want.shape
    # Scores are float16 (as the reference's): allow a float16 rounding of |score| <= 32 plus the
    # float32 accumulation.
    assert np.max(np.abs(got - want)) < 1e-2, np.max(np.abs(got - want))


# ---------------------------------------------------------------- masking and edge cases
def test_bridge_masking_and_no_tail():
    from turbopolar_b200 import CudaKernelBridge, TurboPolarKVCacheRuntime
    from oracle import attention as oatt
    cfg = _cfg(num_q_heads=4, num_kv_heads=2)
    k, v = kv_inputs(4, 2, 192, np.float16)
    rt = TurboPolarKVCacheRuntime(cfg)
    rt.append(T(k), T(v))
    blk, qv, tk, tv, _, seq = rt.get_fused_attention_inputs()
    assert tk is None and seq == 192
    q = np.random.default_rng(1).standard_normal((1, 4, 128)).astype(np.float16)
    pages, _, _ = oracle_cache(k, v, fmt_of(cfg), False)
    for L in (192, 150, 100, 64, 1):
        out, tr = CudaKernelBridge().execute_online_attention_quant_v(T(q), blk, qv, None, None, cfg, L)
        kk, vv = oatt.decode_pages(pages, fmt_of(cfg))
        want = oatt.attention(q[0].astype(np.float64), kk, vv, L, cfg.attention_scale)
        assert np.max(np.abs(N(out)[0] - want)) < ATOL, L
        assert tr["num_queries_per_kv"] == 2


def test_errors():
    from turbopolar_b200 import CudaKernelBridge, TurboPolarKVCacheRuntime
    cfg = _cfg(num_q_heads=8, num_kv_heads=4)
    rt = TurboPolarKVCacheRuntime(cfg)
    k = torch.zeros((1, 4, 1, 128), dtype=torch.float16, device=DEV)
    rt.append(k, k)
    with pytest.raises(ValueError, match="batch size changed"):
        rt.append(torch.zeros((2, 4, 1, 128), dtype=torch.float16, device=DEV), torch.zeros((2, 4, 1, 128), dtype=torch.float16, device=DEV))
    with pytest.raises(ValueError, match="dtype changed"):
        rt.append(k.float(), k.float())
    with pytest.raises(ValueError, match="KV head count changed"):
        rt.append(k[:, :2], k[:, :2])
    bad = k.clone()
    bad[0, 0, 0, 0] = float("inf")
    with pytest.raises(ValueError, match="finite"):
        rt.append(bad, k)
    with pytest.raises(ValueError, match="single query"):
        rt.attention(torch.zeros((1, 8, 2, 128), dtype=torch.float16, device=DEV))
    with pytest.raises(ValueError, match="GQA ratio"):
        rt.attention(torch.zeros((1, 6, 128), dtype=torch.float16, device=DEV))
    with pytest.raises(NotImplementedError, match="QJL"):
        CudaKernelBridge().execute_online_attention_dense_v(None, None, None, None, None, cfg, 1, use_qjl=True)
    rt.reset()
    rt.append(torch.zeros((2, 4, 1, 128), dtype=torch.float16, device=DEV), torch.zeros((2, 4, 1, 128), dtype=torch.float16, device=DEV))
    assert rt._batch_size == 2


def test_batch_two_flattens_heads():
    from turbopolar_b200 import TurboPolarKVCacheRuntime
    cfg = _cfg(num_q_heads=8, num_kv_heads=2)
    k, v = kv_inputs(8, 4, 150, np.float16)   # batch 2 x 2 heads, stored as 4 "heads"
    kb = k.reshape(2, 2, 150, 128)
    vb = v.reshape(2, 2, 150, 128)
    q = np.random.default_rng(2).standard_normal((2, 8, 128)).astype(np.float16)
    rt = TurboPolarKVCacheRuntime(cfg)
    rt.append(T(kb), T(vb))
    out = N(rt.attention(T(q))).astype(np.float64)
    for b in range(2):
        want = oracle_attention(q[b], kb[b:b + 1], vb[b:b + 1], fmt_of(cfg), False, cfg.attention_scale)
        assert np.max(np.abs(out[b] - want)) < ATOL


ADAPTER_FMT = dict(use_int8_radii=True, k_angle_bits_deep=8, split_dim=0)


@pytest.mark.parametrize("batch,t,fmt", [(18, 85, {}), (24, 85, {}), (25, 85, {}), (40, 581, {}), (40, 191, {}),
                                         (128, 300, {}), (64, 581, {}), (40, 191, ADAPTER_FMT),
                                         (64, 191, ADAPTER_FMT),
                                         (30, 200, dict(k_angle_bits_level1=8, k_angle_bits_deep=2, split_dim=32)),
                                         (20, 200, dict(k_angle_bits_level1=8, k_angle_bits_deep=2, split_dim=32))])
def test_large_batches_vs_oracle(batch, t, fmt):
    """Batches of sequences x 8 KV heads: 144 segments (the flat partition), then 160 to 1024
    segments, more than the 148 SMs (whole waves of the flat partition for 160, 192, 200 and 320;
    whole segments per CTA for 240, 512 and 1024).  Contexts of one page
    (warps without a unit in a segment), nine pages, and a decode step that completes a page
    (191 + 1 tokens); the default, adapter and general key formats.  Every sequence matches the
    oracle, for attention and for the step."""
    from turbopolar_b200 import TurboPolarKVCacheRuntime
    cfg = _cfg(num_q_heads=32, num_kv_heads=8, **fmt)
    k, v = kv_inputs(190 + batch + t, 8 * batch, t + 1, np.float16)
    kb, vb = k.reshape(batch, 8, t + 1, 128), v.reshape(batch, 8, t + 1, 128)
    q = np.random.default_rng(193 + batch + t).standard_normal((batch, 32, 128)).astype(np.float16)
    rt = TurboPolarKVCacheRuntime(cfg, max_seq_len=t + 1)
    rt.append(T(kb[:, :, :t]), T(vb[:, :, :t]))
    out = N(rt.attention(T(q))).astype(np.float64)
    step = N(rt.decode_step(T(kb[:, :, t:]), T(vb[:, :, t:]), T(q))).astype(np.float64)
    assert rt.read_device_error() == 0
    for b in range(batch):
        want = oracle_attention(q[b], kb[b:b + 1, :, :t], vb[b:b + 1, :, :t], fmt_of(cfg), cfg.use_int8_radii,
                                cfg.attention_scale)
        assert np.max(np.abs(out[b] - want)) < ATOL, b
        want = oracle_attention(q[b], kb[b:b + 1], vb[b:b + 1], fmt_of(cfg), cfg.use_int8_radii, cfg.attention_scale)
        assert np.max(np.abs(step[b] - want)) < ATOL, b


@pytest.mark.parametrize("batch,t", [(24, 100), (64, 150)])
def test_large_batches_float32_tail_vs_oracle(batch, t):
    """Float32 keys and values (so a float32 dense tail) over more segments than SMs: whole
    waves of the flat partition (192 segments) and whole segments (512), with the records of
    every segment merged for all its query heads in one CTA.  Every sequence matches the oracle."""
    from turbopolar_b200 import TurboPolarKVCacheRuntime
    cfg = _cfg(num_q_heads=32, num_kv_heads=8)
    k, v = kv_inputs(250 + batch + t, 8 * batch, t, np.float32)
    kb, vb = k.reshape(batch, 8, t, 128), v.reshape(batch, 8, t, 128)
    q = np.random.default_rng(251 + batch + t).standard_normal((batch, 32, 128)).astype(np.float16)
    rt = TurboPolarKVCacheRuntime(cfg, max_seq_len=t)
    rt.append(T(kb), T(vb))
    out = N(rt.attention(T(q))).astype(np.float64)
    assert rt.read_device_error() == 0
    for b in range(batch):
        want = oracle_attention(q[b], kb[b:b + 1], vb[b:b + 1], fmt_of(cfg), cfg.use_int8_radii, cfg.attention_scale)
        assert np.max(np.abs(out[b] - want)) < ATOL, b


def test_full_size_c3_layer_vs_oracle():
    """One layer of config 3 at full size (32768 tokens, 32q/8kv) against the oracle."""
    from turbopolar_b200 import TurboPolarKVCacheRuntime
    cfg = _cfg(num_q_heads=32, num_kv_heads=8)
    k, v = kv_inputs(33, 8, 32768, np.float16)
    q = np.random.default_rng(34).standard_normal((1, 32, 128)).astype(np.float16)
    rt = TurboPolarKVCacheRuntime(cfg, max_seq_len=32768 + 128)
    rt.append(T(k), T(v))
    out = N(rt.attention(T(q)))[0].astype(np.float64)
    want = oracle_attention(q[0], k, v, fmt_of(cfg), False, cfg.attention_scale)
    assert np.max(np.abs(out - want)) < ATOL


@pytest.mark.parametrize("tokens", [40, 64, 100, 200])
def test_decompress_multi_head_vs_oracle(tokens):
    """Decompress-on-read (stored pages, then the tail zero-padded, encoded and decoded) for
    several heads, bit-exact against the oracle codec."""
    from turbopolar_b200 import TurboPolarKVCacheRuntime
    from oracle import polar, vquant
    cfg = _cfg(num_q_heads=8, num_kv_heads=4)
    k, v = kv_inputs(30 + tokens, 4, tokens, np.float16)
    rt = TurboPolarKVCacheRuntime(cfg)
    rt.append(T(k), T(v))
    kd, vd = rt.decompress(padded_tail=True)
    n = -(-tokens // 64)
    pad = lambda x: np.concatenate([x, np.zeros(x.shape[:2] + (n * 64 - tokens, 128), x.dtype)], axis=2)
    kb, vb = pad(k).reshape(1, 4, n, 64, 128), pad(v).reshape(1, 4, n, 64, 128)
    enc = polar.encode_block(kb)
    want_k = polar.decode_block(enc["radii"], enc["angle_codes_l1"], enc["angle_codes_deep"], None)
    codes, scales = vquant.quantize(vb)
    want_v = vquant.dequantize(codes, scales)
    np.testing.assert_array_equal(N(kd).view(np.uint16), want_k.reshape(1, 4, n * 64, 128)[:, :, :tokens].view(np.uint16))
    np.testing.assert_array_equal(N(vd).view(np.uint16), want_v.reshape(1, 4, n * 64, 128)[:, :, :tokens].view(np.uint16))
