"""The NumPy oracle against fixtures produced by the reference's own code (CPU only)."""

import numpy as np
import pytest

import inputs
from oracle import attention, polar, runtime, vquant


def _fmt(overrides):
    return dict(l1_bits=overrides.get("k_angle_bits_level1", 4), deep_bits=overrides.get("k_angle_bits_deep", 4),
                split_dim=overrides.get("split_dim", 64))


def _fallback_fp16(q, kd, v, length, scale):
    """``_cpu_online_attention`` (``metal.py:267-291``, entered from ``metal.py:597-603``) as the
    reference evaluates it on float16 arrays (the fixtures' MLX stand-in: each float16 product
    rounded once, float16 sums accumulated in float32, softmax in float32 rounded back, the
    -1e9 mask a float16 -inf).  q (H_q,128), kd, v (H_kv,T,128) float16."""
    f32 = np.float32
    g = q.shape[0] // kd.shape[0]
    kk = np.repeat(kd, g, axis=0)
    prod = (q[:, None, :].astype(f32) * kk.astype(f32)).astype(np.float16)
    s = prod.astype(f32).sum(-1).astype(np.float16)
    s = (s.astype(f32) * f32(np.float16(scale))).astype(np.float16)
    s = np.where(np.arange(s.shape[-1])[None, :] < length, s, np.float16(-np.inf))
    a = s.astype(f32)
    e = np.exp((a - a.max(-1, keepdims=True)).astype(np.float64)).astype(f32)
    w = (e / e.sum(-1, keepdims=True)).astype(np.float16)
    vv = np.repeat(v, g, axis=0)
    return (w[:, :, None].astype(f32) * vv.astype(f32)).astype(np.float16).astype(f32).sum(1).astype(np.float16)


def _cache_fp16(pages, fmt, tail_k, tail_v):
    """Keys and values the reference's fallback attends over: decoded pages then the dense tail,
    float16 ``(H_kv, T, 128)`` (``metal.py:293-312``)."""
    ks, vs = [], []
    if pages is not None and np.asarray(pages["radii"]).shape[1] > 0:
        k, v = attention.decode_pages(pages, fmt)
        ks.append(k)
        vs.append(v)
    if tail_k is not None and tail_k.shape[1] > 0:
        ks.append(tail_k)
        vs.append(tail_v)
    return np.concatenate(ks, 1).astype(np.float16), np.concatenate(vs, 1).astype(np.float16)


@pytest.mark.parametrize("name", list(inputs.CODEC_CASES))
def test_codec_bit_exact(name, golden):
    overrides, _, _ = inputs.CODEC_CASES[name]
    fmt = _fmt(overrides)
    k, v = inputs.codec_inputs(name)
    enc = polar.encode_block(k, int8_radii=overrides.get("use_int8_radii", False), **fmt)
    g = lambda f: golden[f"codec/{name}/{f}"]
    np.testing.assert_array_equal(enc["radii"], g("radii"))
    assert enc["radii"].dtype == g("radii").dtype
    np.testing.assert_array_equal(enc["angle_codes_l1"], g("angle_codes_l1"))
    np.testing.assert_array_equal(enc["angle_codes_deep"], g("angle_codes_deep"))
    if overrides.get("use_int8_radii"):
        np.testing.assert_array_equal(enc["radii_scales"], g("radii_scales"))
    codes, scales = vquant.quantize(v)
    np.testing.assert_array_equal(codes, g("v_codes").reshape(codes.shape))
    np.testing.assert_array_equal(scales, g("v_scales").reshape(scales.shape))
    # Decoder: same float16 keys, bit for bit.
    dec = polar.decode_block(enc["radii"], enc["angle_codes_l1"], enc["angle_codes_deep"], enc["radii_scales"], **fmt)
    np.testing.assert_array_equal(dec.view(np.uint16), g("k_decoded").reshape(dec.shape).view(np.uint16))
    if name == "default_f16":
        np.testing.assert_array_equal(vquant.dequantize(codes, scales), g("v_dequant").reshape(codes.shape))


def test_packed_lengths_contract():
    # tests/benchmarks/test_turbo_polar_offline.py:26-34
    k, _ = inputs.codec_inputs("default_f16")
    enc = polar.encode_block(k)
    assert enc["radii"].shape == (1, 4, 64, 64)
    assert enc["angle_codes_l1"].shape == (1, 4, 64, (32 + 1) // 2)
    assert enc["angle_codes_deep"].shape == (1, 4, 64, polar.packed_len(32, 4))
    enc2 = polar.encode_block(k, l1_bits=8, deep_bits=2, split_dim=32)
    assert enc2["angle_codes_l1"].shape == (1, 4, 64, 16)
    assert enc2["angle_codes_deep"].shape == (1, 4, 64, 12)


def test_c1_runtime_and_fallback_attention(golden, golden_meta):
    ks, vs, q = inputs.c1_inputs()
    model = runtime.CacheModel(4)
    for i in range(ks.shape[0]):
        model.append(ks[i], vs[i])
    assert model.telemetry() == pytest.approx(golden_meta["c1"]["telemetry"])
    pages = model.pages()
    for f in ("radii", "angle_codes_l1", "angle_codes_deep", "v_codes", "v_scales"):
        np.testing.assert_array_equal(pages[f], golden[f"c1/{f}"][0])
    np.testing.assert_array_equal(model.partial_k, golden["c1/tail_k"])
    fmt = model.fmt
    out = attention.attention_dense_tail(q[0], pages, fmt, model.partial_k[0], model.partial_v[0], 100, 1 / np.sqrt(128))
    ref = golden["c1/out"][0].astype(np.float64)
    # The oracle's formula with the reference's float16 roundings gives the reference's output
    # bit for bit; the oracle itself (float64) is within the reference's float16 error of it.
    kk, vv = _cache_fp16(pages, fmt, model.partial_k[0], model.partial_v[0])
    emu = _fallback_fp16(q[0], kk, vv, 100, 1 / np.sqrt(128))
    np.testing.assert_array_equal(emu.view(np.uint16), golden["c1/out"][0].view(np.uint16))
    assert np.max(np.abs(out - ref)) < 2e-3
    k_dec, _ = attention.decode_pages(pages, fmt)
    sc = attention.fused_scores(q[0], k_dec, 1 / np.sqrt(128))
    assert np.max(np.abs(sc - golden["c1/scores"][0].astype(np.float64))) < 1e-2


@pytest.mark.parametrize("t", inputs.SHAPE_TS)
@pytest.mark.parametrize("gqa", (1, 4))
def test_shape_matrix_telemetry_and_partial_encode(t, gqa, golden, golden_meta):
    tag = f"shape/T{t}_g{gqa}"
    k, v = inputs.shape_inputs(t, gqa)
    model = runtime.CacheModel(4 // gqa, split_dim=0)
    model.append(k, v)
    assert model.telemetry() == pytest.approx(golden_meta[tag]["telemetry"])
    assert model.telemetry()["partial_tokens"] == t % 64
    assert model.telemetry()["total_blocks"] == t // 64
    if gqa == 4:
        blocks = list(model.blocks)
        part = model.padded_partial()
        if part is not None:
            blocks.append(part)
        for f in ("radii", "angle_codes_l1", "angle_codes_deep", "v_codes"):
            got = np.stack([b[f][0] for b in blocks], axis=1)
            np.testing.assert_array_equal(got, golden[f"{tag}/{f}"][0])


def test_growth_telemetry(golden_meta):
    model = runtime.CacheModel(2)
    for (k, v), want in zip(inputs.growth_inputs(), golden_meta["growth"]["telemetry"]):
        model.append(k, v)
        assert model.telemetry() == pytest.approx(want)


def test_telemetry_known_answer_c1(golden_meta):
    # Known answer: 100 tokens, 4 KV heads, default format (296 B/token/head for pages).
    t = golden_meta["c1"]["telemetry"]
    assert t["dense_kv_bytes"] == 1 * 4 * 100 * 128 * 2 * 2 == 204800
    assert t["actual_cache_bytes"] == 64 * 4 * 296 + 36 * 4 * 128 * 2 * 2 == 149504
    assert t["total_blocks"] == 1 and t["partial_tokens"] == 36


def test_codec_known_answers():
    # Hand-derived from encoder.py:46-55 with float16 constants pi=3.140625, 2pi=6.28125.
    k = np.zeros((1, 1, 1, 128), np.float16)
    k[..., 0:2] = (1, 0)    # theta=0 -> norm=0.5 -> 7.5 -> round-half-even 8
    k[..., 2:4] = (-1, 0)   # theta=pi(fp16) -> shifted=6.28125 -> norm=1 -> 15
    k[..., 4:6] = (0, 1)    # theta=pi/2 -> 1.5703125; +pi=4.7109375; /2pi=0.75 -> 11.25 -> 11
    k[..., 6:8] = (0, -1)   # theta=-pi/2 -> 1.5703125 -> norm 0.25 -> 3.75 -> 4
    enc = polar.encode_block(k)
    codes = polar.unpack_4bit(enc["angle_codes_l1"], 32)[0, 0, 0]
    assert list(codes[:4]) == [8, 15, 11, 4]
    assert list(enc["radii"][0, 0, 0, :4]) == [1, 1, 1, 1]
    # Zero pair: atan2(0, 0) = 0 -> code 8 with radius 0.
    assert codes[4] == 8 and enc["radii"][0, 0, 0, 4] == 0
    # V: group max 127 -> scale exactly 1, codes equal the inputs.
    v = np.zeros((1, 128), np.float16)
    v[0, :32] = np.arange(-15, 17)
    v[0, 31] = 127
    c, s = vquant.quantize(v)
    assert s[0, 0] == 1 and list(c[0, :31]) == list(range(-15, 16)) and c[0, 31] == 127
    assert s[0, 1] == np.float16(1e-4) and not c[0, 32:].any()


def test_adapter_sequence_oracle(golden):
    """Oracle attention over the cache contents after every decode step agrees with the
    reference adapter's outputs (dense-only, compressed+tail and block-boundary branches of
    turbopolar_fast_attention.py:145-188, which all evaluate the same formula)."""
    qs, ks, vs = inputs.adapter_inputs()
    for name, overrides in inputs.ADAPTER_CASES.items():
        fmt = _fmt(overrides)
        model = runtime.CacheModel(2, int8_radii=True, **fmt)
        want = golden[f"adapter/{name}/out"]
        for i in range(qs.shape[0]):
            model.append(ks[i], vs[i])
            pages = model.pages()
            tk = model.partial_k[0] if model.partial_k is not None else None
            tv = model.partial_v[0] if model.partial_v is not None else None
            out = attention.attention_dense_tail(qs[i][0, :, 0, :], pages, fmt, tk, tv, i + 1, 1 / np.sqrt(128))
            # Bit for bit with the reference's float16 evaluation of the same formula at every
            # step; the float64 oracle within the reference's float16 error (measured 2.03e-3).
            kk, vv = _cache_fp16(pages, fmt, tk, tv)
            emu = _fallback_fp16(qs[i][0, :, 0, :], kk, vv, i + 1, 1 / np.sqrt(128))
            np.testing.assert_array_equal(emu.view(np.uint16), want[i][0].view(np.uint16), err_msg=f"{name} {i}")
            assert np.max(np.abs(out - want[i][0].astype(np.float64))) < 3e-3, (name, i)


def _oracle_prefill(k, v):
    """Decompress-on-read of a cache holding ``k, v`` ``(1, H, T, 128)``: full blocks plus the
    tail zero-padded to a block, each encoded and decoded (``turbo_polar_cache.py:200-319``,
    ``turbopolar_fast_attention.py:56-86``), cut to T tokens."""
    fmt = dict(l1_bits=4, deep_bits=8, split_dim=0)
    T = k.shape[2]
    n = -(-T // 64)
    pad = lambda x: np.concatenate([x, np.zeros(x.shape[:2] + (n * 64 - T, 128), x.dtype)], axis=2)
    kb = pad(k).reshape(1, k.shape[1], n, 64, 128)
    vb = pad(v).reshape(1, v.shape[1], n, 64, 128)
    enc = polar.encode_block(kb, int8_radii=True, **fmt)
    kd = polar.decode_block(enc["radii"], enc["angle_codes_l1"], enc["angle_codes_deep"], enc["radii_scales"], **fmt)
    codes, scales = vquant.quantize(vb)
    vd = vquant.dequantize(codes, scales)
    return kd.reshape(k.shape[:2] + (n * 64, 128))[:, :, :T], vd.reshape(k.shape[:2] + (n * 64, 128))[:, :, :T]


def test_prefill_decompress_on_read(golden):
    """The reference adapter's update_and_fetch on two prefill chunks (100 then 30 tokens)."""
    kp, vp, kp2, vp2 = inputs.prefill_inputs()
    k1, v1 = _oracle_prefill(kp, vp)
    k2, v2 = _oracle_prefill(np.concatenate([kp, kp2], axis=2), np.concatenate([vp, vp2], axis=2))
    for got, key in ((k1, "k_out"), (v1, "v_out"), (k2, "k_out2"), (v2, "v_out2")):
        np.testing.assert_array_equal(got.view(np.uint16), golden[f"prefill/{key}"].view(np.uint16))


@pytest.mark.parametrize("name", list(inputs.DENSE_V_CASES))
def test_dense_v_attention_vs_reference(name):
    """The oracle's attention_dense_v against the reference's execute_online_attention_dense_v
    fallback (dense_v.npz, made by make_golden_dense_v.py): the keys the reference's runtime
    encoded, bit for bit, and the output at every masked length."""
    import os
    g = np.load(os.path.join(os.path.dirname(inputs.__file__), "dense_v.npz"))
    overrides, _ = inputs.DENSE_V_CASES[name]
    fmt = _fmt(overrides)
    k, v, q = inputs.dense_v_inputs(name)
    kb = k[0].reshape(2, 3, 64, 128)
    enc = polar.encode_block(kb, int8_radii=overrides.get("use_int8_radii", False), **fmt)
    for f in ("radii", "angle_codes_l1", "angle_codes_deep"):
        np.testing.assert_array_equal(enc[f], g[f"{name}/{f}"][0])
    rs = None
    if overrides.get("use_int8_radii"):
        rs = enc["radii_scales"][..., 0, 0]
        np.testing.assert_array_equal(rs.reshape(-1), g[f"{name}/radii_scales"].reshape(-1))
    pages = dict(radii=enc["radii"], angle_codes_l1=enc["angle_codes_l1"], angle_codes_deep=enc["angle_codes_deep"],
                 radii_scales=rs, v_codes=np.zeros((2, 3, 64, 128), np.int8), v_scales=np.zeros((2, 3, 64, 4), np.float16))
    kd, _ = attention.decode_pages(pages, fmt)
    scale = 1 / np.sqrt(128)
    for length in inputs.DENSE_V_LENGTHS:
        ref = g[f"{name}/out_L{length}"][0]
        # The oracle's formula evaluated with the reference's float16 roundings: the same output.
        emu = _fallback_fp16(q[0], kd.astype(np.float16), v[0], length, scale)
        np.testing.assert_array_equal(emu.view(np.uint16), ref.view(np.uint16))
        # The oracle itself (float64) lies within the reference's own float16 error of it
        # (measured 2.2e-3 to 3.5e-3; most of it is the float16 rounding of the raw scores q.k,
        # tens in magnitude with these channel-scaled keys).
        out = attention.attention_dense_v(q[0].astype(np.float64), pages, fmt, v[0], length, scale)
        assert np.max(np.abs(out - ref.astype(np.float64))) < 4e-3, length
