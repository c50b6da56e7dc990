"""Llama adapter (``turbopolar_b200.llama``) against the reference adapter
(``benchmarks/turbopolar_fast_attention.py``) and its tests
(``tests/benchmarks/test_turbopolar_fast_attention.py``).

CPU tests cover the host logic: argument validation and its messages, the adapter format,
the causal-mask predicate, patching.  GPU tests compare ``decode_attention`` and
``update_and_fetch`` with the golden outputs of the reference adapter, and run a small
random-init Hugging Face Llama through prefill and teacher-forced decode with the
TurboPolar cache against a dense fp16 cache, gated by the reference's own logit tolerance
(``rfsn_v11/candidates/turbo_polar_adapter.py:97-105``).
"""

import numpy as np
import pytest
import torch

import inputs
from _util import ATOL, fmt_of, oracle_attention

ADAPTER_FMT = dict(use_int8_radii=True, k_angle_bits_deep=8, split_dim=0)


# ---------------------------------------------------------------- CPU: host logic
def test_make_turbo_caches_format_and_errors():
    from transformers.cache_utils import Cache
    from turbopolar_b200.llama import TurboPolarFastCache, make_turbo_caches
    caches = make_turbo_caches(3, 32, 8, 128)
    assert isinstance(caches, Cache) and len(caches) == 3
    assert all(isinstance(c, TurboPolarFastCache) for c in caches)
    cfg = caches[0].config
    assert (cfg.use_int8_radii, cfg.k_angle_bits_deep, cfg.split_dim, cfg.qjl_proj_dim) == (True, 8, 0, 64)
    assert caches[1].offset == 0 and caches[1].empty() and caches.get_seq_length() == 0
    with pytest.raises(ValueError, match="head_dim 64 or 128, got 96"):
        make_turbo_caches(1, 4, 2, 96)
    with pytest.raises(ValueError, match="head_dim == 128"):
        make_turbo_caches(1, 4, 2, 64)
    with pytest.raises(ValueError, match="QJL is not supported"):
        make_turbo_caches(1, 4, 2, 128, use_qjl=True)


@pytest.mark.parametrize("q_shape,k_shape,exc,msg", [
    ((1, 4, 128), (1, 2, 1, 128), ValueError, "must be 4-D"),
    ((2, 4, 1, 128), (2, 2, 1, 128), NotImplementedError, "batch size 1"),
    ((1, 4, 2, 128), (1, 2, 2, 128), ValueError, "single query/key/value token"),
    ((1, 4, 1, 64), (1, 2, 1, 64), NotImplementedError, "head_dim == 128"),
    ((1, 5, 1, 128), (1, 2, 1, 128), ValueError, "GQA ratio to divide evenly, got 5 and 2"),
])
def test_decode_attention_validation(q_shape, k_shape, exc, msg):
    from turbopolar_b200.llama import make_turbo_caches
    cache = make_turbo_caches(1, 4, 2, 128)[0]
    with pytest.raises(exc, match=msg):
        cache.decode_attention(torch.zeros(q_shape, dtype=torch.float16), torch.zeros(k_shape, dtype=torch.float16),
                               torch.zeros(k_shape, dtype=torch.float16), 0.1)
    assert cache.offset == 0


def test_standard_causal_mask_predicate():
    from turbopolar_b200.llama import _is_standard_causal_mask as ok
    assert ok(None, 1, 10)
    full = torch.ones((1, 1, 1, 10), dtype=torch.bool)
    assert ok(full, 1, 10)
    assert not ok(torch.ones((1, 1, 1, 9), dtype=torch.bool), 1, 10)
    window = full.clone()
    window[..., :3] = False
    assert not ok(window, 1, 10)
    # The unshifted lower triangle of one row admits only key 0: not a full-history mask.
    assert not ok(torch.ones((1, 10), dtype=torch.bool).tril()[None, None], 1, 10)
    # Multi-row causal masks, boolean and additive.
    causal = torch.ones((3, 10), dtype=torch.bool).tril(7)[None, None]
    assert ok(causal, 3, 10)
    add = torch.zeros((1, 1, 3, 10), dtype=torch.float16).masked_fill(~causal, torch.finfo(torch.float16).min)
    assert ok(add, 3, 10)
    assert not ok(add + 0.5, 3, 10)
    assert ok(torch.zeros((1, 1, 1, 10)), 1, 10)


def test_patch_and_unpatch_restore_forward():
    from transformers.models.llama import modeling_llama
    from turbopolar_b200 import llama
    orig = modeling_llama.LlamaAttention.forward
    llama.patch_llama_attention(None)
    llama.patch_llama_attention(None)  # idempotent: the saved forward stays the stock one
    assert modeling_llama.LlamaAttention.forward is llama._turbo_attention_forward
    llama.unpatch_llama_attention(None)
    assert modeling_llama.LlamaAttention.forward is orig
    llama.unpatch_llama_attention(None)
    assert modeling_llama.LlamaAttention.forward is orig


# ---------------------------------------------------------------- GPU: against the reference adapter
def _dev():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    from turbopolar_b200 import build
    build.build()
    return torch.device("cuda:0")


@pytest.mark.gpu
@pytest.mark.parametrize("name", list(inputs.ADAPTER_CASES))
def test_fast_cache_decode_sequence_vs_reference(name, golden, golden_meta):
    """TurboPolarFastCache.decode_attention step by step against the reference adapter's
    outputs on the same tokens (dense-only, block boundary and compressed + tail steps)."""
    dev = _dev()
    from turbopolar_b200 import TurboPolarConfig
    from turbopolar_b200.llama import TurboPolarFastCache
    cfg = TurboPolarConfig(head_dim=128, block_size=64, num_q_heads=4, num_kv_heads=2, storage_mode="kv_quant",
                           **inputs.ADAPTER_CASES[name])
    cache = TurboPolarFastCache(cfg)
    qs, ks, vs = inputs.adapter_inputs()
    want = golden[f"adapter/{name}/out"]
    k_all = np.concatenate(list(ks), 2)
    v_all = np.concatenate(list(vs), 2)
    err_ref = err_oracle = 0.0
    for i in range(qs.shape[0]):
        out = cache.decode_attention(torch.from_numpy(qs[i]).to(dev), torch.from_numpy(ks[i]).to(dev),
                                     torch.from_numpy(vs[i]).to(dev), cfg.attention_scale)
        assert out.shape == (1, 4, 128) and out.dtype == torch.float16
        got = out.float().cpu().numpy().astype(np.float64)
        exact = oracle_attention(qs[i][0, :, 0], k_all[:, :, :i + 1], v_all[:, :, :i + 1], fmt_of(cfg),
                                 cfg.use_int8_radii, cfg.attention_scale)
        err_oracle = max(err_oracle, float(np.max(np.abs(got[0] - exact))))
        err_ref = max(err_ref, float(np.max(np.abs(got - want[i].astype(np.float64)))))
    assert err_oracle < ATOL, err_oracle               # float64 oracle on the same tokens
    assert err_ref < 3e-3, (err_ref, err_oracle)      # the reference adapter reduces in float16
    assert cache.offset == qs.shape[0]
    assert cache.runtime.get_io_telemetry() == pytest.approx(golden_meta[f"adapter/{name}"]["telemetry"])
    assert cache.nbytes == golden_meta[f"adapter/{name}"]["telemetry"]["actual_cache_bytes"]


@pytest.mark.gpu
def test_update_and_fetch_vs_reference(golden):
    """Prefill decompress-on-read (tail padded, encoded and decoded) bit-exact against the
    reference adapter, for a first and a second prefill chunk."""
    dev = _dev()
    from turbopolar_b200 import TurboPolarConfig
    from turbopolar_b200.llama import TurboPolarFastCache
    cfg = TurboPolarConfig(head_dim=128, block_size=64, num_q_heads=4, num_kv_heads=2, **ADAPTER_FMT)
    cache = TurboPolarFastCache(cfg)
    kp, vp, kp2, vp2 = inputs.prefill_inputs()
    k1, v1 = cache.update_and_fetch(torch.from_numpy(kp).to(dev), torch.from_numpy(vp).to(dev))
    k2, v2 = cache.update_and_fetch(torch.from_numpy(kp2).to(dev), torch.from_numpy(vp2).to(dev))
    assert k1.shape == (1, 2, 100, 128) and k2.shape == (1, 2, 130, 128)
    for got, key in ((k1, "k_out"), (v1, "v_out"), (k2, "k_out2"), (v2, "v_out2")):
        np.testing.assert_array_equal(got.cpu().numpy().view(np.uint16), golden[f"prefill/{key}"].view(np.uint16))
    # float32 inputs come back as float32
    cache2 = TurboPolarFastCache(cfg)
    k3, _ = cache2.update_and_fetch(torch.from_numpy(kp).to(dev).float(), torch.from_numpy(vp).to(dev).float())
    assert k3.dtype == torch.float32


def _logit_gate(base: np.ndarray, cand: np.ndarray) -> dict:
    """The reference's teacher-forced logit metrics (``turbo_polar_metrics.py``) in NumPy."""
    def log_softmax(x):
        x = x - x.max(axis=-1, keepdims=True)
        return x - np.log(np.exp(x).sum(axis=-1, keepdims=True))
    lp, lq = log_softmax(base), log_softmax(cand)
    kl = float(np.mean(np.sum(np.exp(lp) * (lp - lq), axis=-1)))

    def overlap(k):
        bt = np.argpartition(base, -k, axis=-1)[..., -k:].reshape(-1, k)
        ct = np.argpartition(cand, -k, axis=-1)[..., -k:].reshape(-1, k)
        return float(np.mean([len(set(b.tolist()) & set(c.tolist())) / k for b, c in zip(bt, ct)]))
    d = np.abs(base - cand).ravel()
    cos = float(np.dot(base.ravel(), cand.ravel()) / (np.linalg.norm(base) * np.linalg.norm(cand) + 1e-12))
    m = dict(logit_cosine=cos, kl_divergence=kl, top5_overlap=overlap(5), top10_overlap=overlap(10),
             mean_abs_logit_delta=float(d.mean()), p99_abs_logit_delta=float(np.percentile(d, 99)),
             max_logit_delta=float(d.max()))
    m["gate_passed"] = (cos >= 0.999 and kl <= 0.05 and m["top5_overlap"] >= 0.90 and m["top10_overlap"] >= 0.95
                        and m["mean_abs_logit_delta"] <= 0.02 and m["p99_abs_logit_delta"] <= 0.2
                        and m["max_logit_delta"] <= 1.0)
    return m


def _tiny_llama(dev, seed=3):
    from transformers import LlamaConfig, LlamaForCausalLM
    cfg = LlamaConfig(vocab_size=512, hidden_size=512, intermediate_size=1024, num_hidden_layers=2,
                      num_attention_heads=4, num_key_value_heads=2, head_dim=128, rope_theta=500000.0,
                      max_position_embeddings=4096, attn_implementation="sdpa")
    torch.manual_seed(seed)
    model = LlamaForCausalLM(cfg)
    with torch.no_grad():
        for p in model.parameters():
            p.normal_(0.0, 0.02)
    return model.half().to(dev).eval()


@pytest.mark.gpu
def test_llama_teacher_forced_logits_vs_dense_cache():
    """Random-init Llama, prompt of 96 tokens then 40 teacher-forced decode tokens: logits
    with the TurboPolar cache (prefill through update_and_fetch, decode through the fused
    kernel) against a dense fp16 cache, under the reference's gate."""
    dev = _dev()
    from transformers import DynamicCache
    from turbopolar_b200 import llama
    model = _tiny_llama(dev)
    rng = np.random.default_rng(3)
    ids = torch.from_numpy(rng.integers(0, 512, size=(1, 136))).to(dev)
    prompt, rest = ids[:, :96], ids[:, 96:]

    def run(cache):
        logits = []
        with torch.no_grad():
            out = model(input_ids=prompt, past_key_values=cache, use_cache=True)
            logits.append(out.logits[:, -1].float())
            for t in range(rest.shape[1]):
                out = model(input_ids=rest[:, t:t + 1], past_key_values=cache, use_cache=True)
                logits.append(out.logits[:, -1].float())
        return torch.cat(logits).cpu().numpy()

    base = run(DynamicCache())
    llama.patch_llama_attention(model)
    try:
        caches = llama.make_turbo_caches(2, 4, 2, 128)
        cand = run(caches)
    finally:
        llama.unpatch_llama_attention(model)
    assert caches[0].offset == 136
    m = _logit_gate(base, cand)
    assert m["gate_passed"], m
