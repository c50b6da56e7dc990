"""End-to-end decode with a random-init Llama: the TurboPolar cache against a dense fp16 cache.

    python -m turbopolar_b200.bench_llama [--layers 16 --prompt 2048 --new 256]

The model is the Llama-3.2-1B architecture with 128-channel heads (hidden 2048, 32 query / 8
KV heads x head_dim 128, FFN 8192, vocabulary 128256, RMSNorm, RoPE theta 500000) built by
Hugging Face ``transformers`` from a config, weights ~ N(0, 0.02) in fp16 (seeded; no
checkpoint).  The prompt is uniform random token ids (seed 3).  The dense run prefills the
prompt and decodes ``--new`` tokens greedily; the TurboPolar run (``patch_llama_attention`` +
``make_turbo_caches``: prefill through decompress-on-read, decode through the fused CUDA kernel)
is fed the same tokens (teacher forcing), so the logits of every step compare one to one under
the reference's gate (``rfsn_v11/candidates/turbo_polar_adapter.py:97-105``).  Tokens/s is the
decode phase of each run after a short warm-up run (CUDA events around the token loop; Python
dispatch and the reference's per-append finiteness check included).
Prints one JSON line.
"""

from __future__ import annotations

import argparse
import json

import numpy as np
import torch


def build_model(layers: int, vocab: int, dev, seed: int = 0):
    from transformers import LlamaConfig, LlamaForCausalLM
    cfg = LlamaConfig(vocab_size=vocab, hidden_size=2048, intermediate_size=8192, num_hidden_layers=layers,
                      num_attention_heads=32, num_key_value_heads=8, head_dim=128, rope_theta=500000.0,
                      max_position_embeddings=8192, rms_norm_eps=1e-5, attn_implementation="sdpa",
                      tie_word_embeddings=True)
    torch.manual_seed(seed)
    with torch.device(dev):
        model = LlamaForCausalLM(cfg).half()
    with torch.no_grad():
        for name, p in model.named_parameters():
            if "norm" in name:
                p.fill_(1.0)
            else:
                p.normal_(0.0, 0.02)
    return model.eval()


def logit_gate(base: np.ndarray, cand: np.ndarray) -> dict:
    """The reference's teacher-forced logit metrics (``turbo_polar_metrics.py``)."""
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
             max_logit_delta=float(d.max()),
             greedy_agreement=float(np.mean(base.argmax(-1) == cand.argmax(-1))))
    m["gate_passed"] = bool(cos >= 0.999 and kl <= 0.05 and m["top5_overlap"] >= 0.90 and m["top10_overlap"] >= 0.95
                            and m["mean_abs_logit_delta"] <= 0.02 and m["p99_abs_logit_delta"] <= 0.2
                            and m["max_logit_delta"] <= 1.0)
    return m


def run(model, prompt: torch.Tensor, new: int, cache, forced=None):
    """Prefill, then `new` decode steps (greedy, or the `forced` tokens).  Returns the logits of
    the prefill's last position and of every decode step, the tokens, and decode seconds."""
    logits, tokens = [], []
    with torch.no_grad():
        out = model(input_ids=prompt, past_key_values=cache, use_cache=True)
        last = out.logits[:, -1].float()
        torch.cuda.synchronize()
        s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        s.record()
        for t in range(new):
            logits.append(last)
            nxt = last.argmax(-1, keepdim=True) if forced is None else forced[:, t:t + 1]
            tokens.append(nxt)
            out = model(input_ids=nxt, past_key_values=cache, use_cache=True)
            last = out.logits[:, -1].float()
        e.record()
        torch.cuda.synchronize()
    return torch.cat(logits).cpu().numpy(), torch.cat(tokens, dim=1), s.elapsed_time(e) / 1e3


def main(argv=None):
    ap = argparse.ArgumentParser()
    ap.add_argument("--layers", type=int, default=16)
    ap.add_argument("--prompt", type=int, default=2048)
    ap.add_argument("--new", type=int, default=256)
    ap.add_argument("--vocab", type=int, default=128256)
    a = ap.parse_args(argv)
    from transformers import DynamicCache
    from . import build, llama
    build.build()
    dev = torch.device("cuda:0")
    # The dense baseline's attention: torch SDPA without the cuDNN backend, which builds a new
    # execution plan for every new key length (each decode step) and would time that instead.
    torch.backends.cuda.enable_cudnn_sdp(False)
    model = build_model(a.layers, a.vocab, dev)
    rng = np.random.default_rng(3)
    prompt = torch.from_numpy(rng.integers(0, a.vocab, size=(1, a.prompt))).to(dev)

    run(model, prompt[:, :64], 4, DynamicCache())  # warm-up (kernel selection, allocator)
    base, toks, t_dense = run(model, prompt, a.new, DynamicCache())
    llama.patch_llama_attention(model)
    try:
        run(model, prompt[:, :64], 4, llama.make_turbo_caches(a.layers, 32, 8, 128), forced=toks)  # warm-up
        caches = llama.make_turbo_caches(a.layers, 32, 8, 128)
        cand, _, t_turbo = run(model, prompt, a.new, caches, forced=toks)
    finally:
        llama.unpatch_llama_attention(model)
    dense_bytes = a.layers * 2 * 8 * 128 * 2 * (a.prompt + a.new)
    line = {
        "workload": f"random-init Llama ({a.layers} layers, hidden 2048, 32q/8kv x 128, FFN 8192, vocab {a.vocab})",
        "prompt_tokens": a.prompt, "decode_tokens": a.new, "dtype": "f16", "data": "synthetic (seeded ids)",
        "dense_tokens_per_s": a.new / t_dense, "turbopolar_tokens_per_s": a.new / t_turbo,
        "kv_bytes_dense": dense_bytes, "kv_bytes_turbopolar": int(sum(c.nbytes for c in caches)),
        "logits": logit_gate(base, cand),
    }
    print(json.dumps(line), flush=True)


if __name__ == "__main__":
    main()
