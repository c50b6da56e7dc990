"""End-to-end decode on the device path (the end-to-end configuration's shape at 2 layers):
a random-init Llama (hidden 2048, 32 query / 8 KV heads x 128, FFN 8192, RoPE theta 500000,
vocabulary 32000) prefilled with a 2048-token prompt, then decoded one CUDA-graph replay per
token (``llama_graph.LlamaDecodeGraph``).

* The captured dense step (flash-attention decode) reproduces Hugging Face's own eager forward.
* The fused TurboPolar step (tp_decode_step per layer, adapter key format) matches the same cache
  attended in float32 over its decoded pages: the kernel's arithmetic adds little to the format.
* Teacher-forced on the dense run's greedy tokens, its logits pass the reference's gate
  (``rfsn_v11/candidates/turbo_polar_adapter.py:97-105``).
"""

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu

LAYERS, VOCAB, PROMPT, NEW = 2, 32000, 2048, 12


@pytest.fixture(scope="module")
def setup():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    from turbopolar_b200 import build
    from turbopolar_b200.bench_llama import build_model
    build.build()
    dev = torch.device("cuda:0")
    model = build_model(LAYERS, VOCAB, dev)
    prompt = torch.from_numpy(np.random.default_rng(3).integers(0, VOCAB, size=(1, PROMPT))).to(dev)
    return model, prompt, dev


def _turbo(model, prompt, dev, max_len):
    from turbopolar_b200 import llama
    from turbopolar_b200.bench_llama import prefill
    llama.patch_llama_attention(model)
    try:
        caches = llama.make_turbo_caches(LAYERS, 32, 8, 128, device=dev, max_seq_len=max_len, check_finite=False)
        first = prefill(model, prompt, caches)
    finally:
        llama.unpatch_llama_attention(model)
    return caches, first


def test_graph_decode_dense_hf_fused_and_format_only(setup):
    from transformers import DynamicCache
    from turbopolar_b200.bench_llama import logit_gate, prefill
    from turbopolar_b200.llama_graph import LlamaDecodeGraph
    model, prompt, dev = setup
    max_len = PROMPT + NEW + 64

    # Dense, greedy, captured.
    dc = DynamicCache()
    first = prefill(model, prompt, dc)
    dense = LlamaDecodeGraph(model, dc, max_len)
    dense.capture()
    tok = first.argmax(-1, keepdim=True)
    tokens, base = [tok], []
    dense.token.copy_(tok)
    for _ in range(NEW):
        dense.step()
        base.append(dense.logits.clone())
        tokens.append(dense.next.clone())
        dense.token.copy_(dense.next)
    tokens = torch.cat(tokens[:NEW], 1)
    base = torch.cat(base).cpu().numpy()

    # Hugging Face's eager forward on the same tokens.
    dc2 = DynamicCache()
    prefill(model, prompt, dc2)
    hf = []
    with torch.no_grad():
        for t in range(NEW):
            hf.append(model(input_ids=tokens[:, t:t + 1], past_key_values=dc2, use_cache=True).logits[:, -1].float())
    hf = torch.cat(hf).cpu().numpy()
    assert np.abs(base - hf).max() < 0.03, np.abs(base - hf).max()
    assert np.array_equal(base.argmax(-1), hf.argmax(-1))

    # Fused TurboPolar (captured) and format only (eager), teacher-forced.
    caches, _ = _turbo(model, prompt, dev, max_len)
    fused = LlamaDecodeGraph(model, caches, max_len)
    out_f = torch.empty((NEW, VOCAB), device=dev)
    fused.decode(tokens[:, :1], NEW, forced=tokens, logits_out=out_f)
    assert sum(layer.runtime.read_device_error() for layer in caches.layers) == 0
    assert all(layer.offset == PROMPT + NEW for layer in caches.layers)
    caches2, _ = _turbo(model, prompt, dev, max_len)
    only = LlamaDecodeGraph(model, caches2, max_len, attention="decompressed")
    out_o = torch.empty((NEW, VOCAB), device=dev)
    only.decode(tokens[:, :1], NEW, forced=tokens, logits_out=out_o)
    f, o = out_f.cpu().numpy(), out_o.cpu().numpy()
    assert np.abs(f - o).max() < 0.03, np.abs(f - o).max()
    gate = logit_gate(base, f)
    assert gate["gate_passed"], gate
