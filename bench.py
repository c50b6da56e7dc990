"""Benchmark: compressed-KV decode attention, Llama-3-8B attention shape, 32K context.

Workload (config 3 of the measurement plan): 32 layers, 32 query / 8 KV heads, head_dim 128,
block 64, batch 1, fp16, default key format (4-bit level-1 and deep angles, split_dim 64,
float16 radii) and grouped int8 values.  Each layer's cache is prefilled with 32768 synthetic
tokens (K ~ N(0,1) * c with a fixed per-channel c ~ U(0.5, 4), V ~ N(0,1), seeded), then a
"step" is one decode step: for every layer, append one token and run fused attention (one
tp_decode_step call per layer).  The step is captured once as a CUDA graph (the cache
counters live on the device) and replayed.

Reported (one JSON line on rank 0):
  value     -- decode-attention HBM GB/s over the whole job: algorithmic compressed bytes per
               step (pages + dense tail + q + out, all layers, all ranks) / device step time
  e2e       -- the same metric with every step's inputs copied from pinned host memory and the
               attention outputs copied back, inside the timed region
  roofline  -- the attention kernel alone, timed per launch with CUDA events, against the
               measured HBM copy bandwidth: 32 independent layers in a graph (consecutive
               calls overlap), and as dependent_launch_us / dependent_frac the same launches
               with each layer's query read from the previous layer's output (no overlap)
  strong_128k -- config 4: one 131072-token context per layer split over the N ranks, a
               32-layer decode step; per-layer us, whole-job GB/s and per-GPU fraction of peak
  sharded   -- (N > 1) a probe context split over the ranks, three decode steps through both
               cross-GPU merges (in-launch NVLink exchange and NCCL all-gather), against one GPU
               holding the whole probe and against a float64 softmax over the decoded cache
  c2        -- (N = 1) config 2: 4096-token caches, 1000 seeded queries; us per call
               (independent and dependent), GB/s, and the maximum error over all 1000 queries
               against a float64 softmax over the decoded cache
  cpu_baseline -- the NumPy restatement of the reference's CPU-fallback math on a bounded sample

Multi-GPU (torchrun, N>1): one sequence of N x 32K tokens per layer, split into contiguous
page ranges, one 32K range per rank (the last rank also holds the tail and the new tokens);
every rank's attention launch publishes its per-query-head partial (max, sum, output) into
every rank's buffer over NVLink and merges them (log-sum-exp) in the same launch.  Per-GPU work
is fixed, so scaling is "weak" (``--scaling strong --ctx C`` splits one C-token context).

``--impl reference`` times the NumPy restatement of the reference's CPU fallback
(rfsn_v11/kernels/turbo_polar/metal.py:293-332) instead: the reference itself runs on MLX,
which is absent here, and its Python sources do not travel to the GPU box.
"""

from __future__ import annotations

import argparse
import json
import math
import os
import shutil
import statistics
import subprocess
import sys
import tempfile
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

CTX = 32768
CTX_C4 = 131072
CTX_C2 = 4096
LAYERS = 32
HQ, HKV, D = 32, 8, 128
PAGE = 64
PAGE_BYTES_DEFAULT = 64 * 296  # per page per KV head: radii 8192 + codes 2048 + V 8192 + scales 512
L2_BYTES = 126 * 2 ** 20
METRIC = "decode-attention HBM GB/s (% of B200 peak) and decode tokens/s at 32K ctx"


def _peaks():
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            p = json.load(f)
        return float(p["hbm_gbs"]), "measured"
    except Exception:
        return 6650.0, "fallback"


def _traffic_from_profile():
    """DRAM bytes per attention launch from the committed ncu summary, or None."""
    try:
        with open(os.path.join(ROOT, "profiles", "decode_attention_traffic.json")) as f:
            return json.load(f)
    except Exception:
        return None


def attention_bytes(n_pages: int, tail: int, hkv: int = HKV, hq: int = HQ) -> int:
    """Algorithmic bytes of one attention call: compressed pages + dense fp16 tail + q + out."""
    return n_pages * hkv * PAGE_BYTES_DEFAULT + tail * hkv * D * 2 * 2 + hq * D * 2 * 2


def _total_ctx(args, world: int) -> int:
    return args.ctx * world if args.scaling == "weak" else args.ctx


def workload_config(args, world: int) -> dict:
    """The workload both arms report (identical keys and values)."""
    ctx = _total_ctx(args, world)
    return {"workload": "llama3-8b-attention-32layers-32k-decode", "ctx": ctx, "ctx_per_gpu": ctx // world,
            "layers": LAYERS, "num_q_heads": HQ, "num_kv_heads": HKV, "head_dim": D, "batch": 1,
            "format": "fp16 radii, 4-bit angles (split 64), int8 V group 32",
            "parallelism": f"sequence-shard x{world}" if world > 1 else "single GPU",
            "l2": f"inputs larger than L2 ({LAYERS * (ctx // world // PAGE) * HKV * PAGE_BYTES_DEFAULT / 1e9:.2f} GB "
                  "of pages per step per GPU vs 126 MB L2)"}


# ----------------------------------------------------------------------------- clocks
class ClockSampler:
    def __init__(self, index: int):
        self.index = index
        self.proc = None
        self.path = None

    def __enter__(self):
        fd, self.path = tempfile.mkstemp(suffix=".csv")
        os.close(fd)
        q = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
             "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
             "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")
        try:
            self.proc = subprocess.Popen(["nvidia-smi", f"--id={self.index}", f"--query-gpu={q}",
                                          "--format=csv,noheader,nounits", "-lms", "100"],
                                         stdout=open(self.path, "w"), stderr=subprocess.DEVNULL)
        except Exception:
            self.proc = None
        time.sleep(0.3)
        return self

    def __exit__(self, *exc):
        if self.proc is not None:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except Exception:
                self.proc.kill()

    def summary(self):
        rows = []
        try:
            for line in open(self.path):
                parts = [p.strip() for p in line.split(",")]
                if len(parts) >= 9:
                    rows.append(parts)
        except Exception:
            pass
        finally:
            try:
                os.unlink(self.path)
            except Exception:
                pass
        if not rows:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unavailable"]}
        sm = [float(r[1]) for r in rows if r[1].replace(".", "").isdigit()]
        smax = [float(r[2]) for r in rows if r[2].replace(".", "").isdigit()]
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({n for r in rows for n, v in zip(names, r[5:9]) if v.lower() == "active"})
        loaded = sorted(sm)[len(sm) // 4:] if sm else []
        return {"sm_mhz": statistics.median(loaded) if loaded else None,
                "sm_max_mhz": max(smax) if smax else None, "reasons": reasons, "samples": len(rows)}


# ----------------------------------------------------------------------------- CPU baseline
# The reference's CPU fallback (metal.py:293-332) decodes every page, dequantises the values and
# takes one softmax per query head.  Restated in NumPy (oracle/), it runs here over page chunks
# of each KV head in a spawn process pool (all host cores), each chunk giving an unnormalised
# (max, sum, output) record per query head, merged per head by log-sum-exp: the same softmax,
# split for the cores.  Chunks live in memory-mapped .npy files, so a call ships no pages.
_CHUNKS = {}  # per worker process: the memory maps of the chunks it has seen (shared page cache)
_LIMITS = []


def _one_thread():
    """Pool initializer: one BLAS/OpenMP thread per worker (the pool already uses every core)."""
    from threadpoolctl import threadpool_limits
    _LIMITS.append(threadpool_limits(1))


def _cpu_chunk(args):
    from oracle import attention as oatt
    path, fmt, q, scale = args
    pages = _CHUNKS.get(path)
    if pages is None:
        pages = {name: np.load(os.path.join(path, name + ".npy"), mmap_mode="r") for name in
                 ("radii", "angle_codes_l1", "angle_codes_deep", "v_codes", "v_scales")}
        pages["radii_scales"] = None
        _CHUNKS[path] = pages
    k, v = oatt.decode_pages(pages, fmt)
    return oatt.partial(q, k, v, scale)


class CpuReference:
    """One layer's attention call at ``ctx`` tokens on the host cores (the bounded sample)."""

    def __init__(self, ctx: int, tmp: str):
        import multiprocessing as mp
        from oracle import polar, vquant
        rng = np.random.default_rng(0)
        c = np.random.default_rng(1).uniform(0.5, 4.0, size=128).astype(np.float32)
        n = ctx // PAGE
        self.ctx, self.n_pages = ctx, n
        self.cores = max(1, os.cpu_count() or 1)
        chunks = max(1, min(n, -(-self.cores // HKV)))  # chunks per KV head
        fmt = dict(l1_bits=4, deep_bits=4, split_dim=64)
        self.work, self.heads = [], []
        for h in range(HKV):
            k = (rng.standard_normal((1, n, PAGE, D)).astype(np.float32) * c).astype(np.float16)
            v = rng.standard_normal((1, n, PAGE, D)).astype(np.float16)
            enc = polar.encode_block(k)
            codes, scales = vquant.quantize(v)
            q = rng.standard_normal((HQ // HKV, D)).astype(np.float16).astype(np.float64)
            for j in range(chunks):
                a, b = j * n // chunks, (j + 1) * n // chunks
                if a == b:
                    continue
                path = os.path.join(tmp, f"h{h}c{j}")
                os.makedirs(path)
                for name, arr in (("radii", enc["radii"]), ("angle_codes_l1", enc["angle_codes_l1"]),
                                  ("angle_codes_deep", enc["angle_codes_deep"]), ("v_codes", codes),
                                  ("v_scales", scales)):
                    np.save(os.path.join(path, name + ".npy"), np.ascontiguousarray(arr[:, a:b]))
                self.work.append((path, fmt, q, 1 / math.sqrt(D)))
                self.heads.append(h)
        self.workers = min(self.cores, len(self.work))
        self.pool = mp.get_context("spawn").Pool(self.workers, initializer=_one_thread)

    def call(self) -> np.ndarray:
        from oracle import attention as oatt
        parts = self.pool.map(_cpu_chunk, self.work)
        return np.concatenate([oatt.combine(np.stack([p for p, hh in zip(parts, self.heads) if hh == h]))
                               for h in range(HKV)])

    def close(self):
        self.pool.terminate()
        self.pool.join()


def cpu_baseline(seconds_target: float = 15.0, ctx: int = CTX):
    """Time the CPU restatement of the reference fallback on one layer at ``ctx`` tokens for
    about ``seconds_target`` seconds."""
    tmp = tempfile.mkdtemp(prefix="tp_cpu_")
    ref = CpuReference(ctx, tmp)
    try:
        ref.call()  # warm the workers
        calls, t0 = 0, time.perf_counter()
        while True:
            ref.call()
            calls += 1
            if time.perf_counter() - t0 >= seconds_target:
                break
        dt = (time.perf_counter() - t0) / calls
    finally:
        ref.close()
        shutil.rmtree(tmp, ignore_errors=True)
    byts = attention_bytes(ref.n_pages, 0)
    return {"value": byts / dt / 1e9, "unit": "GB/s", "cores": ref.workers, "kind": "port",
            "sample": f"{calls} single-layer attention calls at {ctx} tokens, {HQ}q/{HKV}kv, "
                      f"{ref.workers} processes ({dt * 1e3:.1f} ms/call)",
            "ms_per_layer_call": dt * 1e3}


def run_reference(args):
    """The reference arm: every step is one layer's attention call at the workload's context
    (1/32 of the GPU arm's decode step), run on the host cores; `steps` of them are timed after
    `warmup` untimed ones."""
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    if rank != 0:
        return 0
    ctx = _total_ctx(args, world)
    tmp = tempfile.mkdtemp(prefix="tp_ref_")
    ref = CpuReference(ctx, tmp)
    try:
        for _ in range(args.warmup):
            ref.call()
        t0 = time.perf_counter()
        for _ in range(args.steps):
            ref.call()
        dt = (time.perf_counter() - t0) / args.steps
    finally:
        ref.close()
        shutil.rmtree(tmp, ignore_errors=True)
    byts = attention_bytes(ref.n_pages, 0)
    value = byts / dt / 1e9
    sample = (f"{args.steps} timed single-layer attention calls at {ctx} tokens, {HQ}q/{HKV}kv, "
              f"{ref.workers} processes over page chunks ({dt * 1e3:.1f} ms/call)")
    line = {
        "metric": METRIC, "value": value, "unit": "GB/s", "n_gpus": args.gpus, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": dt * 1e3, "higher_is_better": True, "scaling": args.scaling,
        "vs_baseline": None, "dtype": "f16", "data": "synthetic", "impl": "reference",
        "config": workload_config(args, world),
        "step": "one layer's attention call over the whole context (the GPU arm's step is 32 of them)",
        "cpu_baseline": {"value": value, "unit": "GB/s", "cores": ref.workers, "kind": "port", "sample": sample},
        "e2e": {"value": value, "unit": "GB/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)
    return 0


# ----------------------------------------------------------------------------- GPU arm
def _make_layers(cfg, ctx_total, world, rank, dev, extra_tokens, seed0, n_layers=LAYERS):
    """Per-layer caches holding this rank's contiguous page range of a ctx_total-token context."""
    import torch
    from turbopolar_b200 import TurboPolarKVCacheRuntime, sharded
    lo, hi = sharded.page_range(ctx_total // PAGE, rank, world)
    last = rank == world - 1
    cap_tokens = (hi - lo) * PAGE + (extra_tokens + PAGE if last else 0)
    chan = torch.from_numpy(np.random.default_rng(1).uniform(0.5, 4.0, size=D).astype(np.float32)).to(dev)
    gen = torch.Generator(device=dev)
    layers = []
    for layer in range(n_layers):
        rt = TurboPolarKVCacheRuntime(cfg, max_seq_len=cap_tokens, check_finite=False, first_page=lo)
        gen.manual_seed(seed0 + 64 * layer + rank)  # each rank draws its own slice of the sequence
        k = (torch.randn((1, HKV, (hi - lo) * PAGE, D), generator=gen, device=dev) * chan).half()
        v = torch.randn((1, HKV, (hi - lo) * PAGE, D), generator=gen, device=dev).half()
        rt.append(k, v)
        if world > 1:
            rt.set_global_length(ctx_total)
        del k, v
        layers.append(rt)
    return layers


def _step_io(dev, seed):
    """New K, V and q of every layer as views of one device buffer, outputs of another."""
    import torch
    gen = torch.Generator(device=dev)
    gen.manual_seed(seed)
    per_layer_in = 2 * HKV * D + HQ * D
    d_in = torch.randn((LAYERS, per_layer_in), generator=gen, device=dev).half()
    d_out = torch.empty((LAYERS, 1, HQ, D), dtype=torch.float16, device=dev)
    k_in = [d_in[i, :HKV * D].view(1, HKV, 1, D) for i in range(LAYERS)]
    v_in = [d_in[i, HKV * D:2 * HKV * D].view(1, HKV, 1, D) for i in range(LAYERS)]
    q_in = [d_in[i, 2 * HKV * D:].view(1, HQ, D) for i in range(LAYERS)]
    out = [d_out[i] for i in range(LAYERS)]
    return d_in, d_out, k_in, v_in, q_in, out


def _decode_step(layers, k_in, v_in, q_in, out, rank, world):
    from turbopolar_b200 import graph, sharded
    if world == 1:
        return graph.DecodeStep(None, layers=[(layers[i], k_in[i], v_in[i], q_in[i], out[i]) for i in range(LAYERS)])
    return sharded.ShardedDecodeStep(layers, k_in, v_in, q_in, out, rank, world)


def _step_bytes(ctx_total, steps_before, steps, world):
    """Algorithmic bytes of `steps` decode steps after `steps_before` earlier ones: every step
    reads the whole context once per layer (split over ranks), plus q and out per rank."""
    total = 0
    for i in range(steps):
        full, tail = divmod(ctx_total + steps_before + i + 1, PAGE)
        total += LAYERS * (full * HKV * PAGE_BYTES_DEFAULT + tail * HKV * D * 4 + world * HQ * D * 4)
    return total


def _max_over_ranks(x: float, world: int, dev) -> float:
    if world == 1:
        return x
    import torch
    import torch.distributed as dist
    t = torch.tensor([x], device=dev, dtype=torch.float64)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def _barrier(world):
    import torch
    import torch.distributed as dist
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()


def _time_replays(step, n, world, dev) -> float:
    """Device ms per replay of `step` over n replays, bracketed by barriers; max over ranks."""
    import torch
    _barrier(world)
    s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    s.record()
    for _ in range(n):
        step.replay()
    e.record()
    _barrier(world)
    return _max_over_ranks(s.elapsed_time(e), world, dev) / n


def _graph_us(launch_all, calls, reps=20) -> float:
    """Device us per call of a captured graph of `calls` attention calls."""
    import torch
    g = torch.cuda.CUDAGraph()
    torch.cuda.synchronize()
    with torch.cuda.graph(g):
        launch_all()
    for _ in range(3):
        g.replay()
    torch.cuda.synchronize()
    s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    s.record()
    for _ in range(reps):
        g.replay()
    e.record()
    torch.cuda.synchronize()
    del g
    return s.elapsed_time(e) / (reps * calls) * 1e3


def _fp64_attention(q, k, v, scale):
    """float64 softmax attention of q [n, H_q, 128] over dense k, v [H_kv, T, 128] (the
    reference fallback's formula, metal.py:305-321, on the decoded cache)."""
    import torch
    g = q.shape[1] // k.shape[0]
    kk = k.double().repeat_interleave(g, dim=0)          # [H_q, T, 128]
    vv = v.double().repeat_interleave(g, dim=0)
    s = torch.einsum("nhd,htd->nht", q.double(), kk) * scale
    w = torch.softmax(s, dim=-1)
    return torch.einsum("nht,htd->nhd", w, vv)


def _strong_128k(cfg, world, rank, dev, peak):
    """Config 4: one 131072-token context per layer split over the ranks; a 32-layer decode step
    (append + attention per layer) in a CUDA graph, 16 timed replays after 3."""
    import torch
    steps, warm = 16, 3
    layers = _make_layers(cfg, CTX_C4, world, rank, dev, steps + warm + 2, seed0=50000)
    d_in, d_out, k_in, v_in, q_in, out = _step_io(dev, 11)
    step = _decode_step(layers, k_in, v_in, q_in, out, rank, world)
    for _ in range(warm):
        step.replay()
    ms = _time_replays(step, steps, world, dev)
    byts = _step_bytes(CTX_C4, warm, steps, world) / steps
    err = sum(rt.read_device_error() for rt in layers)
    if hasattr(step, "release"):
        step.release()
    del step, layers
    torch.cuda.empty_cache()
    gbs = byts / (ms * 1e-3) / 1e9
    return {"ctx": CTX_C4, "ctx_per_gpu": CTX_C4 // world, "n_gpus": world, "layers": LAYERS, "steps": steps,
            "ms_per_step": ms, "us_per_layer": ms * 1e3 / LAYERS, "gbs_job": gbs, "gbs_per_gpu": gbs / world,
            "frac_per_gpu": gbs / world / peak, "device_errors": err,
            "what": "32-layer decode step (append + attention per layer), one 128K context per layer "
                    "split contiguously over the ranks, merged in the launch over NVLink"}


def _sharded_probe(cfg, world, rank, dev):
    """A probe context split over the ranks, three decode steps through each cross-GPU merge,
    against one GPU holding the whole probe (rank 0) and a float64 softmax over it."""
    import torch
    import torch.distributed as dist
    from turbopolar_b200 import TurboPolarKVCacheRuntime, sharded
    t0, steps = 64 * 37 + 21, 3
    gen = torch.Generator(device=dev)
    gen.manual_seed(4242)  # the same full probe on every rank
    chan = torch.from_numpy(np.random.default_rng(1).uniform(0.5, 4.0, size=D).astype(np.float32)).to(dev)
    k = (torch.randn((1, HKV, t0 + steps, D), generator=gen, device=dev) * chan).half()
    v = torch.randn((1, HKV, t0 + steps, D), generator=gen, device=dev).half()
    q = torch.randn((steps, 1, HQ, D), generator=gen, device=dev).half()
    lo, hi = sharded.page_range(t0 // PAGE, rank, world)
    end = t0 if rank == world - 1 else hi * PAGE
    got = {}
    for mode in ("nvlink_exchange", "nccl_allgather"):
        rt = TurboPolarKVCacheRuntime(cfg, first_page=lo, max_seq_len=(end - lo * PAGE) + steps + PAGE,
                                      check_finite=False)
        rt.append(k[:, :, lo * PAGE:end].contiguous(), v[:, :, lo * PAGE:end].contiguous())
        rt.set_global_length(t0)
        k_in = [torch.empty((1, HKV, 1, D), dtype=torch.float16, device=dev)]
        v_in = [torch.empty_like(k_in[0])]
        q_in = [torch.empty((1, HQ, D), dtype=torch.float16, device=dev)]
        out = [torch.empty((1, HQ, D), dtype=torch.float16, device=dev)]
        step = sharded.ShardedDecodeStep([rt], k_in, v_in, q_in, out, rank, world, exchange=mode == "nvlink_exchange")
        outs = []
        for s in range(steps):
            k_in[0].copy_(k[:, :, t0 + s:t0 + s + 1])
            v_in[0].copy_(v[:, :, t0 + s:t0 + s + 1])
            q_in[0].copy_(q[s])
            step.replay()
            outs.append(out[0].clone())
        step.release()
        got[mode] = torch.stack(outs).float()
    ref = torch.empty((steps, 1, HQ, D), dtype=torch.float32, device=dev)
    fp64_err = 0.0
    if rank == 0:
        full = TurboPolarKVCacheRuntime(cfg, max_seq_len=t0 + steps + PAGE, check_finite=False)
        full.append(k[:, :, :t0].contiguous(), v[:, :, :t0].contiguous())
        outs = [full.decode_step(k[:, :, t0 + s:t0 + s + 1].contiguous(), v[:, :, t0 + s:t0 + s + 1].contiguous(),
                                 q[s]).clone() for s in range(steps)]
        ref.copy_(torch.stack(outs).float())
        kd, vd = full.decompress(padded_tail=False)  # stored pages decoded + the dense tail
        for s in range(steps):
            want = _fp64_attention(q[s], kd[0, :, :t0 + s + 1], vd[0, :, :t0 + s + 1], cfg.attention_scale)
            fp64_err = max(fp64_err, float((ref[s].double() - want).abs().max()))
    dist.broadcast(ref, src=0)
    errs = {m: _max_over_ranks(float((g - ref).abs().max()), world, dev) for m, g in got.items()}
    return {"probe_tokens": t0, "decode_steps": steps, "ranks": world,
            "sharded_max_abs_err": max(errs.values()),
            "per_merge_max_abs_err": errs, "single_gpu_vs_fp64_max_abs_err": fp64_err, "tolerance": 2e-3,
            "what": "every rank's merged output of each step vs one GPU holding the whole probe "
                    "(tp_decode_step); that GPU's output vs a float64 softmax over its decoded cache"}


def _c2(cfg, dev, peak):
    """Config 2: 4096-token caches (enough of them to exceed 4x L2), 1000 seeded queries."""
    import torch
    from turbopolar_b200 import TurboPolarKVCacheRuntime
    n_caches = math.ceil(4 * L2_BYTES / (CTX_C2 // PAGE * HKV * PAGE_BYTES_DEFAULT))
    chan = torch.from_numpy(np.random.default_rng(1).uniform(0.5, 4.0, size=D).astype(np.float32)).to(dev)
    gen = torch.Generator(device=dev)
    caches = []
    for i in range(n_caches):
        gen.manual_seed(20000 + i)
        k = (torch.randn((1, HKV, CTX_C2, D), generator=gen, device=dev) * chan).half()
        v = torch.randn((1, HKV, CTX_C2, D), generator=gen, device=dev).half()
        rt = TurboPolarKVCacheRuntime(cfg, max_seq_len=CTX_C2, check_finite=False)
        rt.append(k, v)
        caches.append(rt)
    gen.manual_seed(2)
    qs = torch.randn((1000, 1, HQ, D), generator=gen, device=dev).half()
    outs = torch.empty((n_caches, 1, HQ, D), dtype=torch.float16, device=dev)
    for i, rt in enumerate(caches):
        rt.attention(qs[i], out=outs[i])
    torch.cuda.synchronize()
    ind = _graph_us(lambda: [rt.attention(qs[i], out=outs[i]) for i, rt in enumerate(caches)], n_caches)
    dep = _graph_us(lambda: [rt.attention(qs[0] if i == 0 else outs[i - 1], out=outs[i])
                             for i, rt in enumerate(caches)], n_caches)
    # Error: all 1000 queries on cache 0 against a float64 softmax over its decoded pages.
    got = torch.empty((1000, 1, HQ, D), dtype=torch.float16, device=dev)
    for j in range(1000):
        caches[0].attention(qs[j], out=got[j])
    kd, vd = caches[0].decompress(padded_tail=False)
    err = 0.0
    for a in range(0, 1000, 250):
        want = _fp64_attention(qs[a:a + 250, 0], kd[0], vd[0], cfg.attention_scale)
        err = max(err, float((got[a:a + 250, 0].double() - want).abs().max()))
    nbytes = attention_bytes(CTX_C2 // PAGE, 0)
    del caches
    torch.cuda.empty_cache()
    return {"ctx": CTX_C2, "caches": n_caches, "bytes_per_call": nbytes,
            "us_per_call_independent": ind, "gbs_independent": nbytes / ind / 1e3,
            "frac_independent": nbytes / ind / 1e3 / peak,
            "us_per_call_dependent": dep, "gbs_dependent": nbytes / dep / 1e3, "frac_dependent": nbytes / dep / 1e3 / peak,
            "queries_checked": 1000, "max_abs_err": err, "tolerance": 2e-3,
            "reference": "float64 softmax over the cache decoded by tp_decode_pages (bit-exact with the "
                         "reference decoder; the CPU oracle's formula)",
            "l2": f"{n_caches} distinct caches per graph ({n_caches * nbytes / 1e6:.0f} MB) > 4x L2"}


def run_gpu(args):
    import torch
    import torch.distributed as dist

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        from datetime import timedelta
        dist.init_process_group("nccl", timeout=timedelta(seconds=120), device_id=dev)

    from turbopolar_b200 import TurboPolarConfig, build, graph
    build.build()
    library = {"path": os.path.relpath(build.LIB, ROOT), "source_sha16": build.last_build["source_sha16"],
               "compiled_in_this_run": build.last_build["compiled"]}
    cfg = TurboPolarConfig(num_q_heads=HQ, num_kv_heads=HKV)
    ctx = _total_ctx(args, world)
    layers = _make_layers(cfg, ctx, world, rank, dev, args.steps + args.warmup + 2, seed0=1000)
    torch.cuda.synchronize()
    d_in, d_out, k_in, v_in, q_in, out = _step_io(dev, 7)
    step = _decode_step(layers, k_in, v_in, q_in, out, rank, world)

    for _ in range(args.warmup):
        step.replay()
    _barrier(world)
    with ClockSampler(local) as clocks:
        ms_step = _time_replays(step, args.steps, world, dev)
    value = _step_bytes(ctx, args.warmup, args.steps, world) / args.steps / (ms_step * 1e-3) / 1e9

    # ---- roofline: attention kernel alone, per launch, on its own stream (graph of 32 launches).
    # One call per layer, each on its own cache with its own query and output (consecutive
    # calls are independent, so a page pass may stream while the previous call finishes).
    kern_us = _graph_us(lambda: [graph.launch_attention(layers[i], q_in[i], out[i], cfg.attention_scale,
                                                        partial_out=step.partial_buffer(i) if world > 1 else None)
                                 for i in range(LAYERS)], LAYERS)
    # The same calls with each layer's query read from the previous layer's output, as in a
    # model: every call then waits for the previous one to complete before its page pass
    # streams, so this is the latency of one dependent call.
    dep_us = None
    if world == 1:
        dep_out = torch.empty((LAYERS, 1, HQ, D), dtype=torch.float16, device=dev)
        dep_us = _graph_us(lambda: [graph.launch_attention(layers[i], q_in[0] if i == 0 else dep_out[i - 1],
                                                           dep_out[i], cfg.attention_scale) for i in range(LAYERS)],
                           LAYERS)
    rt0 = layers[0]
    launch_bytes = attention_bytes(rt0.n_pages, rt0.tail_len, hq=HQ)
    peak, peak_kind = _peaks()
    achieved = launch_bytes / (kern_us * 1e-6) / 1e9
    tr = _traffic_from_profile()
    traffic = None
    if tr and world == 1:
        traffic = int(tr["dram_bytes_per_launch"] * (launch_bytes / tr["algorithmic_bytes_per_launch"]))
    roof = {"bound": "hbm", "achieved": achieved, "peak": peak, "unit": "GB/s", "frac": achieved / peak,
            "traffic": traffic, "peak_source": f"{peak_kind} hbm_gbs", "kernel": "decode_attention_kernel",
            "launch_us": kern_us, "algorithmic_bytes_per_launch": launch_bytes,
            "bytes_per_context_token": HKV * 296, "frac_of_8000_spec": achieved / 8000.0}
    if dep_us is not None:
        roof["dependent_launch_us"] = dep_us
        roof["dependent_frac"] = launch_bytes / (dep_us * 1e-6) / 1e9 / peak

    # ---- e2e: host inputs -> device, graph step, outputs -> host, every step.
    h_in = d_in.cpu().pin_memory()
    h_out = torch.empty(d_out.shape, dtype=torch.float16).pin_memory()
    e_steps = max(1, min(args.steps, 32))
    _barrier(world)
    s3, e3 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    t_wall = time.perf_counter()
    s3.record()
    for _ in range(e_steps):
        d_in.copy_(h_in, non_blocking=True)
        step.replay()
        h_out.copy_(d_out, non_blocking=True)
    e3.record()
    _barrier(world)
    e_ms = _max_over_ranks(s3.elapsed_time(e3), world, dev)
    t_wall = time.perf_counter() - t_wall
    e_step_bytes = _step_bytes(ctx, args.warmup + args.steps, e_steps, world) / e_steps
    e2e = {"value": e_step_bytes / (e_ms / e_steps * 1e-3) / 1e9, "unit": "GB/s",
           "h2d_bytes_per_step": h_in.numel() * h_in.element_size(),
           "d2h_bytes_per_step": h_out.numel() * h_out.element_size(), "steps": e_steps,
           "wall_ms_per_step": t_wall * 1e3 / e_steps}
    err = sum(rt.read_device_error() for rt in layers)
    if hasattr(step, "release"):
        step.release()
    del step, layers
    torch.cuda.empty_cache()

    # ---- extra records (after the timed region; every rank takes the same steps).
    extra = {}
    if not args.no_extras:
        if not (args.scaling == "strong" and ctx == CTX_C4):
            extra["strong_128k"] = _strong_128k(cfg, world, rank, dev, peak)
        if world > 1:
            extra["sharded"] = _sharded_probe(cfg, world, rank, dev)
        elif rank == 0:
            extra["c2"] = _c2(cfg, dev, peak)

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        cb = cpu_baseline(seconds_target=args.cpu_seconds)
        cpu = {k: cb[k] for k in ("value", "unit", "cores", "kind", "sample")}
    if rank == 0:
        line = {
            "metric": METRIC, "value": value, "unit": "GB/s", "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": ms_step, "higher_is_better": True, "scaling": args.scaling,
            "vs_baseline": None, "dtype": "f16", "data": "synthetic", "config": workload_config(args, world),
            "decode_tokens_per_s": 1000.0 / ms_step,
            # Rank 0's kernels per layer: the page pass and the PDL split-combine of
            # tp_decode_step (N=1) or tp_decode_step_sharded / tp_decode_attention_sharded (the
            # cross-GPU merge runs inside the split combine).
            "gpu_launches": args.steps * LAYERS * 2,
            "roofline": roof, "e2e": e2e, "cpu_baseline": cpu, "clocks": clocks.summary(),
            "device_errors": err, "library": library, **extra,
        }
        print(json.dumps(line), flush=True)
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()
    return 0


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=128)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", default="turbopolar", choices=["turbopolar", "reference"])
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-extras", action="store_true", help="skip the strong_128k / sharded / c2 records")
    ap.add_argument("--cpu-seconds", type=float, default=15.0)
    ap.add_argument("--ctx", type=int, default=CTX, help="context per GPU (weak) or in total (strong)")
    ap.add_argument("--scaling", default="weak", choices=["weak", "strong"])
    args = ap.parse_args()
    if args.warmup < 3:
        args.warmup = 3
    if args.impl == "reference":
        return run_reference(args)
    return run_gpu(args)


if __name__ == "__main__":
    sys.exit(main())
