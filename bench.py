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
  cpu_baseline -- the NumPy oracle (the reference's CPU-fallback math) on a bounded sample

Multi-GPU (torchrun, N>1): one sequence of N x 32K tokens per layer, split into contiguous
page ranges, one 32K range per rank (the last rank also holds the tail and the new tokens);
every rank's attention launch publishes its per-query-head partial (max, sum, output) into
every rank's buffer over NVLink and merges them (log-sum-exp) in the same launch.  Per-GPU work
is fixed, so scaling is "weak" (``--scaling strong --ctx C`` splits one C-token context).

``--impl reference`` times the oracle port of the reference's CPU fallback instead.
"""

from __future__ import annotations

import argparse
import json
import math
import os
import statistics
import subprocess
import sys
import tempfile
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

CTX = 32768
LAYERS = 32
HQ, HKV, D = 32, 8, 128
PAGE = 64
PAGE_BYTES_DEFAULT = 64 * 296  # per page per KV head: radii 8192 + codes 2048 + V 8192 + scales 512


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
def _cpu_head_attention(args):
    """Oracle attention for the query heads of one KV head over its compressed pages."""
    from oracle import attention as oatt
    pages, fmt, q, scale = args
    k, v = oatt.decode_pages(pages, fmt)
    return oatt.attention(q, k, v, k.shape[1], scale)


def cpu_baseline(seconds_target: float = 15.0, ctx: int = CTX):
    """Time the oracle (the reference's CPU-fallback math: full decode, dequantize, softmax,
    weighted sum) on one layer at ``ctx`` tokens, KV heads spread over a spawn process pool."""
    import multiprocessing as mp
    from oracle import polar, vquant
    rng = np.random.default_rng(0)
    c = np.random.default_rng(1).uniform(0.5, 4.0, size=128).astype(np.float32)
    n = ctx // PAGE
    fmt = dict(l1_bits=4, deep_bits=4, split_dim=64)
    work = []
    for h in range(HKV):
        k = (rng.standard_normal((1, n, PAGE, D)).astype(np.float32) * c).astype(np.float16)
        v = rng.standard_normal((1, n, PAGE, D)).astype(np.float16)
        enc = polar.encode_block(k)
        codes, scales = vquant.quantize(v)
        pages = dict(radii=enc["radii"], angle_codes_l1=enc["angle_codes_l1"], angle_codes_deep=enc["angle_codes_deep"],
                     radii_scales=None, v_codes=codes, v_scales=scales)
        q = rng.standard_normal((HQ // HKV, D)).astype(np.float16).astype(np.float64)
        work.append((pages, fmt, q, 1 / math.sqrt(D)))
    cores = min(os.cpu_count() or 1, HKV)
    ctxm = mp.get_context("spawn")
    with ctxm.Pool(cores) as pool:
        pool.map(_cpu_head_attention, work[:cores])  # warm the workers
        calls, t0 = 0, time.perf_counter()
        while True:
            pool.map(_cpu_head_attention, work)
            calls += 1
            if time.perf_counter() - t0 >= seconds_target:
                break
        dt = (time.perf_counter() - t0) / calls
    byts = attention_bytes(n, 0)
    return {"value": byts / dt / 1e9, "unit": "GB/s", "cores": cores, "kind": "port",
            "sample": f"{calls} single-layer attention calls at {ctx} tokens, {HQ}q/{HKV}kv "
                      f"({dt * 1e3:.1f} ms/call; {LAYERS}-layer step {dt * LAYERS:.2f} s)",
            "ms_per_layer_call": dt * 1e3}


def _total_ctx(args, world: int) -> int:
    return args.ctx * world if args.scaling == "weak" else args.ctx


def run_reference(args):
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return 0
    ctx = _total_ctx(args, int(os.environ.get("WORLD_SIZE", "1")))
    cb = cpu_baseline(seconds_target=max(3.0, min(20.0, 2.0 * (args.steps + args.warmup))), ctx=ctx)
    step_s = cb["ms_per_layer_call"] * 1e-3 * LAYERS
    line = {
        "metric": "decode-attention HBM GB/s (% of B200 peak) and decode tokens/s at 32K ctx",
        "value": cb["value"], "unit": "GB/s", "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": step_s * 1e3, "higher_is_better": True, "scaling": args.scaling, "vs_baseline": None,
        "dtype": "f16", "data": "synthetic", "impl": "reference",
        "config": {"workload": "llama3-8b-attention-32layers-32k-decode", "ctx": ctx, "layers": LAYERS,
                   "num_q_heads": HQ, "num_kv_heads": HKV, "head_dim": D, "batch": 1},
        "decode_tokens_per_s": 1.0 / step_s,
        "cpu_baseline": {k: cb[k] for k in ("value", "unit", "cores", "kind", "sample")},
        "e2e": {"value": cb["value"], "unit": "GB/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)
    return 0


# ----------------------------------------------------------------------------- GPU arm
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

    from turbopolar_b200 import TurboPolarConfig, TurboPolarKVCacheRuntime, build, graph, sharded
    build.build()
    cfg = TurboPolarConfig(num_q_heads=HQ, num_kv_heads=HKV)
    total_steps = args.steps + args.warmup + 2
    CTX = _total_ctx(args, world)
    n_pages_total = CTX // PAGE
    lo, hi = sharded.page_range(n_pages_total, rank, world)
    last = rank == world - 1
    cap_tokens = (hi - lo) * PAGE + (total_steps + PAGE if last else 0)
    chan = torch.from_numpy(np.random.default_rng(1).uniform(0.5, 4.0, size=D).astype(np.float32)).to(dev)
    gen = torch.Generator(device=dev)
    layers = []
    for layer in range(LAYERS):
        rt = TurboPolarKVCacheRuntime(cfg, max_seq_len=cap_tokens, check_finite=False, first_page=lo)
        # Each rank draws its own slice of the layer's sequence.
        gen.manual_seed(1000 + 64 * layer + rank)
        k = (torch.randn((1, HKV, (hi - lo) * PAGE, D), generator=gen, device=dev) * chan).half()
        v = torch.randn((1, HKV, (hi - lo) * PAGE, D), generator=gen, device=dev).half()
        rt.append(k, v)
        if world > 1:
            rt.set_global_length(CTX)
        del k, v
        layers.append(rt)
    torch.cuda.synchronize()

    # Per-step inputs (new K, V and q of every layer) are views of one device buffer and the
    # outputs of another, so the end-to-end leg moves them with one copy each way per step.
    gen.manual_seed(7)
    per_layer_in = 2 * HKV * D + HQ * D
    d_in = torch.randn((LAYERS, per_layer_in), generator=gen, device=dev).half()
    d_out = torch.empty((LAYERS, 1, HQ, D), dtype=torch.float16, device=dev)
    k_in = [d_in[i, :HKV * D].view(1, HKV, 1, D) for i in range(LAYERS)]
    v_in = [d_in[i, HKV * D:2 * HKV * D].view(1, HKV, 1, D) for i in range(LAYERS)]
    q_in = [d_in[i, 2 * HKV * D:].view(1, HQ, D) for i in range(LAYERS)]
    out = [d_out[i] for i in range(LAYERS)]

    if world == 1:
        step = graph.DecodeStep(None, layers=[(layers[i], k_in[i], v_in[i], q_in[i], out[i]) for i in range(LAYERS)])
    else:
        step = sharded.ShardedDecodeStep(layers, k_in, v_in, q_in, out, rank, world)

    def barrier():
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize()

    for _ in range(args.warmup):
        step.replay()
    barrier()
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    pages_before = [(rt.n_pages, rt.tail_len) for rt in layers]
    with ClockSampler(local) as clocks:
        barrier()
        start.record()
        for _ in range(args.steps):
            step.replay()
        end.record()
        barrier()
    ms = start.elapsed_time(end)
    if world > 1:
        t = torch.tensor([ms], device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms = float(t.item())
    ms_step = ms / args.steps
    # Algorithmic bytes over the timed steps: every step reads the whole context once per layer
    # (split over ranks), plus q and out per rank.
    step_bytes = 0
    for i in range(args.steps):
        ctx_tokens = CTX + args.warmup + i + 1
        full, tail = divmod(ctx_tokens, PAGE)
        step_bytes += LAYERS * (full * HKV * PAGE_BYTES_DEFAULT + tail * HKV * D * 4 + world * HQ * D * 4)
    value = step_bytes / args.steps / (ms_step * 1e-3) / 1e9

    # ---- roofline: attention kernel alone, per launch, on its own stream (graph of 32 launches).
    def graph_us(launch_all, reps=20):
        """Device time per launch of a captured graph of LAYERS attention calls."""
        g = torch.cuda.CUDAGraph()
        torch.cuda.synchronize()
        with torch.cuda.graph(g):
            launch_all()
        for _ in range(3):
            g.replay()
        torch.cuda.synchronize()
        s2, e2 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        s2.record()
        for _ in range(reps):
            g.replay()
        e2.record()
        torch.cuda.synchronize()
        del g
        return s2.elapsed_time(e2) / (reps * LAYERS) * 1e3

    # One call per layer, each on its own cache with its own query and output (consecutive
    # calls are independent, so a page pass may stream while the previous call finishes).
    kern_us = graph_us(lambda: [graph.launch_attention(layers[i], q_in[i], out[i], cfg.attention_scale,
                                                       partial_out=step.partial_buffer(i) if world > 1 else None)
                                for i in range(LAYERS)])
    # The same calls with each layer's query read from the previous layer's output, as in a
    # model: every call then waits for the previous one to complete before its page pass
    # streams, so this is the latency of one dependent call.
    dep_us = None
    if world == 1:
        dep_out = torch.empty((LAYERS, 1, HQ, D), dtype=torch.float16, device=dev)
        dep_us = graph_us(lambda: [graph.launch_attention(layers[i], q_in[0] if i == 0 else dep_out[i - 1],
                                                          dep_out[i], cfg.attention_scale) for i in range(LAYERS)])
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
    barrier()
    s3, e3 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    t_wall = time.perf_counter()
    s3.record()
    for _ in range(e_steps):
        d_in.copy_(h_in, non_blocking=True)
        step.replay()
        h_out.copy_(d_out, non_blocking=True)
    e3.record()
    barrier()
    e_ms = s3.elapsed_time(e3)
    if world > 1:
        t = torch.tensor([e_ms], device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        e_ms = float(t.item())
    t_wall = time.perf_counter() - t_wall
    e_step_bytes = step_bytes / args.steps
    e2e = {"value": e_step_bytes / (e_ms / e_steps * 1e-3) / 1e9, "unit": "GB/s",
           "h2d_bytes_per_step": h_in.numel() * h_in.element_size(),
           "d2h_bytes_per_step": h_out.numel() * h_out.element_size(), "steps": e_steps,
           "wall_ms_per_step": t_wall * 1e3 / e_steps}

    err = sum(rt.read_device_error() for rt in layers)
    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        cb = cpu_baseline(seconds_target=args.cpu_seconds)
        cpu = {k: cb[k] for k in ("value", "unit", "cores", "kind", "sample")}
    if rank == 0:
        line = {
            "metric": "decode-attention HBM GB/s (% of B200 peak) and decode tokens/s at 32K ctx",
            "value": value, "unit": "GB/s", "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": ms_step, "higher_is_better": True, "scaling": args.scaling, "vs_baseline": None,
            "dtype": "f16", "data": "synthetic",
            "config": {"workload": "llama3-8b-attention-32layers-32k-decode", "ctx": CTX,
                       "ctx_per_gpu": CTX // world, "layers": LAYERS,
                       "num_q_heads": HQ, "num_kv_heads": HKV, "head_dim": D, "batch": 1,
                       "format": "fp16 radii, 4-bit angles (split 64), int8 V group 32",
                       "parallelism": f"sequence-shard x{world}" if world > 1 else "single GPU",
                       "l2": "inputs larger than L2 (2.48 GB of pages per step vs 126 MB L2)"},
            "decode_tokens_per_s": 1000.0 / ms_step,
            # Rank 0's kernels per layer: the page pass and the PDL split-combine of
            # tp_decode_step (N=1) or tp_decode_attention_sharded (the cross-GPU merge runs
            # inside the split combine).
            "gpu_launches": args.steps * LAYERS * 2,
            "roofline": roof, "e2e": e2e, "cpu_baseline": cpu, "clocks": clocks.summary(),
            "device_errors": err,
        }
        print(json.dumps(line), flush=True)
    step.release() if hasattr(step, "release") else None
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
