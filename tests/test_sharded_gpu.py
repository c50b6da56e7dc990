"""Sequence-sharded decode attention on 2 GPUs (NCCL): contiguous page ranges per rank,
per-query-head partials from ``tp_decode_attention`` / ``tp_decode_step`` (``partial_out``),
an all-gather and ``tp_combine_partials`` -- eager and as a captured decode step over several
layers, against one GPU holding the whole sequence.  Skipped with fewer than 2 GPUs.
"""

import socket
from datetime import timedelta

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from _util import ATOL, fmt_of, kv_inputs, oracle_attention

pytestmark = pytest.mark.gpu


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


T0, STEPS, LAYERS = 64 * 9 + 30, 70, 2


def _worker(rank, world, port, out):
    from turbopolar_b200 import TurboPolarConfig, TurboPolarKVCacheRuntime, build, sharded
    dev = torch.device("cuda", rank)
    torch.cuda.set_device(dev)
    dist.init_process_group("nccl", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world,
                            timeout=timedelta(seconds=60), device_id=dev)
    steps_objs = []
    xs = []
    try:
        build.build()
        cfg = TurboPolarConfig(num_q_heads=8, num_kv_heads=2)
        k, v = kv_inputs(61, 2, T0 + STEPS, np.float16)
        q = np.random.default_rng(62).standard_normal((STEPS, 1, 8, 128)).astype(np.float16)
        lo, hi = sharded.page_range(T0 // 64, rank, world)
        last = rank == world - 1
        end = T0 if last else hi * 64
        T = lambda x: torch.from_numpy(np.ascontiguousarray(x)).to(dev)

        def shard_runtime():
            r = TurboPolarKVCacheRuntime(cfg, first_page=lo, max_seq_len=(end - lo * 64) + STEPS + 64,
                                         check_finite=False)
            r.append(T(k[:, :, lo * 64:end]), T(v[:, :, lo * 64:end]))
            r.set_global_length(T0)
            return r

        res = {}
        rt = shard_runtime()
        res["eager_nccl"] = sharded.sharded_attention(rt, T(q[0])).float().cpu().numpy()
        x = sharded.PeerExchange(8)
        xs.append(x)
        res["eager_peer"] = sharded.exchange_attention(rt, T(q[0]), x).float().cpu().numpy()
        res["errors"] = rt.read_device_error()
        for mode, n_steps in (("peer", STEPS), ("nccl", 10)):
            rts = [shard_runtime() for _ in range(LAYERS)]
            k_in = [torch.zeros((1, 2, 1, 128), dtype=torch.float16, device=dev) for _ in range(LAYERS)]
            v_in = [torch.zeros((1, 2, 1, 128), dtype=torch.float16, device=dev) for _ in range(LAYERS)]
            q_in = [torch.zeros((1, 8, 128), dtype=torch.float16, device=dev) for _ in range(LAYERS)]
            outs = [torch.zeros((1, 8, 128), dtype=torch.float16, device=dev) for _ in range(LAYERS)]
            step = sharded.ShardedDecodeStep(rts, k_in, v_in, q_in, outs, rank, world, exchange=mode == "peer")
            steps_objs.append(step)
            got = []
            for i in range(n_steps):
                t = T0 + i
                for layer in range(LAYERS):
                    k_in[layer].copy_(T(k[:, :, t:t + 1]))
                    v_in[layer].copy_(T(v[:, :, t:t + 1]))
                    q_in[layer].copy_(T(q[i]))
                step.replay()
                got.append(torch.stack(outs).float().cpu().numpy())
            res[mode] = np.stack(got)
            res["errors"] += sum(r.read_device_error() for r in rts)
        out[rank] = res
    finally:
        for st in steps_objs:
            st.release()
        for x in xs:
            x.close()
        dist.destroy_process_group()


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs 2 GPUs")
def test_two_gpu_sharded_attention_and_decode_steps():
    from turbopolar_b200 import TurboPolarConfig, TurboPolarKVCacheRuntime, build
    build.build()
    manager = mp.get_context("spawn").Manager()
    out = manager.dict()
    mp.start_processes(_worker, args=(2, _free_port(), out), nprocs=2, join=True, start_method="spawn")
    assert sorted(out.keys()) == [0, 1]
    cfg = TurboPolarConfig(num_q_heads=8, num_kv_heads=2)
    k, v = kv_inputs(61, 2, T0 + STEPS, np.float16)
    q = np.random.default_rng(62).standard_normal((STEPS, 1, 8, 128)).astype(np.float16)
    want0 = oracle_attention(q[0][0], k[:, :, :T0], v[:, :, :T0], fmt_of(cfg), False, cfg.attention_scale)
    for r in range(2):
        assert out[r]["errors"] == 0
        for key in ("eager_nccl", "eager_peer"):
            assert np.max(np.abs(out[r][key][0] - want0)) < ATOL, key
    # Every step of every layer, both exchanges, against one GPU holding the whole sequence.
    dev = torch.device("cuda:0")
    T = lambda x: torch.from_numpy(np.ascontiguousarray(x)).to(dev)
    full = TurboPolarKVCacheRuntime(cfg)
    full.append(T(k[:, :, :T0]), T(v[:, :, :T0]))
    for i in range(STEPS):
        t = T0 + i
        want = full.decode_step(T(k[:, :, t:t + 1]), T(v[:, :, t:t + 1]), T(q[i])).float().cpu().numpy()
        for r in range(2):
            for mode in ("peer", "nccl"):
                if i >= out[r][mode].shape[0]:
                    continue
                for layer in range(LAYERS):
                    err = np.max(np.abs(out[r][mode][i, layer] - want))
                    assert err < ATOL, (mode, r, i, layer, err)
