"""Sequence-sharded decode attention: the host protocol on CPU with gloo (world size 2).

Each rank holds a contiguous page range of every KV head (``sharded.page_range``; the last
rank also holds the dense tail), computes per-query-head partials (m, l, o), all-gathers them
and merges with the log-sum-exp rule that ``tp_combine_partials`` implements; the merged
output must equal single-device attention over the whole sequence.  The partials come from the
oracle here (no GPU); the CUDA path runs the same protocol in ``test_sharded_gpu.py``.  The
rank-failure tests at the end run ``StepMonitor`` in three spawned processes over a TCP store,
with the failures injected on the host.
"""

import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from _util import kv_inputs, oracle_cache

SCALE = 1.0 / np.sqrt(128.0)


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _inputs():
    k, v = kv_inputs(51, 2, 64 * 7 + 20, np.float16)
    q = np.random.default_rng(52).standard_normal((8, 128)).astype(np.float16)
    return k, v, q


def _decoded(k, v):
    """The whole sequence as the kernels see it: decoded pages, then the dense tail."""
    from oracle import attention as oatt
    fmt = dict(l1_bits=4, deep_bits=4, split_dim=64)
    pages, tk, tv = oracle_cache(k, v, fmt, False)
    pk, pv = oatt.decode_pages(pages, fmt)
    return (np.concatenate([pk, tk], axis=1).astype(np.float64), np.concatenate([pv, tv], axis=1).astype(np.float64))


def _worker(rank, world, port, out):
    from oracle import attention as oatt
    from turbopolar_b200.sharded import page_range
    dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world)
    try:
        k, v, q = _inputs()
        kk, vv = _decoded(k, v)
        n_pages = k.shape[2] // 64
        lo, hi = page_range(n_pages, rank, world)
        end = kk.shape[1] if rank == world - 1 else hi * 64  # the last rank also holds the tail
        part = oatt.partial(q.astype(np.float64), kk[:, lo * 64:end], vv[:, lo * 64:end], SCALE)
        gathered = [torch.zeros(part.shape, dtype=torch.float64) for _ in range(world)]
        dist.all_gather(gathered, torch.from_numpy(part))
        out[rank] = oatt.combine(np.stack([g.numpy() for g in gathered]))
    finally:
        dist.destroy_process_group()


def test_page_range_partitions_pages():
    from turbopolar_b200.sharded import page_range
    for n in (0, 1, 7, 64, 513, 2048):
        for world in (1, 2, 3, 4, 8):
            ranges = [page_range(n, r, world) for r in range(world)]
            assert ranges[0][0] == 0 and ranges[-1][1] == n
            assert all(a[1] == b[0] for a, b in zip(ranges, ranges[1:]))
            assert max(h - l for l, h in ranges) - min(h - l for l, h in ranges) <= 1


def test_combine_of_partials_equals_whole_attention():
    """Single process: the partials of any split of the tokens merge to the full result."""
    from oracle import attention as oatt
    k, v, q = _inputs()
    kk, vv = _decoded(k, v)
    want = oatt.attention(q.astype(np.float64), kk, vv, kk.shape[1], SCALE)
    for cuts in ([0, 100, 200, kk.shape[1]], [0, 0, 64, kk.shape[1]], [0, kk.shape[1]]):
        parts = [oatt.partial(q.astype(np.float64), kk[:, a:b], vv[:, a:b], SCALE) for a, b in zip(cuts, cuts[1:])]
        np.testing.assert_allclose(oatt.combine(np.stack(parts)), want, rtol=0, atol=1e-12)


def test_gloo_two_ranks_match_single_device():
    k, v, q = _inputs()
    kk, vv = _decoded(k, v)
    from oracle import attention as oatt
    want = oatt.attention(q.astype(np.float64), kk, vv, kk.shape[1], SCALE)
    manager = mp.get_context("spawn").Manager()
    out = manager.dict()
    mp.start_processes(_worker, args=(2, _free_port(), out), nprocs=2, join=True, start_method="spawn")
    assert sorted(out.keys()) == [0, 1]
    for r in range(2):
        np.testing.assert_allclose(out[r], want, rtol=0, atol=1e-12)


# ---------------------------------------------------------------------------- rank failures
# StepMonitor (sharded.py) is the host-side check that every rank has reached a step before any
# rank launches it.  Failures are injected on the host: a rank raises and leaves, exits, or skips
# a step; the surviving ranks must raise RankFailure naming it, within the monitor's timeout,
# before launching that step.
STEPS = 5
FAIL_AT = 3


def _monitor_worker(rank, world, port, mode, out):
    import os
    import time
    from datetime import timedelta
    from turbopolar_b200.sharded import RankFailure, StepMonitor
    store = dist.TCPStore("127.0.0.1", port, world, rank == 0, timeout=timedelta(seconds=60))
    mon = StepMonitor(rank, world, store=store, prefix="steps", timeout_s=2.0)
    launched = []
    t0 = time.monotonic()
    try:
        for k in range(1, STEPS + 1):
            if rank == 1 and k == FAIL_AT and mode == "raise":
                try:
                    raise RuntimeError("injected failure")
                except RuntimeError:
                    out[rank] = ("left", launched, "")
                    return
            if rank == 1 and k == FAIL_AT and mode == "exit":
                out[rank] = ("exited", launched, "")
                os._exit(0)
            if rank == 1 and k == FAIL_AT and mode == "skip":
                continue
            mon.step(k)
            launched.append(k)  # stands for the step's launches
            time.sleep(0.01)
        out[rank] = ("ok", launched, "")
    except RankFailure as e:
        out[rank] = ("failure", launched, str(e), time.monotonic() - t0)
    finally:
        if rank == 0:
            time.sleep(3.0)  # rank 0 serves the store; let the others finish their reads


def _run_monitor(mode, world=3):
    manager = mp.get_context("spawn").Manager()
    out = manager.dict()
    mp.start_processes(_monitor_worker, args=(world, _free_port(), mode, out), nprocs=world, join=True,
                       start_method="spawn")
    return dict(out)


def test_step_monitor_all_ranks_healthy():
    out = _run_monitor("none")
    for r in range(3):
        assert out[r][0] == "ok" and out[r][1] == list(range(1, STEPS + 1)), out[r]


@pytest.mark.parametrize("mode", ["raise", "exit"])
def test_step_monitor_detects_a_rank_that_left(mode):
    out = _run_monitor(mode)
    for r in (0, 2):
        status, launched, msg, elapsed = out[r]
        assert status == "failure", out[r]
        assert launched == list(range(1, FAIL_AT)), out[r]  # nothing launched for the missing step
        assert "rank 1 did not reach step 3" in msg
        assert elapsed < 20.0


def test_step_monitor_detects_a_skipped_step():
    """A rank that skips a step is found at that step; the skipping rank, one step ahead, finds
    that nobody else reached its next one."""
    out = _run_monitor("skip")
    for r in (0, 2):
        status, launched, msg, _ = out[r]
        assert status == "failure", out[r]
        assert launched == list(range(1, FAIL_AT)) and "rank 1 did not reach step 3" in msg, out[r]
    status, launched, msg, _ = out[1]
    assert status == "failure" and launched == list(range(1, FAIL_AT)) and "did not reach step 4" in msg, out[1]
