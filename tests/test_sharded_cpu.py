"""Sequence-sharded decode attention: the host protocol on CPU with gloo (world size 2).

Each rank holds a contiguous page range of every KV head (``sharded.page_range``; the last
rank also holds the dense tail), computes per-query-head partials (m, l, o), all-gathers them
and merges with the log-sum-exp rule that ``tp_combine_partials`` implements; the merged
output must equal single-device attention over the whole sequence.  The partials come from the
oracle here (no GPU); the CUDA path runs the same protocol in ``test_sharded_gpu.py``.
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
