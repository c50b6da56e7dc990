"""Failure detection on one GPU without a fault: a bounded wait that runs out.

A sequence-sharded attention call (tp_decode_attention_sharded) waits, inside its launch, for
every rank's record of each query head.  Here rank 0 is given a two-rank exchange whose other
"rank" is a second local buffer that nothing ever writes: the wait must run out after its
budget (about a second), the call must record workspace error word 3 and return, and the GPU
context must stay usable -- nothing traps, faults or hangs.  A rank that dies between steps is
the host-side case, covered by the gloo tests.
"""

import ctypes
import time

import numpy as np
import pytest
import torch

from _util import ATOL, fmt_of, kv_inputs, oracle_attention

pytestmark = pytest.mark.gpu


def test_exchange_wait_runs_out_and_reports():
    from turbopolar_b200 import TurboPolarConfig, TurboPolarKVCacheRuntime, _lib
    dev = torch.device("cuda:0")
    cfg = TurboPolarConfig(num_q_heads=8, num_kv_heads=2)
    k, v = kv_inputs(7, 2, 200, np.float16)
    rt = TurboPolarKVCacheRuntime(cfg)
    rt.append(torch.from_numpy(k).to(dev), torch.from_numpy(v).to(dev))
    q = torch.from_numpy(np.random.default_rng(8).standard_normal((1, 8, 128)).astype(np.float16)).to(dev)
    lib = _lib.lib()
    nbytes = lib.tp_exchange_bytes(2, 8)
    own = torch.zeros(nbytes, dtype=torch.uint8, device=dev)
    silent = torch.zeros(nbytes, dtype=torch.uint8, device=dev)  # the rank that never publishes
    x = _lib.Exchange(2, 0, (ctypes.c_void_p * _lib.MAX_RANKS)(own.data_ptr(), silent.data_ptr()))
    ws = torch.zeros(lib.tp_decode_attention_workspace_size(2, 8), dtype=torch.uint8, device=dev)
    out = torch.full((1, 8, 128), float("nan"), dtype=torch.float16, device=dev)
    t0 = time.perf_counter()
    _lib.check(lib.tp_decode_attention_sharded(
        ctypes.byref(rt.pool_struct()), ctypes.byref(rt.tail_struct()), rt.state(), None, q.data_ptr(), _lib.TP_F16,
        8, float(cfg.attention_scale), out.data_ptr(), ctypes.byref(x), ws.data_ptr(), ws.numel(),
        torch.cuda.current_stream().cuda_stream))
    torch.cuda.synchronize()
    elapsed = time.perf_counter() - t0
    assert int(ws[:4].view(torch.int32).item()) == 3  # a rank's records never arrived
    assert elapsed < 30.0, elapsed
    # The context is still usable: a plain call on the same cache matches the oracle.
    got = rt.attention(q).float().cpu().numpy()[0]
    want = oracle_attention(q.cpu().numpy()[0], k, v, fmt_of(cfg), False, cfg.attention_scale)
    assert np.max(np.abs(got - want)) <= ATOL
