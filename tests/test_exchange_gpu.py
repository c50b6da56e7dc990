"""The in-launch cross-GPU merge (exchange_merge in csrc/tp_attention.cu) on one GPU.

Rank 0 of a W-rank sequence shard calls tp_decode_attention_sharded; the records of ranks
1..W-1 -- each shard's per-query-head (m, l, o) partial, as its own launch would publish it --
are written into rank 0's exchange buffer beforehand as 64-bit words tagged with the call's
epoch, so the launch finds every record present and nothing waits on another kernel.  The merged
output must equal attention over the whole sequence.  Two calls in a row use both record slots
(epoch e lives in slot e & 1); W = 2, 3 and 8 cover both thread halves of the poll (even and odd
ranks) and its two-pass form.
"""

import ctypes

import numpy as np
import pytest
import torch

from _util import ATOL, fmt_of, kv_inputs, oracle_attention

pytestmark = pytest.mark.gpu

DEV = "cuda:0"
HQ, HKV = 8, 2


@pytest.fixture(scope="module", autouse=True)
def _built():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    from turbopolar_b200 import build
    build.build()


def _epoch_offset(world, hq):
    """Byte offset of the epoch word in an exchange buffer (records [2][world][H_q][130] words)."""
    return (2 * world * hq * 130 * 8 + 255) // 256 * 256


@pytest.mark.parametrize("world", [2, 3, 8])
def test_exchange_merges_prewritten_records_over_two_calls(world):
    from turbopolar_b200 import TurboPolarConfig, TurboPolarKVCacheRuntime, _lib, sharded
    lib = _lib.lib()
    cfg = TurboPolarConfig(num_q_heads=HQ, num_kv_heads=HKV)
    n_pages, tail = 24, 13
    t = 64 * n_pages + tail
    k, v = kv_inputs(400 + world, HKV, t, np.float16)
    shards = []
    for r in range(world):
        lo, hi = sharded.page_range(n_pages, r, world)
        end = t if r == world - 1 else hi * 64
        rt = TurboPolarKVCacheRuntime(cfg, first_page=lo, check_finite=False)
        rt.append(torch.from_numpy(k[:, :, lo * 64:end].copy()).to(DEV), torch.from_numpy(v[:, :, lo * 64:end].copy()).to(DEV))
        rt.set_global_length(t)
        shards.append(rt)
    nbytes = lib.tp_exchange_bytes(world, HQ)
    assert nbytes == _epoch_offset(world, HQ) + 256
    bufs = [torch.zeros(nbytes, dtype=torch.uint8, device=DEV) for _ in range(world)]
    x = _lib.Exchange(world, 0, (ctypes.c_void_p * _lib.MAX_RANKS)(*[b.data_ptr() for b in bufs]))
    ws = torch.zeros(lib.tp_decode_attention_workspace_size(HKV, HQ), dtype=torch.uint8, device=DEV)
    words = bufs[0][:_epoch_offset(world, HQ)].view(torch.int64).view(2, world, HQ, 130)
    rng = np.random.default_rng(500 + world)
    for call in (1, 2):
        q = rng.standard_normal((1, HQ, 128)).astype(np.float16)
        qd = torch.from_numpy(q).to(DEV)
        slot = call & 1
        for r in range(1, world):  # the other ranks' records, as their launches publish them
            part = torch.empty((HQ, _lib.PARTIAL_FLOATS), dtype=torch.float32, device=DEV)
            shards[r].attention(qd, partial_out=part)
            bits = part.view(torch.int32).to(torch.int64) & 0xFFFFFFFF
            words[slot, r] = bits | (call << 32)
        out = torch.full((1, HQ, 128), float("nan"), dtype=torch.float16, device=DEV)
        _lib.check(lib.tp_decode_attention_sharded(
            ctypes.byref(shards[0].pool_struct()), ctypes.byref(shards[0].tail_struct()), shards[0].state(), None,
            qd.data_ptr(), _lib.TP_F16, HQ, float(cfg.attention_scale), out.data_ptr(), ctypes.byref(x),
            ws.data_ptr(), ws.numel(), torch.cuda.current_stream().cuda_stream))
        torch.cuda.synchronize()
        assert int(ws[:4].view(torch.int32).item()) == 0, "a record was not found"
        epoch = int(bufs[0][_epoch_offset(world, HQ):_epoch_offset(world, HQ) + 4].view(torch.int32).item())
        assert epoch == call
        # Rank 0's own record went into every rank's buffer, tagged with this epoch.
        for b in bufs:
            mine = b[:_epoch_offset(world, HQ)].view(torch.int64).view(2, world, HQ, 130)[slot, 0]
            assert bool(((mine >> 32) == call).all())
        want = oracle_attention(q[0], k, v, fmt_of(cfg), False, cfg.attention_scale)
        err = float(np.max(np.abs(out.float().cpu().numpy()[0] - want)))
        assert err < ATOL, (call, err)
