"""tp_decode_attention_noalloc: decode attention with no caller-provided scratch.

Callers such as a plugin inside a runtime that owns every device allocation, or code running
while a stream is being captured (where cudaMalloc is not allowed), cannot allocate the
workspace tp_decode_attention needs; this entry point uses a fixed scratch array held in the
library's device memory instead.  These tests call it through the C ABI and check it against
the workspace-taking entry point on the same inputs, for two calls in a row (the array keeps
the previous call's contents, which must not leak into the next result), read the array's
error word back through tp_noalloc_error, and check one result against the CPU oracle.
"""

import ctypes

import numpy as np
import pytest
import torch

from _util import ATOL, fmt_of, kv_inputs, oracle_attention

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def lib():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    from turbopolar_b200 import _lib, build
    build.build()
    return _lib.lib()


def _noalloc(lib, rt, q, out):
    from turbopolar_b200 import _lib
    return lib.tp_decode_attention_noalloc(
        ctypes.byref(rt.pool_struct()), ctypes.byref(rt.tail_struct()), rt.state(), None, q.data_ptr(),
        _lib.TP_F16, q.shape[0] * q.shape[1], float(rt.config.attention_scale), out.data_ptr(), None,
        torch.cuda.current_stream().cuda_stream)


def _error_word(lib):
    from turbopolar_b200 import _lib
    word = ctypes.c_int32(-1)
    _lib.check(lib.tp_noalloc_error(ctypes.byref(word), torch.cuda.current_stream().cuda_stream))
    return word.value


def test_noalloc_matches_workspace_entry_point_twice(lib):
    """Both entry points launch the same kernels on the same inputs, so their outputs must be
    identical bit for bit; the first call is also checked against the CPU oracle directly."""
    from turbopolar_b200 import TurboPolarConfig, TurboPolarKVCacheRuntime, _lib
    dev = torch.device("cuda:0")
    cfg = TurboPolarConfig(num_q_heads=32, num_kv_heads=8)
    k, v = kv_inputs(91, 8, 3000, np.float16)      # 46 pages + a 56-token dense tail
    rt = TurboPolarKVCacheRuntime(cfg)
    rt.append(torch.from_numpy(k).to(dev), torch.from_numpy(v).to(dev))
    rng = np.random.default_rng(92)
    for call in range(2):
        q = torch.from_numpy(rng.standard_normal((1, 32, 128)).astype(np.float16)).to(dev)
        want = rt.attention(q)                       # tp_decode_attention with its own workspace
        got = torch.full_like(want, float("nan"))
        _lib.check(_noalloc(lib, rt, q, got))
        torch.cuda.synchronize()
        assert torch.equal(got, want), (call, (got.float() - want.float()).abs().max().item())
        assert _error_word(lib) == 0                 # no stage wait ran out
        if call == 0:
            ref = oracle_attention(q.cpu().numpy()[0], k, v, fmt_of(cfg), False, cfg.attention_scale)
            err = float(np.max(np.abs(got.float().cpu().numpy()[0] - ref)))
            assert err <= ATOL, err


def test_noalloc_rejects_layouts_beyond_its_scratch(lib):
    from turbopolar_b200 import _lib
    f = _lib.Format(4, 4, 64, 0)
    pool = _lib.PagePool(None, None, 4096, 0, f)
    tail = _lib.Tail(None, None, 0)
    st = lib.tp_decode_attention_noalloc(ctypes.byref(pool), ctypes.byref(tail), _lib.State(0, 1, 1, 0), None,
                                         ctypes.c_void_p(16), 0, 4096, 0.1, ctypes.c_void_p(16), None, None)
    with pytest.raises(ValueError, match="maximum"):
        _lib.check(st)
