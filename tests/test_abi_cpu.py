"""CPU-only checks: the C-ABI library loads and exports every declared symbol, the
configuration contract, and host-side validation (no kernel launches)."""

import ctypes
import os
import re

import pytest
import torch

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _declared_symbols():
    src = open(os.path.join(ROOT, "include", "turbopolar.h")).read()
    src = re.sub(r"/\*.*?\*/", "", src, flags=re.S)
    return sorted(set(re.findall(r"\b(tp_[a-z_0-9]+)\s*\(", src)))


@pytest.fixture(scope="module")
def lib():
    from turbopolar_b200 import _lib, build
    build.build()
    return _lib.lib()


def test_library_exports_every_declared_symbol(lib):
    declared = _declared_symbols()
    assert "tp_decode_attention" in declared and "tp_append" in declared
    handle = ctypes.CDLL(os.path.join(ROOT, "turbopolar_b200", "libturbopolar.so"))
    for name in declared:
        assert hasattr(handle, name), name
    from turbopolar_b200 import _lib
    assert sorted(_lib.EXPORTED) == declared


def test_version_and_row_bytes(lib):
    from turbopolar_b200 import _lib
    assert lib.tp_version() == 3
    cases = {  # (l1_bits, deep_bits, split_dim) -> (l1_row, deep_row); test_turbo_polar_offline.py:26-34
        (4, 4, 64): (16, 16), (4, 8, 0): (0, 64), (8, 2, 32): (16, 12), (4, 8, 128): (32, 0), (4, 2, 2): (1, 16),
    }
    for (l1, deep, split), want in cases.items():
        f = _lib.Format(l1, deep, split, 0)
        a, b = ctypes.c_int32(), ctypes.c_int32()
        assert lib.tp_row_bytes(ctypes.byref(f), ctypes.byref(a), ctypes.byref(b)) == 0
        assert (a.value, b.value) == want
    # Unit (half page) of the kernel layout: 32 x (radii row + 128 value codes + code row + 8
    # scale bytes), i.e. the reference's bytes per token x 32 without the radius scale.
    units = {(4, 4, 64, 0): 9472, (4, 8, 0, 1): 8448, (8, 2, 32, 0): 9344, (4, 2, 2, 0): 32 * (128 + 128 + 17 + 8)}
    for (l1, deep, split, i8), want in units.items():
        u = ctypes.c_int32()
        assert lib.tp_unit_bytes(ctypes.byref(_lib.Format(l1, deep, split, i8)), ctypes.byref(u)) == 0
        assert u.value == want and u.value % 16 == 0
    f = _lib.Format(3, 4, 64, 0)
    assert lib.tp_row_bytes(ctypes.byref(f), None, None) == _lib.TP_ERR_UNSUPPORTED
    assert "k_angle_bits_level1" in lib.tp_last_error().decode()


def test_error_statuses_map_to_reference_exceptions(lib):
    from turbopolar_b200 import _lib
    f = _lib.Format(4, 4, 64, 0)
    pool = _lib.PagePool(None, None, 4, 0, f)
    tail = _lib.Tail(None, None, 0)
    # Empty cache -> ValueError, before any launch.
    st = lib.tp_decode_attention(ctypes.byref(pool), ctypes.byref(tail), _lib.State(0, 0, 0, 0), None,
                                 ctypes.c_void_p(16), 0, 8, 0.1, ctypes.c_void_p(16), None, None, 0, None)
    with pytest.raises(ValueError, match="empty cache"):
        _lib.check(st)
    st = lib.tp_decode_attention(ctypes.byref(pool), ctypes.byref(tail), _lib.State(0, 1, 1, 0), None,
                                 ctypes.c_void_p(16), 0, 7, 0.1, ctypes.c_void_p(16), None, None, 0, None)
    with pytest.raises(ValueError, match="divisible"):
        _lib.check(st)
    f2 = _lib.Format(4, 3, 64, 0)
    pool2 = _lib.PagePool(None, None, 4, 0, f2)
    with pytest.raises(NotImplementedError):
        _lib.check(lib.tp_decode_pages(ctypes.byref(pool2), 0, 0, None, None, None))


def test_dense_v_rejects_bad_arguments_before_any_launch(lib):
    """tp_decode_attention_dense_v's argument checks (pages only, the token range, the value
    array's alignment and strides), each a ValueError before any CUDA call."""
    from turbopolar_b200 import _lib
    f = _lib.Format(4, 4, 64, 0)
    pool = _lib.PagePool(ctypes.c_void_p(1 << 20), None, 2, 4, f)
    v = ctypes.c_void_p(1 << 24)

    def call(state, v=v, stride=4 * 64 * 128, tokens=4 * 64):
        return lib.tp_decode_attention_dense_v(ctypes.byref(pool), state, v, stride, tokens, ctypes.c_void_p(16), 0,
                                               4, 0.1, ctypes.c_void_p(16), None, None, 0, None)

    cases = [
        ((2, 5, 133, 0), {}, "pages only"),
        ((2, 0, 100, 1), {}, "pages only"),
        ((0, 0, 1, 0), {}, "n_pages must be in"),
        ((5, 0, 1, 0), {}, "n_pages must be in"),
        ((2, 0, 129, 0), {}, "seq_len must be in"),
        ((2, 0, 0, 0), {}, "seq_len must be in"),
        ((2, 0, 100, 0), dict(v=ctypes.c_void_p((1 << 24) + 8)), "16-byte aligned"),
        ((2, 0, 100, 0), dict(tokens=99), "v_tokens"),
        ((2, 0, 100, 0), dict(stride=4 * 64 * 128 + 4), "v_head_stride"),
        ((2, 0, 100, 0), dict(stride=64 * 128), "v_head_stride"),
    ]
    for state, kw, pattern in cases:
        with pytest.raises(ValueError, match=pattern):  # the message is read right after the call
            _lib.check(call(_lib.State(*state), **kw))


def test_workspace_size(lib):
    n = lib.tp_decode_attention_workspace_size(8, 32)
    assert n > 0 and n % 256 == 0
    assert lib.tp_decode_attention_workspace_size(8, 31) == 0


# ---------------------------------------------------------------- configuration contract
# tests/unit/test_supported_config_contract.py and tests/test_turbo_polar_cache_runtime.py:80-88

def test_supported_config_constructs():
    from turbopolar_b200 import TurboPolarConfig
    cfg = TurboPolarConfig(head_dim=128, block_size=64, num_q_heads=8, num_kv_heads=4, use_qjl=False,
                           storage_mode="kv_quant")
    assert cfg.head_dim == 128 and cfg.block_size == 64 and not cfg.use_qjl
    assert cfg.attention_scale == pytest.approx(1 / 128 ** 0.5)
    assert TurboPolarConfig(attention_scale=0.5).attention_scale == 0.5


@pytest.mark.parametrize("kwargs,pattern", [
    (dict(head_dim=64), "head_dim == 128"),
    (dict(head_dim=256), "head_dim == 128"),
    (dict(block_size=32), "block_size == 64"),
    (dict(use_qjl=True), "use_qjl=False"),
    (dict(storage_mode="dense_v_debug"), "storage_mode='kv_quant'"),
    (dict(v_bits=4), "v_bits must be 8"),
    (dict(num_q_heads=7), "num_q_heads must be divisible"),
    (dict(split_dim=3), "split_dim must be even"),
    (dict(storage_mode="bogus"), "unknown storage_mode"),
    (dict(qjl_proj_dim=12), "divisible by 8"),
])
def test_unsupported_configs_raise(kwargs, pattern):
    from turbopolar_b200 import TurboPolarConfig
    base = dict(head_dim=128, block_size=64, num_q_heads=4, num_kv_heads=4)
    base.update(kwargs)
    with pytest.raises(ValueError, match=re_escape(pattern)):
        TurboPolarConfig(**base)


def re_escape(s):
    return re.escape(s)


def test_append_rejects_without_gpu_work():
    from turbopolar_b200 import TurboPolarConfig, TurboPolarKVCacheRuntime
    rt = TurboPolarKVCacheRuntime(TurboPolarConfig(num_q_heads=4, num_kv_heads=4))
    with pytest.raises(TypeError):
        rt.append([1], [2])
    with pytest.raises(ValueError, match="4-D"):
        rt.append(torch.zeros(1, 4, 128), torch.zeros(1, 4, 128))
    with pytest.raises(ValueError, match="must match"):
        rt.append(torch.zeros(1, 4, 1, 128), torch.zeros(1, 4, 2, 128))
    with pytest.raises(ValueError, match="at least one token"):
        rt.append(torch.zeros(1, 4, 0, 128), torch.zeros(1, 4, 0, 128))
    with pytest.raises(ValueError, match="only float16 and float32"):
        rt.append(torch.zeros(1, 4, 1, 128, dtype=torch.float64), torch.zeros(1, 4, 1, 128, dtype=torch.float64))
    with pytest.raises(ValueError, match="CUDA"):
        rt.append(torch.zeros(1, 4, 1, 128), torch.zeros(1, 4, 1, 128))
    assert rt.get_io_telemetry() == {}
    with pytest.raises(RuntimeError, match="no blocks"):
        rt.attention(torch.zeros(1, 4, 128))


def test_build_is_keyed_by_a_hash_of_sources_and_flags(lib):
    """A second build() with the same sources and flags reuses the library; other flags change
    the hash, so a library built with them is not taken for the product build."""
    from turbopolar_b200 import build
    build.build()
    assert build.last_build["compiled"] is False
    assert build.last_build["source_sha16"] == build.source_hash()
    with open(build.STAMP) as f:
        assert f.read().strip() == build.source_hash()
    assert build.source_hash(["-DTP_QK_CUDA_CORES=1"]) != build.source_hash()
