"""Canary guard bytes (turbopolar_b200.guard) on CPU tensors: a buffer allocated with guards on
reads as zeros, writes inside it pass the check, and a byte changed just before or just past it
fails the check with the buffer's name -- including for a page pool dropped by growth."""

import pytest
import torch


@pytest.fixture()
def guard():
    from turbopolar_b200 import guard
    guard.enable(512)
    yield guard
    guard.disable()


def test_guard_detects_writes_outside_a_buffer(guard):
    t = guard.zeros((3, 5), torch.float16, "cpu", "probe")
    assert t.shape == (3, 5) and t.dtype == torch.float16 and not bool(t.any())
    t.fill_(1.0)  # the whole payload
    assert guard.check() == 1
    base = guard._live[0][0]
    base[512 + 30] = 0  # first byte past the 30-byte payload
    with pytest.raises(AssertionError, match="probe changed: first at 1 bytes past the end"):
        guard.check()
    base[512 + 30] = guard.PATTERN
    base[511] = 0  # last byte before it
    with pytest.raises(AssertionError, match="1 bytes before"):
        guard.check()


def test_guarded_page_pool_and_growth(guard):
    from turbopolar_b200.pages import PagePool
    fmt = dict(l1_bits=4, deep_bits=8, split_dim=0, int8_radii=1)
    pool = PagePool(2, 4, fmt, "cpu")
    assert pool.pages.shape == (2, 4, 2 * pool.unit_bytes) and pool.radii_scales.shape == (2, 4)
    pool.pages.fill_(3)
    grown = pool.grown(8, 4)  # checks the old pool's guards before it is dropped
    assert bool((grown.pages[:, :4] == 3).all()) and not bool(grown.pages[:, 4:].any())
    # A write one byte past the radius scales of the grown pool.
    rec = [r for r in guard._live if r[1]() is grown.radii_scales][0]
    rec[0][rec[2] + rec[3]] = 0
    with pytest.raises(AssertionError, match="radius scales changed"):
        guard.check()


def test_guards_off_by_default():
    from turbopolar_b200 import guard
    assert not guard.enabled()
    t = guard.zeros((4,), torch.int32, "cpu", "plain")
    assert t._base is None and not guard._live
