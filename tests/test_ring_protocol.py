"""Model check of the page pass's copy ring (decode_attention_kernel in csrc/tp_attention.cu).

The kernel's consumer warp w takes CTA units w, w + C, ... and owns ring stages [w*S, w*S + S);
issuing lane p serves the consumers w = p (mod NP).  Each stage has a "full" mbarrier (one
arrival with the expected bytes, then the bulk copy's bytes) and an "empty" one (the consumer's
release).  mbarrier parity waits only tell phase parity apart, so a wait that runs two phases
ahead of its barrier passes on a stale phase.  This test drives the same indexing under random
schedules with that parity rule and checks that no barrier takes a second arrival in a phase and
every consumer reads the unit it expects -- and that the shared-ring assignment (stage k % R,
producer k % NP) the kernel does not use fails the same check.
"""

import random

import pytest


class _Bar:
    def __init__(self):
        self.ph, self.arrived, self.tx = 0, False, False

    def done(self, parity):  # try_wait.parity: the phase of that parity has completed
        return (self.ph & 1) != parity

    def arrive(self):
        assert not self.arrived, "second arrival in one phase"
        self.arrived = True
        self.settle()

    def settle(self):
        if self.arrived and not self.tx:
            self.ph, self.arrived = self.ph + 1, False


def _simulate(n, C, S, NP, seed, owned=True, R=None):
    rng = random.Random(seed)
    R = R or C * S
    full = [_Bar() for _ in range(R)]
    empty = [_Bar() for _ in range(R)]
    data, inflight = [None] * R, []

    def stage_of(k):
        if owned:
            w, j = k % C, k // C
            return w * S + j % S, j // S
        return k % R, k // R

    def issue(k):
        slot, wrap = stage_of(k)
        if wrap > 0:
            while not empty[slot].done((wrap - 1) & 1):
                yield
        assert not full[slot].arrived, "issue into a stage whose copy is pending"
        full[slot].tx = True
        full[slot].arrive()
        inflight.append((slot, k))
        yield

    def producer(p):
        if owned:
            for j in range((n + C - 1) // C):
                for w in range(p, C, NP):
                    if w + C * j < n:
                        yield from issue(w + C * j)
        else:
            for k in range(p, n, NP):
                yield from issue(k)

    def consumer(w):
        for k in range(w, n, C):
            slot, wrap = stage_of(k)
            while not full[slot].done(wrap & 1):
                yield
            assert data[slot] == k, f"read unit {data[slot]} expecting {k}"
            yield
            empty[slot].arrive()

    alive = [producer(p) for p in range(NP)] + [consumer(w) for w in range(C)]
    steps = 0
    while alive or inflight:
        steps += 1
        assert steps < 10 ** 6, "no progress"
        if inflight and rng.random() < 0.3:
            slot, k = inflight.pop(rng.randrange(len(inflight)))
            data[slot] = k
            full[slot].tx = False
            full[slot].settle()
            continue
        if alive:
            a = rng.choice(alive)
            try:
                next(a)
            except StopIteration:
                alive.remove(a)


@pytest.mark.parametrize("C,S", [(7, 2), (8, 2), (7, 3), (6, 3), (4, 4)])
@pytest.mark.parametrize("NP", [1, 4, 8])
def test_owned_stages_never_alias(C, S, NP):
    for n in (1, C - 1, C + 1, 55, 221):
        for seed in range(8):
            _simulate(max(n, 1), C, S, NP, seed)


def test_shared_ring_aliases():
    failures = 0
    for seed in range(40):
        try:
            _simulate(221, 8, 2, 4, seed, owned=False, R=18)
        except AssertionError:
            failures += 1
    assert failures > 0
