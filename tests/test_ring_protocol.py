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
    def __init__(self, count=1):
        self.ph, self.count, self.arrived, self.tx = 0, count, 0, 0

    def done(self, parity):  # try_wait.parity: the phase of that parity has completed
        return (self.ph & 1) != parity

    def arrive(self, tx=0):
        assert self.arrived < self.count, "more arrivals than the barrier's count in one phase"
        self.arrived += 1
        self.tx += tx
        self.settle()

    def settle(self):
        if self.arrived == self.count and self.tx == 0:
            self.ph, self.arrived = self.ph + 1, 0


def _simulate(n, C, S, NP, seed, owned=True, R=None, split=1):
    """C consumers with S stages each; NP issuing lanes (owned=False: stage k % R, lane k % NP);
    with `split`, lanes split * w .. split * w + split - 1 each copy one part of consumer w's units."""
    rng = random.Random(seed)
    R = R or C * S
    full = [_Bar(split) for _ in range(R)]
    empty = [_Bar() for _ in range(R)]
    data, inflight = [[None] * split for _ in range(R)], []

    def stage_of(k):
        if owned:
            w, j = k % C, k // C
            return w * S + j % S, j // S
        return k % R, k // R

    def issue(k, part=0):
        slot, wrap = stage_of(k)
        if wrap > 0:
            while not empty[slot].done((wrap - 1) & 1):
                yield
        full[slot].arrive(tx=1)
        inflight.append((slot, part, k))
        yield

    def producer(p):
        if owned and split > 1:
            w, part = divmod(p, split)
            for k in range(w, n, C):
                yield from issue(k, part)
        elif owned:
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
            assert all(d == k for d in data[slot]), f"read units {data[slot]} expecting {k}"
            yield
            empty[slot].arrive()

    lanes = C * split if split > 1 else NP
    alive = [producer(p) for p in range(lanes)] + [consumer(w) for w in range(C)]
    steps = 0
    while alive or inflight:
        steps += 1
        assert steps < 10 ** 6, "no progress"
        if inflight and rng.random() < 0.3:
            slot, part, k = inflight.pop(rng.randrange(len(inflight)))
            data[slot][part] = k
            full[slot].tx -= 1
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


@pytest.mark.parametrize("split", [2, 4])
def test_split_copies_never_alias(split):
    for n in (1, 6, 8, 55, 221):
        for seed in range(8):
            _simulate(n, 7, 2, 0, seed, split=split)


def test_shared_ring_aliases():
    failures = 0
    for seed in range(40):
        try:
            _simulate(221, 8, 2, 4, seed, owned=False, R=18)
        except AssertionError:
            failures += 1
    assert failures > 0
