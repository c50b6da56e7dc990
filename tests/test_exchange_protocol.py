"""Model check of the cross-GPU exchange's record slots (exchange_merge in csrc/tp_attention.cu).

Every rank's sharded call of epoch e stores its record (one query head's (m, l, o) words, each
tagged with e) into every rank's exchange buffer, then reads the records of all ranks from its own
buffer, accepting a word only when it carries e.  A rank starts its call of epoch e + 1 only
after its epoch-e merge has completed (consecutive calls on one exchange never overlap on a GPU),
but nothing orders one rank's next call against a slower rank's reads.  With one record slot per
writer, a fast rank's epoch e + 1 record can overwrite its epoch e record in a slower rank's
buffer before that rank has read it: the slower rank then waits for a word that never comes (its
bounded wait runs out).  The kernel writes epoch e to slot e & 1.  This test drives the protocol
under random schedules and checks that with two slots no reader ever finds its record replaced
and every call completes, and that the one-slot layout does strand a reader.
"""

import random


def _simulate(world, epochs, slots, seed):
    """Returns None when every rank completes every epoch, or a description of the first
    stranded read."""
    rng = random.Random(seed)
    # buf[reader][slot][writer] = epoch tag of the record there (0: never written).
    buf = [[[0] * world for _ in range(slots)] for _ in range(world)]

    def rank(r):
        for e in range(1, epochs + 1):
            s = e % slots
            targets = list(range(world))
            rng.shuffle(targets)
            for t in targets:          # peer stores, one step each
                buf[t][s][r] = e
                yield "run"
            pending = list(range(world))
            rng.shuffle(pending)
            while pending:             # polls of its own buffer, one record per step
                w = pending[0]
                tag = buf[r][s][w]
                if tag == e:
                    pending.pop(0)
                    yield "run"
                elif tag > e:
                    yield f"rank {r} epoch {e}: writer {w}'s record already carries epoch {tag}"
                    return
                else:
                    rng.shuffle(pending)
                    yield "wait"

    gens = {r: rank(r) for r in range(world)}
    for _ in range(200000):
        if not gens:
            return None
        r = rng.choice(sorted(gens))
        try:
            status = next(gens[r])
        except StopIteration:
            del gens[r]
            continue
        if status not in ("run", "wait"):
            return status
    return "no progress (deadlock)"


def test_two_slots_by_epoch_parity_never_strand_a_reader():
    for seed in range(3000):
        world = 2 + seed % 7  # 2 .. 8 ranks
        assert _simulate(world, epochs=6, slots=2, seed=seed) is None, seed


def test_one_slot_strands_a_slow_reader():
    failures = [seed for seed in range(400) if _simulate(2 + seed % 3, epochs=6, slots=1, seed=seed)]
    assert failures, "the one-slot layout should be able to overwrite an unread record"
