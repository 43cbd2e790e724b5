"""CPU model of the producer/consumer ring used by the decode kernels.

The kernels move K/V tiles into NS shared-memory stages with bulk copies that
complete an mbarrier ("full"); consumer warp w takes tiles w, w+NW, ... and
releases a stage by arriving on its "empty" mbarrier.  A parity wait
(``mbarrier.try_wait.parity``) succeeds when the barrier's current phase parity
differs from the requested one, so it is only unambiguous while the waiter is
at most one phase ahead.  This model replays the protocol under random
interleavings and asynchronous copy completion and checks that every consumer
reads the tile it expects and the producer never overwrites a stage that is
still in use.  The host plan keeps NS a multiple of NW; the model shows why.
"""
import random

import pytest


class MBarrier:
    def __init__(self, count):
        self.count = count
        self.pending = count
        self.tx = 0
        self.phase = 0

    def _maybe_complete(self):
        if self.pending == 0 and self.tx == 0:
            self.phase += 1
            self.pending = self.count

    def arrive(self, expect_tx=0):
        self.tx += expect_tx
        self.pending -= 1
        self._maybe_complete()

    def complete_tx(self, nbytes):
        self.tx -= nbytes
        self._maybe_complete()

    def try_wait(self, parity):
        return (self.phase & 1) != parity


def simulate(NS, NW, n_tiles, seed):
    rng = random.Random(seed)
    full = [MBarrier(1) for _ in range(NS)]
    empty = [MBarrier(1) for _ in range(NS)]
    slot_data = [None] * NS          # tile id whose bytes are in the slot
    slot_busy = [None] * NS          # tile id a consumer is reading
    inflight = []                    # (slot, tile) copies not yet landed
    errors = []

    def producer():
        for t in range(n_tiles):
            s = t % NS
            if t >= NS:
                while not empty[s].try_wait(((t // NS) & 1) ^ 1):
                    yield
            if slot_busy[s] is not None:
                errors.append(f"producer overwrote slot {s} (tile {slot_busy[s]} in use) with tile {t}")
            full[s].arrive(expect_tx=2)
            inflight.append((s, t))
            yield

    def consumer(w):
        for t in range(w, n_tiles, NW):
            s = t % NS
            while not full[s].try_wait((t // NS) & 1):
                yield
            if slot_data[s] != t:
                errors.append(f"warp {w} read slot {s} expecting tile {t}, found {slot_data[s]}")
            slot_busy[s] = t
            yield
            slot_busy[s] = None
            empty[s].arrive()
            yield

    procs = [producer()] + [consumer(w) for w in range(NW)]
    alive = list(range(len(procs)))
    steps = 0
    while (alive or inflight) and steps < 200000:
        steps += 1
        if inflight and (not alive or rng.random() < 0.3):
            s, t = inflight.pop(rng.randrange(len(inflight)))
            slot_data[s] = t
            full[s].complete_tx(2)
            continue
        i = rng.choice(alive)
        try:
            next(procs[i])
        except StopIteration:
            alive.remove(i)
    if alive:
        errors.append("deadlock")
    return errors


@pytest.mark.parametrize("NS,NW", [(4, 4), (8, 4), (12, 4), (16, 4), (2, 2), (6, 2)])
def test_ring_is_safe_when_stages_are_a_multiple_of_consumers(NS, NW):
    for seed in range(60):
        for n_tiles in (1, NS - 1, NS, NS + 1, 3 * NS + 2, 40):
            assert simulate(NS, NW, max(n_tiles, 1), seed) == [], (NS, NW, n_tiles, seed)


@pytest.mark.parametrize("NS,NW", [(3, 4), (7, 4)])
def test_ring_breaks_when_stages_are_not_a_multiple_of_consumers(NS, NW):
    bad = sum(bool(simulate(NS, NW, 40, seed)) for seed in range(60))
    assert bad > 0
