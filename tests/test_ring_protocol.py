"""CPU model of decode_kernel's stage ring (decode.cu): one producer issues
stage ids in (group, segment, unit) order into a ring of n_stages slots;
consumer warps wait on the slot's `full` mbarrier with the lap's phase
parity, after waiting on its `empty` mbarrier for the previous lap's
release, and release it with DARR arrivals in total.

An mbarrier's parity only tells two consecutive phases apart, so a warp may
never wait on a slot two laps ahead of its last release. The model runs the
kernel's stage formulas under random interleavings and checks that every
wait sees the lap it means and that no phase gets more arrivals than its
count. A multi-phase ring (one unit sequence, then another, in the same
ring) needs a consumer barrier between the phases when the first one ends in
a partial group; the model shows it.
"""
import random

import pytest

DW, DARR, NC = 8, 8, 16  # units per group, releases per stage, consumer warps


def tpr_of(wg):
    return 2 if wg > DW // 2 else (4 if wg > DW // 4 else 8)


class Bar:
    """mbarrier: arrival count, transaction bytes, completed-phase counter."""

    def __init__(self, count):
        self.count, self.pend, self.tx, self.phase = count, count, 0, 0

    def arrive(self, c=1):
        self.pend -= c
        assert self.pend >= 0, "more arrivals than the phase expects"
        self._complete()

    def expect_tx(self, nbytes):
        self.tx += nbytes
        self.arrive()

    def complete_tx(self, nbytes):
        self.tx -= nbytes
        self._complete()

    def _complete(self):
        if self.pend == 0 and self.tx == 0:
            self.phase += 1
            self.pend = self.count

    def try_wait(self, parity):
        return (self.phase & 1) != parity


def run_ring(phases, n_stages, seed, consumer_barrier):
    """phases: [(units, segments per unit)] processed in order (gate/up, down)."""
    rnd = random.Random(seed)
    full = [Bar(1) for _ in range(n_stages)]
    empty = [Bar(DARR) for _ in range(n_stages)]
    inflight = []
    bases, b = [], 0
    for nu, nseg in phases:
        bases.append(b)
        b += nu * nseg

    def producer():
        for (nu, nseg), base in zip(phases, bases):
            for gi in range((nu + DW - 1) // DW):
                wg = min(DW, nu - gi * DW)
                for seg in range(nseg):
                    for w in range(wg):
                        sid = base + gi * nseg * DW + seg * wg + w
                        st, ph = sid % n_stages, (sid // n_stages) & 1
                        if sid >= n_stages:
                            while not empty[st].try_wait(ph ^ 1):
                                yield
                        assert full[st].phase == sid // n_stages, "producer reuses a slot early"
                        full[st].expect_tx(16)
                        inflight.append(full[st])
                    yield

    met = [0]

    def consumer(c):
        for pi, ((nu, nseg), base) in enumerate(zip(phases, bases)):
            if pi > 0 and consumer_barrier and phases[pi - 1][0] % DW and nu > 0:
                met[0] += 1
                while met[0] < NC * pi:
                    yield
            for gi in range((nu + DW - 1) // DW):
                wg = min(DW, nu - gi * DW)
                tpr = tpr_of(wg)
                ul = c // tpr
                if ul >= wg:
                    continue
                sid = base + gi * nseg * DW + ul
                for _ in range(nseg):
                    st, ph = sid % n_stages, (sid // n_stages) & 1
                    if sid >= n_stages:
                        while not empty[st].try_wait(ph ^ 1):
                            yield
                        assert empty[st].phase == sid // n_stages, "previous-lap wait aliased"
                    while not full[st].try_wait(ph):
                        yield
                    assert full[st].phase == sid // n_stages + 1, "full wait aliased"
                    yield
                    empty[st].arrive(DARR // tpr)
                    sid += wg

    alive = [producer()] + [consumer(c) for c in range(NC)]
    steps = 0
    while alive:
        steps += 1
        assert steps < 2_000_000, "no progress"
        if inflight and rnd.random() < 0.5:
            inflight.pop(rnd.randrange(len(inflight))).complete_tx(16)
        g = rnd.choice(alive)
        try:
            next(g)
        except StopIteration:
            alive.remove(g)


@pytest.mark.parametrize("units", [9, 17, 25, 33, 8, 3])
def test_single_phase_ring(units):
    """decode_kernel: groups of one geometry, a partial group only at the end."""
    for seed in range(40):
        run_ring([(units, 4)], 14, seed, consumer_barrier=False)


def test_two_phases_need_the_consumer_barrier():
    """7 units (a partial group) then 11 of another geometry in one ring:
    without the barrier a warp idle in the partial group reaches a slot two
    laps ahead."""
    with pytest.raises(AssertionError, match="aliased|more arrivals"):
        for seed in range(200):
            run_ring([(7, 4), (11, 2)], 14, seed, consumer_barrier=False)
    for seed in range(200):
        run_ring([(7, 4), (11, 2)], 14, seed, consumer_barrier=True)


def test_two_phases_random_shapes():
    rnd = random.Random(0)
    for trial in range(150):
        n_gu, n_dn = rnd.randint(0, 26), rnd.randint(0, 26)
        nsg, nsd = rnd.choice([(4, 2), (8, 3), (1, 1), (2, 6), (16, 8)])
        run_ring([(n_gu, nsg), (n_dn, nsd)], rnd.choice([9, 14, 19, 27]), trial, consumer_barrier=True)

