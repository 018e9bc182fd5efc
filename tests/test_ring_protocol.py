"""CPU model of decode_kernel's stage ring (csrc/decode.cu, decode_dev.cuh).

The producer side is the kernel's: a CTA's units are taken DW at a time (a
group); for each segment of the group, producer lane w issues unit w's stage
(waiting on the slot's `empty` mbarrier for the previous lap's release), the
lanes independently of one another, and all lanes meet at a named barrier
before the next segment. Consumer warps (TPR per unit) wait for the slot's
previous lap to be released, then on the slot's `full` mbarrier with the
lap's phase parity, and release it with DARR arrivals in total.

An mbarrier's parity only tells two consecutive phases apart. A fast consumer
can reach lap L of a slot while lap L-1 is not yet issued -- its producer
lane is still waiting for a slow unit to release lap L-2 -- so a parity test
of the release barrier would take lap L-2's pending phase for the release it
wants, read stale data and over-release the slot. The kernel therefore
counts releases per slot (a monotonic shared-memory counter) for the
consumers' previous-lap wait; the producer keeps the parity wait, which
cannot alias (it issues lap L only after lap L-1, and issued lap L-1 only
after lap L-2 was released). The model runs random interleavings, some with
a few consumer warps scheduled a hundred times less often, and checks that
every wait sees the lap it means and that no phase gets more arrivals than
its count; with a parity previous-lap wait it finds the aliasing.
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


def run_ring(nu, nseg, n_stages, seed, counted=True, slow=()):
    """One CTA with nu units of nseg segments each in an n_stages ring."""
    rnd = random.Random(seed)
    full = [Bar(1) for _ in range(n_stages)]
    empty = [Bar(DARR) for _ in range(n_stages)]
    rel = [0] * n_stages  # release counts (count_add / count_wait)
    inflight = []
    n_groups = (nu + DW - 1) // DW
    met = {}

    def lane(w):
        for gi in range(n_groups):
            wg = min(DW, nu - gi * DW)
            for seg in range(nseg):
                if w < wg:
                    sid = gi * nseg * DW + seg * wg + w
                    st, ph = sid % n_stages, (sid // n_stages) & 1
                    if sid >= n_stages:
                        while not empty[st].try_wait(ph ^ 1):
                            yield
                    assert full[st].phase == sid // n_stages, "producer reuses a slot early"
                    full[st].expect_tx(16)
                    inflight.append(full[st])
                met[(gi, seg)] = met.get((gi, seg), 0) + 1
                while met[(gi, seg)] < DW:  # producer_sync (named barrier)
                    yield

    def consumer(c):
        for gi in range(n_groups):
            wg = min(DW, nu - gi * DW)
            tpr = tpr_of(wg)
            ul = c // tpr
            if ul >= wg:
                continue
            sid = gi * nseg * DW + ul
            for _ in range(nseg):
                st, ph = sid % n_stages, (sid // n_stages) & 1
                if sid >= n_stages:
                    if counted:
                        while rel[st] < (sid // n_stages) * DARR:
                            yield
                    else:
                        while not empty[st].try_wait(ph ^ 1):
                            yield
                    assert empty[st].phase == sid // n_stages, "previous-lap wait aliased"
                while not full[st].try_wait(ph):
                    yield
                assert full[st].phase == sid // n_stages + 1, "full wait aliased"
                yield
                empty[st].arrive(DARR // tpr)
                rel[st] += DARR // tpr
                sid += wg

    gens = {("p", w): lane(w) for w in range(DW)}
    for c in range(NC):
        gens[c] = consumer(c)
    steps = 0
    while gens:
        steps += 1
        assert steps < 5_000_000, "no progress"
        if inflight and rnd.random() < 0.5:
            inflight.pop(rnd.randrange(len(inflight))).complete_tx(16)
        keys = list(gens)
        key = rnd.choices(keys, weights=[0.01 if k in slow else 1.0 for k in keys])[0]
        try:
            next(gens[key])
        except StopIteration:
            del gens[key]


# Ring geometries of the shipped kernel (segments per unit, stages): Q4_K with
# four superblocks per stage, 9 stages x 2 segments (d=2048) or x 4 (d=4096);
# Q6_K with two, 14 x 2 (ff=768) and 7-stage-wide rows; and deeper rings.
GEOMS = [(2, 9), (4, 9), (2, 14), (4, 14), (4, 19)]


@pytest.mark.parametrize("units", [3, 8, 9, 17, 25, 33, 40])
def test_ring_even_speeds(units):
    for seed in range(20):
        nseg, ns = GEOMS[seed % len(GEOMS)]
        run_ring(units, nseg, ns, seed)


def test_ring_with_slow_warps():
    """A few consumer warps much slower than the rest (an expert with more
    rows, a warp held up elsewhere): the counted previous-lap wait holds."""
    for trial in range(200):
        rnd = random.Random(trial)
        nseg, ns = rnd.choice(GEOMS)
        slow = set(rnd.sample(range(NC), rnd.randint(1, 3)))
        run_ring(rnd.choice([16, 17, 24, 25, 32, 33, 40]), nseg, ns, trial, counted=True, slow=slow)


def test_parity_previous_lap_wait_aliases():
    """The same schedules with a parity test for the previous lap's release
    (the kernel's earlier form) alias: a fast warp passes two laps early."""
    with pytest.raises(AssertionError, match="aliased|more arrivals"):
        for trial in range(200):
            rnd = random.Random(trial)
            nseg, ns = rnd.choice(GEOMS)
            slow = set(rnd.sample(range(NC), rnd.randint(1, 3)))
            run_ring(rnd.choice([16, 17, 24, 25, 32, 33, 40]), nseg, ns, trial, counted=False, slow=slow)
