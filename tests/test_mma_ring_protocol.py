"""CPU model of mma_grouped_kernel's pipeline (csrc/mma.cu), one CTA.

Roles, as in the kernel:
* producer (warp 0, one lane): per work item and K chunk, at each
  superblock's first chunk a raw stage (wait `raw_empty` of the previous lap,
  expect_tx on `raw_full`, bulk copies land later in any order), then an
  operand stage (wait `op_empty` of the previous lap, expect_tx on `op_full`,
  the activation tile's TMA lands later);
* MMA issuer (warp 1, one lane): per item waits `acc_empty` of the previous
  item, then per chunk waits `op_full` and issues the tensor-core work, which
  runs later in issue order, reads the stage's operands until it completes
  and only then arrives on `op_empty` (tcgen05.commit); after the item's last
  chunk a commit arrives on `acc_full`;
* eight dequantisation warps: per chunk wait `raw_full` at a superblock's
  first chunk, wait `op_empty` of the previous lap, write their part of the
  stage's weight operand, arrive on `op_full`; release the raw stage after a
  superblock's last chunk (or the item's); per item wait `acc_full`, read the
  accumulator, arrive on `acc_empty`.

The operand ring's depth is a launch value (2 .. 6 stages, from the shared
memory left beside the activation tiles), the raw ring has two stages, the
K range of an item is whole superblocks of a split (the last superblock may be
short). Random interleavings, some with one role scheduled far less often,
check that every wait sees the lap it means, that no stage is overwritten
while a reader (a warp or the tensor core) still needs it, that the
accumulator is not overwritten while the epilogue reads it, and that the run
ends. Mistakes planted in the model's protocol are caught.
"""
import random

import pytest

from test_ring_protocol import Bar

RAWS, NDQ = 2, 8


def k_range(s, S, nsb, nkc):
    """Chunks [kc0, kc1) of split s (the kernel's k_range lambda)."""
    return 4 * (s * nsb // S), min(nkc, 4 * ((s + 1) * nsb // S))


def cta_items(bid, grid, total, S, nsb, nkc):
    return [k_range(w % S, S, nsb, nkc) for w in range(bid, total * S, grid)]


def run_pipeline(items, ops, seed, slow=None, plant=None):
    rnd = random.Random(seed)
    raw_full = [Bar(1) for _ in range(RAWS)]
    raw_empty = [Bar(NDQ) for _ in range(RAWS)]
    op_full = [Bar(1 + NDQ) for _ in range(ops)]
    op_empty = [Bar(1) for _ in range(ops)]
    acc_full, acc_empty = Bar(1), Bar(NDQ)
    # Contents: which lap each buffer holds (None while a copy is in flight).
    raw_lap = [None] * RAWS
    op_b = [None] * ops
    op_a = [[None] * NDQ for _ in range(ops)]
    busy_readers = [0] * ops  # tensor-core work issued on a stage, not complete
    acc = {"item": None, "chunks": 0, "readers": 0}
    landings = []  # (bar, buffer setter) of copies in flight, land in any order
    mma_q = []  # tensor-core work in issue order
    done = set()

    def producer():
        raw_it, it = 0, 0
        for kc0, kc1 in items:
            for kc in range(kc0, kc1):
                if kc & 3 == 0:
                    r = raw_it % RAWS
                    if raw_it >= RAWS:
                        while not raw_empty[r].try_wait(((raw_it // RAWS) & 1) ^ 1):
                            yield
                    assert raw_empty[r].phase >= raw_it // RAWS, "raw stage refilled before its release"
                    raw_full[r].expect_tx(1)
                    raw_lap[r] = None

                    def land_raw(r=r, lap=raw_it):
                        raw_lap[r] = lap
                        raw_full[r].complete_tx(1)
                    landings.append(land_raw)
                    raw_it += 1
                o, lap = it % ops, it
                if it >= ops and plant != "producer_skips_op_empty":
                    while not op_empty[o].try_wait(((it // ops) & 1) ^ 1):
                        yield
                assert busy_readers[o] == 0, "activation tile overwritten under the tensor core"
                op_full[o].expect_tx(1)
                op_b[o] = None

                def land_b(o=o, lap=lap):
                    op_b[o] = lap
                    op_full[o].complete_tx(1)
                landings.append(land_b)
                it += 1
                yield
        # Drain: the last `ops` operand copies land before the CTA exits.
        for i in range(max(0, it - ops), it):
            while not op_full[i % ops].try_wait((i // ops) & 1):
                yield
        done.add("producer")

    def mma():
        it = 0
        for ti, (kc0, kc1) in enumerate(items):
            if ti > 0:
                while not acc_empty.try_wait((ti - 1) & 1):
                    yield
                assert acc["readers"] == 0, "accumulator reused while the epilogue reads it"
            for kc in range(kc0, kc1):
                o = it % ops
                while not op_full[o].try_wait((it // ops) & 1):
                    yield
                assert op_full[o].phase == it // ops + 1, "op_full wait aliased"
                busy_readers[o] += 1
                mma_q.append(("chunk", o, it, ti, kc == kc0))
                it += 1
                yield
            mma_q.append(("acc", None, None, ti, False))
        # Drain: the last commit covers every earlier tensor-core operation.
        if it > 0:
            while not op_empty[(it - 1) % ops].try_wait(((it - 1) // ops) & 1):
                yield
        done.add("mma")

    def run_mma_op():
        kind, o, lap, ti, first = mma_q.pop(0)
        if kind == "chunk":
            assert op_b[o] == lap, "tensor core read a stale activation tile"
            assert all(a == lap for a in op_a[o]), "tensor core read a stale weight tile"
            assert acc["readers"] == 0, "accumulator written while the epilogue reads it"
            if first:
                acc["item"], acc["chunks"] = ti, 0
            assert acc["item"] == ti, "accumulation into another item's accumulator"
            acc["chunks"] += 1
            busy_readers[o] -= 1
            op_empty[o].arrive()
        else:
            acc_full.arrive()

    def dequant(w):
        raw_it, it = 0, 0
        for ti, (kc0, kc1) in enumerate(items):
            r = held = 0
            released = True
            for kc in range(kc0, kc1):
                kk = kc & 3
                if kk == 0:
                    r, held = raw_it % RAWS, raw_it
                    while not raw_full[r].try_wait((raw_it // RAWS) & 1):
                        yield
                    assert raw_lap[r] == held, "dequantised a stale raw stage"
                    released = False
                o = it % ops
                if it >= ops and not (plant == "dequant_skips_op_empty" and w == 0):
                    while not op_empty[o].try_wait(((it // ops) & 1) ^ 1):
                        yield
                assert busy_readers[o] == 0, "weight tile overwritten under the tensor core"
                op_a[o][w] = None
                yield
                assert raw_lap[r] == held, "raw stage refilled while being dequantised"
                op_a[o][w] = it
                op_full[o].arrive()
                it += 1
                # The kernel releases a raw stage after its superblock's last
                # chunk (or the item's); the planted mistake after its first.
                last = kk == 3 or kc == kc1 - 1
                if not released and (last or plant == "early_raw_release"):
                    raw_empty[r].arrive()
                    raw_it += 1
                    released = True
            while not acc_full.try_wait(ti & 1):
                yield
            assert acc["item"] == ti and acc["chunks"] == kc1 - kc0, "epilogue read an unfinished accumulator"
            acc["readers"] += 1
            yield
            acc["readers"] -= 1
            acc_empty.arrive()
        done.add(("dq", w))

    gens = {"producer": producer(), "mma": mma()}
    for w in range(NDQ):
        gens[("dq", w)] = dequant(w)
    steps = 0
    while gens or landings or mma_q:
        steps += 1
        assert steps < 2_000_000, "no progress: the protocol deadlocks"
        choices = list(gens)
        if landings:
            choices.append("land")
        if mma_q:
            choices.append("tc")
        pick = rnd.choice(choices)
        if slow is not None and pick == slow and rnd.random() < 0.97:
            continue
        if pick == "land":
            landings.pop(rnd.randrange(len(landings)))()
        elif pick == "tc":
            run_mma_op()
        else:
            try:
                next(gens[pick])
            except StopIteration:
                del gens[pick]
    assert done == {"producer", "mma"} | {("dq", w) for w in range(NDQ)}
    assert acc["readers"] == 0 and not any(busy_readers)
    return steps


# (rows of work items for this CTA): a grid of G CTAs over `total` tiles, S
# splits of nsb superblocks, nkc chunks of 64 (a short last superblock when
# nkc is not a multiple of 4, e.g. 1408 columns -> 22 chunks).
SHAPES = [
    dict(bid=0, grid=148, total=40, S=3, nsb=8, nkc=32),   # split K, one item
    dict(bid=5, grid=148, total=300, S=1, nsb=3, nkc=12),  # several items, whole K
    dict(bid=2, grid=4, total=3, S=2, nsb=6, nkc=22),      # short last superblock
    dict(bid=1, grid=2, total=5, S=1, nsb=1, nkc=4),       # one superblock per item
]


def _items(shape):
    return cta_items(shape["bid"], shape["grid"], shape["total"], shape["S"], shape["nsb"], shape["nkc"])


def test_k_ranges_cover_every_chunk_once():
    """The splits of an item partition its chunks into whole superblocks and
    none is empty (split_count never exceeds the superblock count)."""
    for nsb in range(1, 20):
        for nkc in (4 * nsb, 4 * nsb - 1, 4 * nsb - 2, 4 * nsb - 3):
            for S in range(1, nsb + 1):
                got = []
                for s in range(S):
                    kc0, kc1 = k_range(s, S, nsb, nkc)
                    assert kc0 % 4 == 0 and kc0 < kc1
                    got.extend(range(kc0, kc1))
                assert got == list(range(nkc))


@pytest.mark.parametrize("ops", [2, 3, 4, 6])
@pytest.mark.parametrize("shape", range(len(SHAPES)))
def test_pipeline_random_interleavings(ops, shape):
    items = _items(SHAPES[shape])
    assert items
    for seed in range(6):
        run_pipeline(items, ops, seed)


@pytest.mark.parametrize("slow", ["producer", "mma", ("dq", 3), "land", "tc"])
def test_pipeline_with_a_slow_role(slow):
    items = _items(SHAPES[1])
    for ops in (2, 5):
        for seed in range(3):
            run_pipeline(items, ops, 100 + seed, slow=slow)


@pytest.mark.parametrize("plant, slow", [("producer_skips_op_empty", "tc"), ("dequant_skips_op_empty", "tc"),
                                         ("early_raw_release", ("dq", 3))])
def test_planted_protocol_mistakes_are_caught(plant, slow):
    """The model is strong enough to see the mistakes the waits prevent. With
    the deepest operand ring the producer may run a superblock ahead, so an
    early raw release lets it refill a stage still being dequantised (with two
    operand stages the operand ring alone would hold it back)."""
    items = _items(SHAPES[1])
    caught = 0
    for seed in range(40):
        try:
            run_pipeline(items, 6, seed, slow=slow, plant=plant)
        except AssertionError:
            caught += 1
    assert caught >= 30, caught
