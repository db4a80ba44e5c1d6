"""The GEMM engine's operand ring and int4 staging ring (csrc/gemm.cu), simulated on the host with the mbarrier
semantics the kernel relies on, under random interleavings of its warp roles:

  producers (2 warps, k-blocks of one ring-index parity each): wait `empty`, arrive `full` with transaction bytes
  TMA-Q (1 warp): wait `q_empty`, arrive `q_full` with transaction bytes, stage by stage
  dequant (3 groups x 4 warps, k-blocks of ring index g mod 3): pass staging stages they own nothing of, wait
      `empty`, wait `q_full` on their first k-block of a stage, release `q_empty` after their last, arrive `full`
  MMA (1 warp): per tile wait `acc_empty` of its accumulator (two, alternating), then wait `full` of every k-block
      in order and commit `empty` (when its MMAs complete), then commit `acc_full`
  epilogue (12 warps): per tile wait `acc_full`, read the accumulator, arrive `acc_empty`

A barrier phase completes when all its arrivals are in and its transaction bytes have landed. TMA completions are
asynchronous events in any order; MMA commits arrive in issue order (a tcgen05.commit arrives once every MMA issued
before it has completed, so a later commit never arrives before an earlier one), which is what makes the ring's
consumption in order. A wait is the hardware's parity test (the phase with the waited
parity is the last completed one); the check is that every wait that passes sees exactly the round it means (no
stale pass one phase behind, no overrun two ahead), and that every schedule runs to completion (no deadlock)."""
import random

import pytest

STAGES, GROUPS, DEQ_WARPS, EPI_WARPS = 4, 3, 4, 12


class Bar:
    def __init__(self, name, count):
        self.name, self.count, self.phase, self.arrived, self.tx = name, count, 0, 0, 0

    def arrive(self, tx=0):
        self.arrived += 1
        self.tx += tx
        self._maybe_complete()

    def complete_tx(self, tx):
        self.tx -= tx
        self._maybe_complete()

    def _maybe_complete(self):
        if self.arrived == self.count and self.tx == 0:
            self.phase += 1
            self.arrived = 0

    def parity_passes(self, rnd):
        """try_wait.parity for round `rnd` (parity rnd & 1; round -1 passes on a fresh barrier)."""
        return (self.phase & 1) != (rnd & 1) if rnd >= 0 else True


def roles(tiles, q_stages, Q_SUB):
    """Generators of (op, ...) for every warp, mirroring the device loops."""
    full = [Bar(f"full{s}", DEQ_WARPS + 1) for s in range(STAGES)]
    empty = [Bar(f"empty{s}", 1) for s in range(STAGES)]
    q_full = [Bar(f"q_full{s}", 1) for s in range(q_stages)]
    q_empty = [Bar(f"q_empty{s}", GROUPS * DEQ_WARPS) for s in range(q_stages)]
    acc_full = [Bar(f"acc_full{a}", 1) for a in range(2)]
    acc_empty = [Bar(f"acc_empty{a}", EPI_WARPS) for a in range(2)]

    def producer(prod):
        it = 0
        for nkb, nkq in tiles:
            it0 = it
            it += nkb
            for kb in range(1 if (it0 & 1) != prod else 0, nkb, 2):
                r = it0 + kb
                yield ("wait", empty[r % STAGES], r // STAGES - 1)
                yield ("arrive_tx", full[r % STAGES], 8192)

    def tma_q():
        qi = 0
        for nkb, nkq in tiles:
            for kq in range((nkq + Q_SUB - 1) // Q_SUB):
                yield ("wait", q_empty[qi % q_stages], qi // q_stages - 1)
                yield ("arrive_tx", q_full[qi % q_stages], 4096)
                qi += 1

    def mma():
        it = acc_it = 0
        for nkb, nkq in tiles:
            acc = acc_it & 1
            yield ("wait", acc_empty[acc], (acc_it >> 1) - 1)
            for kb in range(nkb):
                yield ("wait", full[it % STAGES], it // STAGES)
                yield ("commit", empty[it % STAGES])
                it += 1
            yield ("commit", acc_full[acc])
            acc_it += 1

    def epilogue():
        for acc_it in range(len(tiles)):
            acc = acc_it & 1
            yield ("wait", acc_full[acc], acc_it >> 1)
            yield ("arrive", acc_empty[acc])

    def dequant(g):
        it = qi = 0
        for nkb, nkq in tiles:
            it0 = it
            it += nkb
            nst = (nkq + Q_SUB - 1) // Q_SUB
            qdone, qheld = 0, -1
            for kb in range((g + GROUPS - it0 % GROUPS) % GROUPS, nkb, GROUPS):
                r = it0 + kb
                q4 = kb < nkq
                kq = kb // Q_SUB
                if q4:
                    while qdone < kq:
                        qs = qi + qdone
                        yield ("wait", q_full[qs % q_stages], qs // q_stages)
                        yield ("arrive", q_empty[qs % q_stages])
                        qdone += 1
                yield ("wait", empty[r % STAGES], r // STAGES - 1)
                if q4:
                    qs = qi + kq
                    if qheld != kq:
                        yield ("wait", q_full[qs % q_stages], qs // q_stages)
                        qheld = kq
                    if kb + GROUPS >= nkq or (kb + GROUPS) // Q_SUB != kq:
                        yield ("arrive", q_empty[qs % q_stages])
                        qdone, qheld = kq + 1, -1
                yield ("arrive", full[r % STAGES])
            while qdone < nst:
                qs = qi + qdone
                yield ("wait", q_full[qs % q_stages], qs // q_stages)
                yield ("arrive", q_empty[qs % q_stages])
                qdone += 1
            qi += nst

    gens = [producer(0), producer(1), tma_q(), mma()]
    gens += [dequant(g) for g in range(GROUPS) for _ in range(DEQ_WARPS)]
    gens += [epilogue() for _ in range(EPI_WARPS)]
    return gens


def run(tiles, q_stages, rng, q_sub=4):
    gens = roles(tiles, q_stages, q_sub)
    pending = [next(g, None) for g in gens]
    inflight = []  # asynchronous TMA completions (bar, tx), any order
    commits = []   # MMA commits, arriving in issue order
    steps = 0
    while True:
        runnable = [i for i, op in enumerate(pending) if op is not None and
                    (op[0] != "wait" or op[1].parity_passes(op[2]))]
        choices = [("role", i) for i in runnable] + [("async", j) for j in range(len(inflight))]
        if commits:
            choices.append(("commit", 0))
        if not choices:
            stuck = [(i, op[0], op[1].name, op[2]) for i, op in enumerate(pending) if op is not None]
            assert not stuck, f"deadlock: {stuck[:6]}"
            return steps
        kind, i = rng.choice(choices)
        steps += 1
        if kind == "async":
            bar, tx = inflight.pop(i)
            bar.complete_tx(tx)
            continue
        if kind == "commit":
            commits.pop(0).arrive()
            continue
        op = pending[i]
        if op[0] == "wait":
            bar, rnd = op[1], op[2]
            assert rnd < bar.phase <= rnd + 1 or (rnd < 0 and bar.phase == 0), (
                f"role {i} wait on {bar.name} for round {rnd} passed at phase {bar.phase}")
        elif op[0] == "arrive":
            op[1].arrive()
        elif op[0] == "arrive_tx":
            op[1].arrive(op[2])
            inflight.append((op[1], op[2]))
        elif op[0] == "commit":
            commits.append(op[1])
        pending[i] = next(gens[i], None)


@pytest.mark.parametrize("q_sub,q_stages", [(4, 2), (4, 3), (4, 4), (2, 4)])
def test_ring_barriers_random_schedules(q_sub, q_stages):
    rng = random.Random(q_stages * 10 + q_sub)
    for _ in range(150):
        tiles = []
        for _ in range(rng.randint(1, 6)):
            nkq = rng.choice([0, 0, 1, 3, 4, 5, 8, 9, 32])
            tiles.append((nkq + rng.choice([0, 1]) if nkq else rng.randint(1, 9), nkq))
        run(tiles, q_stages, rng, q_sub)


def test_ring_barriers_detect_a_broken_protocol():
    """The checker catches the aliasing it is meant to catch: with fewer ring slots than dequant groups (the kernel
    asserts kNumDeqGroups <= kStages), a group's parity wait on `empty` can pass one phase too early, and some
    schedule shows it."""
    rng = random.Random(7)
    tiles = [(32, 32), (8, 8), (33, 0), (32, 32)]
    global STAGES
    saved = STAGES
    try:
        STAGES = 2  # fewer slots than dequant groups: a group's empty wait can alias (kNumDeqGroups <= kStages)
        with pytest.raises(AssertionError, match="passed at phase"):
            for _ in range(200):
                run(tiles, 3, rng)
    finally:
        STAGES = saved
