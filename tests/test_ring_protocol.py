"""The int4 staging-ring walk of the GEMM engine's dequant warps (csrc/gemm.cu, dequant role), mirrored step by step
on the host and checked for the invariants the device relies on, for staging stages of 2 and 4 k-blocks:
  - every staging stage of every int4 tile is released exactly once by every dequant group (the q_empty barrier
    counts kNumDeqGroups x kNumDeqWarps arrivals per phase);
  - a group waits for a stage (q_full) before it reads it, and releases it only after its last owned k-block there;
  - a group holds at most one stage at a time and walks the stages in order (so a parity wait cannot alias).
Tiles mix int4 and non-int4 problems, odd k-block counts and the LoRA extension k-block."""
import itertools
import random

import pytest

GROUPS = 3


def walk(tiles, qsub, grp):
    """Events (kind, stage, kb) of group `grp`: tiles is a list of (nkb, nkq) (nkq = int4 k-blocks, 0 for
    TMA-sourced weights). Mirrors the device loop: pass_stage for stages without an owned k-block, q_full wait on
    the first owned k-block of a stage, release after the last."""
    ev = []
    it = qi = 0
    for nkb, nkq in tiles:
        it0 = it
        it += nkb
        kb0 = (grp + GROUPS - it0 % GROUPS) % GROUPS
        nstages = (nkq + qsub - 1) // qsub
        qdone, qheld = 0, -1
        for kb in range(kb0, nkb, GROUPS):
            q4 = kb < nkq
            kq = kb // qsub
            if q4:
                while qdone < kq:
                    ev += [("wait", qi + qdone, None), ("release", qi + qdone, None)]
                    qdone += 1
            if q4:
                if qheld != kq:
                    ev.append(("wait", qi + kq, kb))
                    qheld = kq
                ev.append(("read", qi + kq, kb))
                kb_next = kb + GROUPS
                if kb_next >= nkq or kb_next // qsub != kq:
                    ev.append(("release", qi + kq, kb))
                    qdone, qheld = kq + 1, -1
        while qdone < nstages:
            ev += [("wait", qi + qdone, None), ("release", qi + qdone, None)]
            qdone += 1
        qi += nstages
    return ev, qi


def owned(tiles, qsub):
    """stage -> set of (group, kb) that read it, from the ring assignment (k-block r -> group r mod 3)."""
    out = {}
    it = qi = 0
    for nkb, nkq in tiles:
        for kb in range(nkq):
            out.setdefault(qi + kb // qsub, set()).add(((it + kb) % GROUPS, kb))
        it += nkb
        qi += (nkq + qsub - 1) // qsub
    return out


def check(tiles, qsub):
    stages_total = None
    reads = {}
    for g in range(GROUPS):
        ev, nst = walk(tiles, qsub, g)
        stages_total = nst
        held = set()
        released = []
        last = -1
        for kind, st, kb in ev:
            if kind == "wait":
                assert not held, f"group {g} waits stage {st} while holding {held}"
                assert st == last + 1, f"group {g} waits stage {st} out of order (last {last})"
                held.add(st)
            elif kind == "read":
                assert st in held, f"group {g} reads stage {st} without waiting"
                reads.setdefault(st, set()).add((g, kb))
            else:
                assert st in held, f"group {g} releases stage {st} it does not hold"
                held.discard(st)
                released.append(st)
                last = st
        assert not held
        assert released == list(range(nst)), f"group {g}: releases {released}"
    own = owned(tiles, qsub)
    assert set(reads) == set(own) and all(reads[s] == own[s] for s in own)
    assert stages_total == sum((nkq + qsub - 1) // qsub for _, nkq in tiles)


@pytest.mark.parametrize("qsub", [2, 4])
def test_staging_walk_fixed_tiles(qsub):
    # forward gate/up (32 int4 k-blocks), down (8), selected bf16 + LoRA extension (33, no int4), odd int4 counts
    tiles = [(32, 32), (8, 8), (33, 0), (7, 7), (1, 1), (5, 4), (3, 2), (32, 32), (9, 9)]
    check(tiles, qsub)


@pytest.mark.parametrize("qsub", [2, 4])
def test_staging_walk_random_tiles(qsub):
    rnd = random.Random(5)
    for _ in range(300):
        tiles = []
        for _ in range(rnd.randint(1, 12)):
            nkq = rnd.choice([0, 0, 1, 2, 3, 5, 8, 13, 32])
            nkb = nkq + rnd.choice([0, 1]) if nkq else rnd.randint(1, 9)
            tiles.append((nkb, nkq))
        check(tiles, qsub)


def test_every_rotation_of_the_ring():
    # the tile's first ring index decides which group starts; cover all offsets for short tiles
    for pre, nkq in itertools.product(range(GROUPS), range(1, 10)):
        for qsub in (2, 4):
            check([(pre, 0)] * (pre > 0) + [(nkq + 1, nkq), (nkq, nkq)], qsub)
