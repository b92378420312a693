"""The paged decode kernel's mbarrier protocol, replayed on the CPU.

`mitten_b200/csrc/decode.cu` (`paged_decode_kernel`) runs four roles per
CTA -- producer (warp 4), MMA issuer (warp 5), softmax (warps 0-3), segment
epilogue (warps 6-9) -- that synchronise only through mbarriers waited on by
phase parity.  A parity wait for phase k returns once k has completed, but
if the barrier has meanwhile completed phase k + 1 as well, the parity reads
"not yet" again and the waiter hangs (bounded in the kernel: it gives up
with a timeout error).  This model replays every wait and arrival of the
kernel, in the kernel's order per role, under random interleavings of the
roles and random completion times of the MMA commits (they complete in
issue order, later than issued), and checks for random segment layouts that
(1) no waiter is ever two phases behind the barrier it waits on, and
(2) every role finishes (no deadlock).
"""
from __future__ import annotations

import random

import pytest

STAGES = 3  # K/V ring stages below head_dim 256


class Bar:
    def __init__(self):
        self.done = 0  # completed phases (every barrier here completes once per use)


class Aliased(AssertionError):
    pass


def roles(first, last, rng, bars, commits):
    """Generators, one per role; each yields the (barrier, phase) it waits on
    before going on, or None to let the scheduler switch roles."""
    n = len(first)
    B = bars

    def wait(name, phase):
        return (B[name], phase, name)

    def producer():
        qcnt = 0
        for i in range(n):
            if first[i]:
                if qcnt >= 2:
                    yield wait(("QEmpty", qcnt & 1), (qcnt >> 1) - 1)
                B[("QFull", qcnt & 1)].done += 1  # TMA bytes land (modelled at once)
                qcnt += 1
            if i >= STAGES:
                yield wait(("KVEmpty", i % STAGES), i // STAGES - 1)
            B[("KVFull", i % STAGES)].done += 1
            yield None

    def mma():
        q_seg = o_seg = -1
        next_s = 0

        def issue_s(j):
            nonlocal q_seg
            if first[j]:
                q_seg += 1
                yield wait(("QFull", q_seg & 1), q_seg >> 1)
            yield wait(("KVFull", j % STAGES), j // STAGES)
            commits.append(("SFull", j & 1))
            if last[j]:
                commits.append(("QEmpty", q_seg & 1))

        for i in range(n):
            while next_s <= i:
                yield from issue_s(next_s)
                next_s += 1
            # the issuer issues S(i+1) early when its operands are there
            if next_s == i + 1 and next_s < n and rng.random() < 0.5:
                j = next_s
                ready = B[("KVFull", j % STAGES)].done > j // STAGES
                if first[j]:
                    ready = ready and B[("QFull", (q_seg + 1) & 1)].done > (q_seg + 1) >> 1
                if ready:
                    yield from issue_s(j)
                    next_s += 1
            yield wait(("PFull", i & 1), i >> 1)
            if first[i]:
                o_seg += 1
                if o_seg >= 2:
                    yield wait(("OFree", o_seg & 1), (o_seg >> 1) - 1)
            commits.append(("ODone", i & 1))
            commits.append(("KVEmpty", i % STAGES))
            if last[i]:
                commits.append(("OSeg", o_seg & 1))
            yield None

    def softmax():
        seg = -1
        for i in range(n):
            if first[i]:
                seg += 1
            yield wait(("SFull", i & 1), i >> 1)
            rescale = (not first[i]) and rng.random() < 0.3
            if rescale:
                yield wait(("ODone", (i - 1) & 1), (i - 1) >> 1)
            elif i >= 2:
                yield wait(("ODone", i & 1), (i - 2) >> 1)
            B[("PFull", i & 1)].done += 1
            if last[i]:
                if seg >= 2:
                    yield wait(("OFree", seg & 1), (seg >> 1) - 1)
                B[("EFull", seg & 1)].done += 1
            yield None

    def epilogue():
        seg = -1
        for i in range(n):
            if first[i]:
                seg += 1
            if last[i]:
                yield wait(("EFull", seg & 1), seg >> 1)
                yield wait(("OSeg", seg & 1), seg >> 1)
                B[("OFree", seg & 1)].done += 1
            yield None

    return [producer(), mma(), softmax(), epilogue()]


def run_once(seg_tiles, rng):
    first, last = [], []
    for t in seg_tiles:
        for j in range(t):
            first.append(j == 0)
            last.append(j == t - 1)
    # a CTA's range may start or end inside a segment: its first tile then
    # starts a piece, its last tile ends one (decode.cu: i == 0 / n_local - 1)
    cut0 = rng.randrange(0, min(3, len(first)))
    cut1 = rng.randrange(0, min(3, len(first) - cut0))
    first, last = first[cut0:len(first) - cut1], last[cut0:len(last) - cut1]
    first[0] = True
    last[-1] = True
    bars = {}
    names = ["QFull", "QEmpty", "SFull", "PFull", "ODone", "OFree", "EFull", "OSeg"]
    for nm in names:
        for b in range(2):
            bars[(nm, b)] = Bar()
    for nm in ["KVFull", "KVEmpty"]:
        for b in range(STAGES):
            bars[(nm, b)] = Bar()
    commits = []  # MMA commits issued, completing later in issue order
    gens = roles(first, last, rng, bars, commits)
    blocked = [None] * len(gens)
    alive = [True] * len(gens)
    steps = 0
    while any(alive):
        steps += 1
        assert steps < 100000, "no progress"
        # complete a prefix of the outstanding commits
        if commits and rng.random() < 0.5:
            for _ in range(rng.randint(1, len(commits))):
                bars[commits.pop(0)].done += 1
        runnable = []
        for r, g in enumerate(gens):
            if not alive[r]:
                continue
            w = blocked[r]
            if w is not None:
                bar, phase, name = w
                if bar.done >= phase + 2:
                    raise Aliased(f"{name} waited for phase {phase} but {bar.done} phases completed")
                if bar.done < phase + 1:
                    continue
            runnable.append(r)
        if not runnable:
            if commits:
                bars[commits.pop(0)].done += 1
                continue
            raise AssertionError(f"deadlock: {[blocked[r][2] if blocked[r] else None for r in range(4)]}")
        r = rng.choice(runnable)
        blocked[r] = None
        try:
            w = next(gens[r])
        except StopIteration:
            alive[r] = False
            continue
        if w is not None:
            bar, phase, name = w
            if bar.done >= phase + 2:
                raise Aliased(f"{name} waited for phase {phase} but {bar.done} phases completed")
            blocked[r] = w


@pytest.mark.parametrize("seed", range(40))
def test_decode_handoff_never_aliases_or_deadlocks(seed):
    rng = random.Random(seed)
    for _ in range(25):
        n_seg = rng.randint(1, 12)
        seg_tiles = [rng.choice([1, 1, 1, 2, 3, 6]) for _ in range(n_seg)]
        run_once(seg_tiles, rng)


def test_model_detects_a_missing_free_wait():
    """The check has teeth: without the softmax's wait for the epilogue of
    segment seg - 2 (which frees the per-buffer slot), one-tile segments let
    the softmax complete a slot's hand-off barrier twice before the epilogue
    has seen the first completion."""
    found = False
    for seed in range(200):
        rng = random.Random(seed)
        try:
            run_once_without_free_wait([1] * 10, rng)
        except Aliased:
            found = True
            break
    assert found


def run_once_without_free_wait(seg_tiles, rng):
    """run_once with the softmax role's OFree wait removed (planted mistake)."""
    global roles
    orig = roles

    def patched(first, last, rng_, bars, commits):
        gens = orig(first, last, rng_, bars, commits)

        def softmax_no_wait():
            seg = -1
            n = len(first)
            for i in range(n):
                if first[i]:
                    seg += 1
                yield (bars[("SFull", i & 1)], i >> 1, ("SFull", i & 1))
                if i >= 2:
                    yield (bars[("ODone", i & 1)], (i - 2) >> 1, ("ODone", i & 1))
                bars[("PFull", i & 1)].done += 1
                if last[i]:
                    bars[("EFull", seg & 1)].done += 1
                yield None

        gens[2] = softmax_no_wait()
        return gens

    roles = patched
    try:
        run_once(seg_tiles, rng)
    finally:
        roles = orig
