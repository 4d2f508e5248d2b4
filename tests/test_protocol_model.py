"""A model of the device-side completion protocols, run under random
interleavings (CPU): ranks as sequences of atomic steps over shared flag words,
a scheduler that picks any rank able to move.  Checked for every run: nothing
deadlocks, every consumer sees exactly its own call's data, and a rank that
skips a call makes its peers' bounded waits give up instead of hanging.

Forward exchange (fu_qkv.cu, fused_qkv_exchange_kernel): at start the kernel
reads e = epoch + 1 and publishes "entered e" into every member's entry flags;
before its first store into peer d's receive buffer it waits until every
member has entered e; after its stores it publishes e into every member's exit
flag and waits until every member has published e into its own; then the
epoch advances.  A kernel starts only when the previous work on its stream,
including the consumer of the previous outputs, has finished.

Output side (fu_oproj.cu, oproj_exchange_kernel): at start "entered e"; a
push into member s's gather buffer waits until s has entered e, then counts
on s's ready counter; the GEMM waits until its counter holds one count per
peer, reads the buffer, and the kernel resets the counter at its end."""

import random

import pytest


class Deadlock(Exception):
    pass


def run(ranks, seed, max_steps=100000):
    """Drive generator-based ranks: each yields a predicate that must hold
    before its next step.  Returns when all finish; raises on a deadlock."""
    rnd = random.Random(seed)
    waiting = {}
    for r, g in enumerate(ranks):
        waiting[r] = next(g, None)
    live = {r for r, w in waiting.items() if w is not None}
    for _ in range(max_steps):
        if not live:
            return
        ready = [r for r in live if waiting[r]()]
        idle = 0
        while not ready and idle < 1000:      # time passes: bounded waits may give up
            idle += 1
            ready = [r for r in live if waiting[r]()]
        if not ready:
            raise Deadlock(sorted(live))
        r = rnd.choice(ready)
        waiting[r] = next(ranks[r], None)
        if waiting[r] is None:
            live.discard(r)
    raise AssertionError("did not finish")


# ---------------------------------------------------------------- forward exchange
def forward_world(S, calls, skip=None, timeout_steps=None):
    entry = [[0] * S for _ in range(S)]   # entry[d][s]: member s entered, seen by d
    exit_ = [[0] * S for _ in range(S)]   # exit[d][s]: member s finished writing into d
    recv = [[0] * S for _ in range(S)]    # recv[d][s]: call whose data s wrote into d
    epoch = [0] * S
    log = []

    def bounded(pred, budget):
        # A wait that gives up after `budget` scheduler visits (the kernel's
        # timeout); returns whether it was satisfied.
        state = {"n": 0, "ok": None}

        def check():
            if pred():
                state["ok"] = True
                return True
            state["n"] += 1
            if budget is not None and state["n"] > budget:
                state["ok"] = False
                return True
            return False
        return check, state

    def rank(r):
        for c in range(calls):
            if skip == (r, c):
                continue                      # this rank never launches call c
            e = epoch[r] + 1                  # the kernel reads the epoch
            for d in range(S):
                entry[d][r] = e               # CTA 0 publishes entry
            yield lambda: True
            check, st = bounded(lambda: all(entry[r][s] >= e for s in range(S)), timeout_steps)
            yield check                       # before the first peer store
            if not st["ok"]:
                log.append(("timeout", r, c))
                return
            for d in range(S):
                recv[d][r] = e                # stores into every member
                yield lambda: True
            for d in range(S):
                exit_[d][r] = e
            check, st = bounded(lambda: all(exit_[r][s] >= e for s in range(S)), timeout_steps)
            yield check
            if not st["ok"]:
                log.append(("timeout", r, c))
                return
            epoch[r] = e
            # The consumer on this rank's stream, before the next call starts.
            seen = list(recv[r])
            log.append(("consume", r, e, seen))
            yield lambda: True

    return [rank(r) for r in range(S)], log


@pytest.mark.parametrize("S", [1, 2, 3, 4])
def test_forward_protocol_no_deadlock_and_consumers_see_their_call(S):
    for seed in range(300):
        ranks, log = forward_world(S, calls=4)
        run(ranks, seed)
        consumed = [x for x in log if x[0] == "consume"]
        assert len(consumed) == S * 4
        for _, r, e, seen in consumed:
            assert seen == [e] * S, (seed, r, e, seen)


@pytest.mark.parametrize("S", [2, 3])
def test_forward_protocol_skipped_call_ends_in_timeouts(S):
    """The last rank never launches the call (as in the multi-GPU fault case):
    every other rank's bounded wait gives up, and none hangs."""
    for seed in range(100):
        ranks, log = forward_world(S, calls=1, skip=(S - 1, 0), timeout_steps=50)
        run(ranks, seed)
        assert sorted(x[1] for x in log if x[0] == "timeout") == list(range(S - 1))


# ---------------------------------------------------------------- output side
def oproj_world(S, calls):
    entry = [[0] * S for _ in range(S)]
    ready = [0] * S                           # per-owner counter (one m-block)
    gather = [[0] * S for _ in range(S)]      # gather[s][me]: call whose rows me pushed into s
    epoch = [0] * S
    log = []

    def rank(r):
        for c in range(calls):
            e = epoch[r] + 1
            for d in range(S):
                entry[d][r] = e
            yield lambda: True
            # Push: one unit per peer, in any order the scheduler picks.
            for s in [x for x in range(S) if x != r]:
                yield (lambda s=s: entry[r][s] >= e)
                gather[s][r] = e
                yield lambda: True
                ready[s] += 1
            # GEMM: wait for one count per peer, then read the buffer.
            yield lambda: ready[r] >= S - 1
            seen = [gather[r][s] for s in range(S) if s != r]
            assert ready[r] == S - 1          # nobody counts into the next call yet
            log.append(("gemm", r, e, seen))
            ready[r] = 0                      # the last CTA resets the counter
            epoch[r] = e
            yield lambda: True

    return [rank(r) for r in range(S)], log


@pytest.mark.parametrize("S", [1, 2, 3, 4])
def test_oproj_protocol_no_deadlock_and_gemm_reads_its_call(S):
    for seed in range(300):
        ranks, log = oproj_world(S, calls=4)
        run(ranks, seed)
        gemms = [x for x in log if x[0] == "gemm"]
        assert len(gemms) == S * 4
        for _, r, e, seen in gemms:
            assert seen == [e] * (S - 1), (seed, r, e, seen)


def test_model_detects_a_missing_entry_wait():
    """The model is sharp enough to catch a broken protocol: without the entry
    wait, a fast rank overwrites a slow rank's gather buffer before it is read."""
    S, calls = 3, 4

    def broken(r, entry, gather, ready, epoch, log):
        for c in range(calls):
            e = epoch[r] + 1
            yield lambda: True
            for s in [x for x in range(S) if x != r]:
                gather[s][r] = e              # no wait for s to have entered e
                yield lambda: True
                ready[s] += 1
            yield lambda: ready[r] >= S - 1
            log.append([gather[r][s] == e for s in range(S) if s != r])
            ready[r] -= S - 1
            epoch[r] = e
            yield lambda: True

    bad = 0
    for seed in range(300):
        entry = [[0] * S for _ in range(S)]
        gather = [[0] * S for _ in range(S)]
        ready, epoch, log = [0] * S, [0] * S, []
        run([broken(r, entry, gather, ready, epoch, log) for r in range(S)], seed)
        bad += sum(not all(x) for x in log)
    assert bad > 0
