"""Model check of the batch 5-16 GEMV's warp-pair protocol (vibeblade_b200/csrc/vbq_gemv_wide.cu).

Warps 2G and 2G + 1 share one B table and meet at a 64-thread named barrier (bar.sync with
a count of 64), which completes only when both warps arrive.  Per stage each warp:

  1. waits for the stage (a bounded wait that may give up),
  2. computes whether its digits left their range (or it is the first stage),
  3. writes its flags (needs a rescale; gave up) and meets the partner (barrier 1),
  4. reads both warps' flags: if either gave up, both leave the loop; if either needs a
     rescale, both flush their sums with the current steps, meet again (barrier 3), and
     then each rescales its own half of the batch rows (writing the shared steps),
  5. writes its half of the table and meets the partner (barrier 2), then runs its MMAs.

The model runs both warps under random schedules, give-ups and rescale decisions and
checks what the kernel relies on: the two warps always take the same barriers in the same
order (a barrier met by one warp only would hang the pair), both leave at the same stage,
a flush never reads a step the partner has already changed, and the flags a warp reads
are the ones written for the same stage.
"""
from __future__ import annotations

import random


def _warp(w, flags, steps, log, rng_need, rng_ok, nst, mode="kernel"):
    """One warp as a generator of ('bar', id) events, mirroring the kernel's loop.
    mode "leave_alone" / "no_bar3" are protocols the kernel does not use (controls)."""
    for it in range(nst):
        ok = rng_ok.random() > 0.03
        need = it == 0 or rng_need.random() < 0.2
        if mode == "leave_alone" and not ok:
            log.append((w, "leave", it))
            return
        flags[w] = (it, need, ok)
        yield ("bar", 1)
        mine, other = flags[w], flags[w ^ 1]
        log.append((w, "flags", it, mine[0], other[0]))
        gave_up = (not mine[2]) or (not other[2])
        if gave_up:
            log.append((w, "leave", it))
            return
        if mine[1] or other[1]:
            if it > 0:
                log.append((w, "flush", it, tuple(steps)))
            if mode != "no_bar3":
                yield ("bar", 3)
            steps[w] = it  # this warp's half of the batch rows gets a new step
        yield ("bar", 2)
        log.append((w, "mma", it))
    log.append((w, "done", nst))


def simulate(seed: int, nst: int = 40, mode: str = "kernel"):
    rng = random.Random(seed)
    flags = [None, None]
    steps = [-1, -1]
    log = []
    # both warps see the same rescale decisions only through the flags; their own draws
    # differ, as their digits do (different batch rows)
    warps = [_warp(w, flags, steps, log, random.Random(seed * 2 + w), random.Random(seed * 7 + w), nst, mode)
             for w in (0, 1)]
    waiting = [None, None]
    done = [False, False]
    events = []
    for _ in range(100000):
        if all(done):
            return log, events, None
        runnable = [w for w in (0, 1) if not done[w] and waiting[w] is None]
        if not runnable:
            # both waiting: they must wait at the same barrier
            if waiting[0] != waiting[1]:
                return log, events, f"barrier mismatch {waiting}"
            events.append(waiting[0])
            waiting = [None, None]
            continue
        w = rng.choice(runnable)
        try:
            ev = next(warps[w])
            waiting[w] = ev
        except StopIteration:
            done[w] = True
            if waiting[w ^ 1] is not None and not done[w ^ 1]:
                return log, events, f"warp {w} left while warp {w ^ 1} waits at {waiting[w ^ 1]}"
    return log, events, "no progress"


def test_pair_protocol_never_splits_the_barriers():
    for seed in range(300):
        log, events, err = simulate(seed)
        assert err is None, (seed, err)
        leaves = [e for e in log if e[1] == "leave"]
        dones = [e for e in log if e[1] == "done"]
        # both warps leave together, at the same stage, or both run to the end
        assert (len(leaves) == 2 and leaves[0][2] == leaves[1][2]) or (not leaves and len(dones) == 2), seed
        # the flags a warp reads after barrier 1 were written for the same stage
        assert all(e[3] == e[2] and e[4] == e[2] for e in log if e[1] == "flags"), seed
        # a flush sees the steps of the previous rescale, not the one of this stage
        assert all(all(s < e[2] for s in e[3]) for e in log if e[1] == "flush"), seed


def _violations(mode):
    bad = 0
    for seed in range(300):
        log, events, err = simulate(seed, mode=mode)
        flush_ok = all(all(v < e[2] for v in e[3]) for e in log if e[1] == "flush")
        if err is not None or not flush_ok:
            bad += 1
    return bad


def test_model_sees_broken_protocols():
    """Controls: a warp leaving on its own timeout strands its partner at a barrier, and a
    rescale without the barrier after the flushes lets a flush read a changed step."""
    assert _violations("leave_alone") > 0
    assert _violations("no_bar3") > 0
