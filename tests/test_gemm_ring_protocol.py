"""Model check of the prefill GEMM's raw-weight ring (vibeblade_b200/csrc/vbq_gemm.cu).

One TMA thread loads K step `it` into slot it % 3 of a 3-deep ring; two groups of
dequant warps take alternate steps (group it & 1), release the slot as soon as the bytes
are in registers (8 arrivals on the slot's "empty" barrier) and wait for the next step
with an mbarrier parity wait.  TMA loads complete out of order.

An mbarrier only tracks the parity of its current phase: `try_wait.parity(P)` succeeds when
the current phase's parity differs from P, which is exact only for a waiter at most one
phase ahead of the barrier.  With one "full" barrier per slot, a 3-deep ring and two
groups, a group revisits a slot two phases later and can take the completion from two
phases back for its own while the other group's load is still in flight: it reads stale
bytes, releases the slot early, and the producer then arrives on a phase whose arrival is
spent.  The kernel keeps one full barrier per (slot, group); this model checks that the
per-group barriers deliver every step's own bytes under random latencies, and that the
shared-barrier protocol does not (so the model has the power to see the hazard)."""
from __future__ import annotations

import random

STAGES = 3            # kRStages
CYCLE = 2 * STAGES    # kRCycle: steps it and it + CYCLE share slot and group


class Barrier:
    """mbarrier: arrival count, transaction bytes, phase; parity waits."""

    def __init__(self, count: int):
        self.count = count
        self.pending = count
        self.tx = 0
        self.phase = 0          # index of the current (incomplete) phase
        self.over_arrivals = 0  # arrivals on a phase whose arrival count was spent

    def _maybe_complete(self) -> None:
        if self.pending == 0 and self.tx == 0:
            self.phase += 1
            self.pending = self.count

    def arrive(self, n: int = 1, tx: int = 0) -> None:
        if self.pending < n:
            self.over_arrivals += 1
            self.pending = 0
        else:
            self.pending -= n
        self.tx += tx
        self._maybe_complete()

    def complete_tx(self, nbytes: int) -> None:
        self.tx -= nbytes
        self._maybe_complete()

    def try_wait_parity(self, parity: int) -> bool:
        return (self.phase & 1) != parity


def simulate(per_group: bool, seed: int, nk: int = 48) -> dict:
    rng = random.Random(seed)
    nbytes = 9216
    full = [[Barrier(1), Barrier(1)] for _ in range(STAGES)]
    empty = [Barrier(8) for _ in range(STAGES)]
    slot = [None] * STAGES
    landing: list[tuple[int, int, int, Barrier]] = []  # (time, step, slot, barrier)
    stale = []

    def full_bar(it: int) -> tuple[Barrier, int]:
        q = it % STAGES
        if per_group:
            return full[q][it & 1], (it // CYCLE) & 1
        return full[q][0], (it // STAGES) & 1

    def producer():
        for it in range(nk):
            q = it % STAGES
            yield ("wait", lambda q=q, it=it: empty[q].try_wait_parity(((it // STAGES) & 1) ^ 1))
            bar, _ = full_bar(it)
            bar.arrive(1, tx=nbytes)
            lat = rng.randint(8, 20) + (rng.randint(30, 70) if rng.random() < 0.2 else 0)
            landing.append((now + lat, it, q, bar))
            yield ("delay", 1)

    def group(g: int):
        for it in range(g, nk, 2):
            q = it % STAGES
            bar, par = full_bar(it)
            yield ("wait", lambda bar=bar, par=par: bar.try_wait_parity(par))
            if slot[q] != it:
                stale.append((it, slot[q]))
            empty[q].arrive(8)
            yield ("delay", rng.randint(2, 12))

    actors = [producer(), group(0), group(1)]
    state = [("delay", 0)] * len(actors)
    ready_at = [0] * len(actors)
    done = [False] * len(actors)
    now = 0
    while not all(done) or landing:
        for ev in [e for e in landing if e[0] <= now]:
            landing.remove(ev)
            _, it, q, bar = ev
            slot[q] = it
            bar.complete_tx(nbytes)
        for i, a in enumerate(actors):
            while not done[i]:
                kind, arg = state[i]
                if kind == "delay" and now < ready_at[i]:
                    break
                if kind == "wait" and not arg():
                    break
                try:
                    state[i] = next(a)
                except StopIteration:
                    done[i] = True
                    break
                if state[i][0] == "delay":
                    ready_at[i] = now + state[i][1]
        now += 1
        if now > 100000:
            return {"deadlock": True, "stale": stale, "over": 0}
    over = sum(b.over_arrivals for pair in full for b in pair)
    return {"deadlock": False, "stale": stale, "over": over}


def test_per_group_full_barriers_deliver_every_step():
    for seed in range(200):
        r = simulate(per_group=True, seed=seed)
        assert not r["deadlock"], seed
        assert r["stale"] == [], (seed, r["stale"][:3])
        assert r["over"] == 0, seed


def test_shared_full_barrier_aliases_phases():
    """The protocol the kernel no longer uses: the model finds stale reads."""
    bad = [s for s in range(200) if simulate(per_group=False, seed=s)["stale"]]
    assert bad, "the model no longer exercises two-phase-ahead parity waits"
