"""A CPU model of the batch-1 row kernel's slot ring (qraf_b200/csrc/matvec_rows.cuh,
qmv_rows_kernel): stage s belongs to warp s % 16 and lives in slot s % nst; lane 0
of each warp issues its first stages into their slots (those below the launch's
`early` count before the activations are staged, the rest after the CTA barrier that
ends the staging); a warp that finishes stage s
issues stage s + nst into the slot it just freed (bulk copies completing on the
slot's mbarrier later, in any order), publishing the stage id in shared memory; a
consumer waits for its own stage id, then for the slot's phase parity.

Checked under random interleavings for ring depths 1..32 and a range of stage
counts: every warp reads its slot only when it holds the warp's own stage, no
parity wait is lapped, and every warp finishes.  A planted mistake (the stage-id
wait left out) is reported."""
from __future__ import annotations

import random

import pytest

WARPS = 16


class Bar:
    def __init__(self):
        self.pending, self.tx, self.completed = 1, 0, 0

    def arrive_expect_tx(self, tx):
        self.pending -= 1
        self.tx += tx
        self._check()

    def complete_tx(self, tx):
        self.tx -= tx
        self._check()

    def _check(self):
        if self.pending == 0 and self.tx == 0:
            self.completed += 1
            self.pending = 1

    def try_wait_parity(self, parity):
        """mbarrier.try_wait.parity: true while the phase in progress has the other parity
        (so, on a fresh barrier, parity 1 reads as completed)."""
        return (self.completed & 1) != parity


def run_model(nst, nstages, seed, stage_id_wait=True, early=None):
    """early: stages of the first lap issued before the CTA barrier that ends the
    activation staging (the rest of the lap after it); None = the whole lap."""
    rng = random.Random(seed)
    early = nst if early is None else early
    arrived = [0]                   # warps at the staging barrier
    full = [Bar() for _ in range(nst)]
    slot_stage = [None] * nst
    content = [None] * nst          # the stage whose bytes the slot holds (set when the copy lands)
    reading = [None] * nst          # the stage a warp is reading from the slot right now
    copies = []                     # (slot, stage): copies in flight

    def issue(s, slot):
        assert reading[slot] is None, "a copy was issued into a slot still being read"
        full[slot].arrive_expect_tx(1)
        copies.append((slot, s))
        slot_stage[slot] = s

    def warp_prog(w):
        # lane 0 issues the warp's first stages below `early`, the CTA stages the
        # activations (a barrier every warp reaches), then the rest of the lap
        for s in range(w, min(nst, nstages, early), WARPS):
            issue(s, s)
            yield
        arrived[0] += 1
        while arrived[0] < WARPS:
            yield
        for s in range(w, min(nst, nstages), WARPS):
            if s >= early:
                issue(s, s)
                yield
        slot, phase = w % nst, (w // nst) & 1
        for s in range(w, nstages, WARPS):
            if stage_id_wait:
                while slot_stage[slot] != s:
                    yield
            while not full[slot].try_wait_parity(phase):
                yield
            assert content[slot] == s, f"warp {w} read slot {slot} holding stage {content[slot]} for stage {s}"
            assert full[slot].completed == s // nst + 1, "the parity wait matched another fill of the slot"
            reading[slot] = s
            yield                          # compute on the slot's bytes
            assert content[slot] == s, "the slot was overwritten while its stage was being read"
            reading[slot] = None
            if s + nst < nstages:
                issue(s + nst, slot)
            # advance by WARPS stages: slot += WARPS (mod nst), the phase flips once per wrap
            for _ in range(WARPS):
                slot += 1
                if slot == nst:
                    slot, phase = 0, phase ^ 1
            yield

    progs = {w: warp_prog(w) for w in range(WARPS)}
    steps = 0
    while progs or copies:
        steps += 1
        assert steps < 2_000_000, "no progress: a wait is left without its copy"
        if copies and (not progs or rng.random() < 0.4):
            slot, s = copies.pop(rng.randrange(len(copies)))
            content[slot] = s
            full[slot].complete_tx(1)
            continue
        w = rng.choice(list(progs))
        try:
            next(progs[w])
        except StopIteration:
            del progs[w]


@pytest.mark.parametrize("nst", [1, 2, 3, 5, 8, 16, 17, 32])
@pytest.mark.parametrize("nstages", [1, 7, 16, 40, 97])
@pytest.mark.parametrize("early", [0, 4, 6, None])
def test_slot_ring_is_safe_and_live(nst, nstages, early):
    for seed in range(5):
        run_model(nst, nstages, seed=seed * 31 + nst * 1000 + nstages, early=early)


def test_model_catches_a_missing_stage_id_wait():
    with pytest.raises(AssertionError):
        for seed in range(200):
            run_model(3, 60, seed=seed, stage_id_wait=False)
