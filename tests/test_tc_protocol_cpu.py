"""A CPU model of the tensor-core tile's barrier protocol (qraf_b200/csrc/matmul_tc.cuh,
qmm_tc_kernel): the raw-unit producer, the four transform warps, the activation
producer, the MMA warp with its asynchronous MMAs and commits, and the eight
epilogue warps, each written as the kernel runs it (rings advanced by counters,
every role synchronising once per pair of stages, waits on the second stage of a
pair where arrivals come in stage order), interleaved at random.

The model checks what the GPU tests cannot reach shape by shape:
  * no role reads a slot before its producer wrote that stage into it, and no
    producer overwrites a slot before its consumer is done with the old stage;
  * no parity wait is lapped (a waiter never finds its barrier two phases on);
  * every role finishes (no wait is left without its arrivals),
for every ring depth the host planner can choose and a range of stage counts."""
from __future__ import annotations

import random

import pytest

R_DONE = 32   # ring of per-stage "MMA done" barriers


class Bar:
    """mbarrier: `count` arrivals (plus transaction bytes) complete a phase."""

    def __init__(self, count):
        self.count, self.pending, self.tx, self.completed = count, count, 0, 0

    def arrive(self, tx=0):
        self.pending -= 1
        self.tx += tx
        self._check()

    def complete_tx(self, tx):
        self.tx -= tx
        self._check()

    def _check(self):
        if self.pending == 0 and self.tx == 0:
            self.completed += 1
            self.pending = self.count

    def ready(self, phase_index):
        """try_wait.parity for the completion of phase `phase_index` (0-based)."""
        if self.completed >= phase_index + 2 and (self.completed & 1) == ((phase_index + 1) & 1):
            raise AssertionError("parity wait lapped: the barrier moved two phases past the waiter")
        return self.completed >= phase_index + 1 and (self.completed - phase_index) % 2 == 1


class Ring:
    def __init__(self, n):
        self.n, self.slot, self.lap = n, 0, 0

    @property
    def wrapped(self):
        return self.lap > 0

    def next(self):
        self.slot += 1
        if self.slot == self.n:
            self.slot, self.lap = 0, self.lap + 1


def run_model(nunits, spu, nraw, nab, nbb, nd, ns, nf, seed, epi_warps=8, xf_warps=4):
    rng = random.Random(seed)
    nst = nunits * spu
    raw_full = [Bar(1) for _ in range(nraw)]
    raw_empty = [Bar(xf_warps) for _ in range(nraw)]
    a_full = [Bar(xf_warps) for _ in range(nab)]
    b_full = [Bar(1) for _ in range(nbb)]
    mma_done = [Bar(1) for _ in range(R_DONE)]
    d_empty = [Bar(epi_warps) for _ in range(nd)]
    s_full = [Bar(xf_warps) for _ in range(ns)]
    s_empty = [Bar(epi_warps) for _ in range(ns)]
    f_full = [Bar(1) for _ in range(nf)]
    f_empty = [Bar(epi_warps) for _ in range(nf)]
    # slot contents: the stage (or unit) last written, and per-slot bookkeeping of readers
    raw_c, a_c, b_c, d_c, s_c, f_c = ([None] * nraw, [None] * nab, [None] * nbb, [None] * nd, [None] * ns,
                                      [None] * nf)
    a_w = [set() for _ in range(nab)]       # transform warps that wrote the current stage
    s_w = [set() for _ in range(ns)]
    async_ops = []                           # pending (kind, payload) completions
    mma_queue = []                           # issued MMA stages not yet complete (in order)
    mma_completed = [-1]                     # highest completed MMA stage
    commits = []                             # (stage whose completion it waits for, barrier)

    def wait(bar, phase_index):
        while not bar.ready(phase_index):
            yield

    def raw_producer():
        r = Ring(nraw)
        for u in range(nunits):
            if r.wrapped:
                yield from wait(raw_empty[r.slot], r.lap - 1)
                assert raw_c[r.slot] is not None
            raw_full[r.slot].arrive(tx=1)
            async_ops.append(("raw", (r.slot, u)))
            r.next()
            yield

    def transform(w):
        rr, ra, rs, rm = Ring(nraw), Ring(nab), Ring(ns), Ring(R_DONE)
        s = 0
        for u in range(nunits):
            yield from wait(raw_full[rr.slot], rr.lap)
            assert raw_c[rr.slot] == u, "transform read a raw slot before its unit landed"
            raw_empty[rr.slot].arrive()
            rr.next()
            for _ in range(0, spu, 2):
                if ra.wrapped:   # MMAs up to stage s + 1 - nab have read both A slots
                    yield from wait(mma_done[rm.slot + 1], rm.lap)
                    rm.next()
                    rm.next()
                if rs.wrapped:
                    yield from wait(s_empty[rs.slot + 1], rs.lap - 1)
                for h in range(2):
                    old = a_c[ra.slot + h]
                    if old is not None and old != s + h:
                        assert mma_completed[0] >= old, "transform overwrote an A slot the MMA had not read"
                    olds = s_c[rs.slot + h]
                    if olds is not None and olds != s + h:
                        assert olds in done_epi, "transform overwrote a scale slot the epilogue had not read"
                    if a_c[ra.slot + h] != s + h:
                        a_c[ra.slot + h], a_w[ra.slot + h] = s + h, set()
                        s_c[rs.slot + h], s_w[rs.slot + h] = s + h, set()
                    a_w[ra.slot + h].add(w)
                    s_w[rs.slot + h].add(w)
                yield
                for h in range(2):   # lane 0 arrives one barrier after another
                    a_full[ra.slot + h].arrive()
                    yield
                    s_full[rs.slot + h].arrive()
                    yield
                ra.next(), ra.next(), rs.next(), rs.next()
                s += 2

    def act_producer():
        rb, rf, rm = Ring(nbb), Ring(nf), Ring(R_DONE)
        for s in range(0, nst, 2):
            if rb.wrapped:   # the MMAs up to stage s + 1 - nbb have read both slots
                yield from wait(mma_done[rm.slot + 1], rm.lap)
                rm.next()
                rm.next()
            for h in range(2):
                old = b_c[rb.slot + h]
                if old is not None:
                    assert mma_completed[0] >= old, "activation tile overwritten before its MMA read it"
                b_full[rb.slot + h].arrive(tx=1)
                async_ops.append(("b", (rb.slot + h, s + h)))
            yield
            if rf.wrapped:
                yield from wait(f_empty[rf.slot + 1], rf.lap - 1)
            for h in range(2):
                old = f_c[rf.slot + h]
                if old is not None:
                    assert old in done_epi, "factor slot overwritten before the epilogue read it"
                f_full[rf.slot + h].arrive(tx=1)
                async_ops.append(("f", (rf.slot + h, s + h)))
            rb.next(), rb.next(), rf.next(), rf.next()
            yield

    def mma_warp():
        ra, rb, rd, rm = Ring(nab), Ring(nbb), Ring(nd), Ring(R_DONE)
        for s in range(0, nst, 2):
            yield from wait(a_full[ra.slot + 1], ra.lap)
            yield from wait(b_full[rb.slot], rb.lap)
            yield from wait(b_full[rb.slot + 1], rb.lap)
            if rd.wrapped:
                yield from wait(d_empty[rd.slot + 1], rd.lap - 1)
            for h in range(2):
                assert a_c[ra.slot + h] == s + h and len(a_w[ra.slot + h]) == xf_warps, \
                    "MMA issued on an A slot the transform had not finished"
                old = d_c[rd.slot + h]
                if old is not None:
                    assert old in done_epi, "MMA overwrote an accumulator the epilogue had not read"
                mma_queue.append((s + h, ra.slot + h, rb.slot + h, rd.slot + h))
                commits.append((s + h, mma_done[rm.slot + h]))
            ra.next(), ra.next(), rb.next(), rb.next(), rd.next(), rd.next(), rm.next(), rm.next()
            yield

    done_epi = set()
    epi_seen = {}

    def epilogue(w):
        rd, rs, rf, rm = Ring(nd), Ring(ns), Ring(nf), Ring(R_DONE)
        for s in range(0, nst, 2):
            yield from wait(mma_done[rm.slot + 1], rm.lap)
            yield from wait(s_full[rs.slot + 1], rs.lap)
            yield from wait(f_full[rf.slot], rf.lap)
            yield from wait(f_full[rf.slot + 1], rf.lap)
            for h in range(2):
                assert mma_completed[0] >= s + h and d_c[rd.slot + h] == s + h, "epilogue read an unfinished D"
                assert s_c[rs.slot + h] == s + h and len(s_w[rs.slot + h]) == xf_warps, "scales not ready"
                assert f_c[rf.slot + h] == s + h, "factors not ready"
            yield
            for h in range(2):
                epi_seen.setdefault(s + h, set()).add(w)
                if len(epi_seen[s + h]) == epi_warps:
                    done_epi.add(s + h)
                d_empty[rd.slot + h].arrive()
                yield
                s_empty[rs.slot + h].arrive()
                yield
                f_empty[rf.slot + h].arrive()
                yield
            rd.next(), rd.next(), rs.next(), rs.next(), rf.next(), rf.next(), rm.next(), rm.next()

    roles = {"raw": raw_producer(), "act": act_producer(), "mma": mma_warp()}
    for w in range(xf_warps):
        roles[f"xf{w}"] = transform(w)
    for w in range(epi_warps):
        roles[f"epi{w}"] = epilogue(w)
    live = dict(roles)
    steps = 0
    while live or async_ops or mma_queue:
        steps += 1
        assert steps < 2_000_000, "no progress: the protocol deadlocked"
        choices = list(live) + (["async"] if async_ops else []) + (["mma_exec"] if mma_queue else [])
        if not choices:
            break
        pick = rng.choice(choices)
        if pick == "async":
            kind, (slot, idx) = async_ops.pop(rng.randrange(len(async_ops)))
            if kind == "raw":
                raw_c[slot] = idx
                raw_full[slot].complete_tx(1)
            elif kind == "b":
                b_c[slot] = idx
                b_full[slot].complete_tx(1)
            else:
                f_c[slot] = idx
                f_full[slot].complete_tx(1)
            continue
        if pick == "mma_exec":   # the oldest issued MMA completes (reads A, B; writes D)
            s, a_slot, b_slot, d_slot = mma_queue.pop(0)
            assert a_c[a_slot] == s and b_c[b_slot] == s, "MMA read an operand slot holding another stage"
            d_c[d_slot] = s
            mma_completed[0] = s
            while commits and commits[0][0] <= s:
                commits.pop(0)[1].arrive()
            continue
        try:
            next(live[pick])
        except StopIteration:
            del live[pick]
    assert not commits
    assert done_epi == set(range(nst)), "the epilogue did not take every stage"
    return steps


# ring depths the host planner can choose (plan_tc): nd = min(8, 512 / (2 n_pad)),
# nbb even in [4, 16], nab 4, ns = nf = 16; raw units nraw in [2, 8]
CONFIGS = [
    # (nraw, nab, nbb, nd)
    (4, 4, 16, 8),   # 16 vectors
    (4, 4, 8, 4),    # 32 vectors
    (2, 4, 4, 2),    # 64 vectors
    (8, 4, 16, 8),
    (3, 4, 6, 2),
]


@pytest.mark.parametrize("nraw,nab,nbb,nd", CONFIGS)
@pytest.mark.parametrize("spu,nunits", [(2, 1), (2, 9), (4, 1), (4, 7), (4, 20), (2, 40)])
def test_pair_protocol_is_safe_and_live(nraw, nab, nbb, nd, spu, nunits):
    for seed in range(6):
        run_model(nunits, spu, nraw, nab, nbb, nd, 16, 16, seed=seed * 7919 + nunits)


def test_model_catches_a_broken_implication():
    """Planted mistake (in the model only): the epilogue waits for the commit of the
    FIRST stage of a pair instead of the second, so the second stage's accumulators
    may still be in flight; the model must report it."""
    import inspect

    good = "yield from wait(mma_done[rm.slot + 1], rm.lap)\n            yield from wait(s_full"
    src = inspect.getsource(run_model)
    assert good in src
    src = src.replace(good, "yield from wait(mma_done[rm.slot], rm.lap)\n            yield from wait(s_full")
    ns = {}
    exec(compile("import random\nR_DONE = 32\n" + inspect.getsource(Bar) + inspect.getsource(Ring) + src,
                 "<model>", "exec"), ns)
    with pytest.raises(AssertionError):
        for seed in range(40):
            ns["run_model"](6, 4, 4, 4, 16, 8, 16, 16, seed=seed)
