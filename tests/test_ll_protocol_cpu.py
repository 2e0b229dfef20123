"""A CPU model of the fused all-gather's word protocol (qraf_b200/csrc/matvec_rows.cuh,
store_out / sharded_gather; the call numbering of qraf_cuda_matvec_q_sharded in capi.cu).

Each rank runs a chain of sharded calls.  A call reads the rank's call counter
(call = seq + 1), computes its own rows and stores every element as one 8-byte
word (call << 32 | value bits) into each peer's receive array, in the half given by
the call's parity; then it polls its own receive array for the other ranks' rows
until every word carries this call's number, copies them out, and sets seq = call.
A rank's next call starts only after its previous one completed (stream order:
the next launch writes after its dependency wait).  Remote stores land one word at
a time, after arbitrary delays and in any order (relaxed stores over NVLink).

Checked under random interleavings for 2, 4 and 8 ranks: every element a rank
reads is the value the owning rank computed for that same call (no stale word of
an earlier call, no word of a later call overwriting one still to be read), and
every rank finishes every call (no poll is left waiting)."""
from __future__ import annotations

import random

import pytest


def value(call, rank, i):
    return (call * 1_000_003 + rank * 7919 + i) & 0xFFFFFFFF


def run_model(world, rows_per_rank, calls, seed, cap_halves=2):
    rng = random.Random(seed)
    n = world * rows_per_rank
    recv = [[[0] * n for _ in range(cap_halves)] for _ in range(world)]   # [rank][half][element]
    in_flight = []                                                         # (dst, half, idx, word)
    seq = [0] * world

    def rank_prog(r):
        for _ in range(calls):
            call = seq[r] + 1
            half = call & 1
            own = range(r * rows_per_rank, (r + 1) * rows_per_rank)
            for i in own:   # store_out: this rank's rows into every peer's receive array
                word = (call << 32) | value(call, r, i)
                for dst in range(world):
                    if dst != r:
                        in_flight.append((dst, half, i, word))
                yield
            for i in range(n):   # sharded_gather: the other ranks' rows of this call
                if i in own:
                    continue
                while (recv[r][half][i] >> 32) != call:
                    yield
                got = recv[r][half][i] & 0xFFFFFFFF
                assert got == value(call, i // rows_per_rank, i), \
                    f"rank {r} call {call} element {i}: read a value of another call"
            seq[r] = call
            yield

    progs = {r: rank_prog(r) for r in range(world)}
    steps = 0
    while progs or in_flight:
        steps += 1
        assert steps < 5_000_000, "no progress: a poll is left waiting"
        if in_flight and (not progs or rng.random() < 0.5):
            dst, half, i, word = in_flight.pop(rng.randrange(len(in_flight)))
            old = recv[dst][half][i]
            if old:   # the word it replaces must already have been read: two calls back, and dst is past it
                assert (old >> 32) + 2 == (word >> 32), "a word landed over one of the previous call in that half"
                assert seq[dst] >= (old >> 32), "a word landed over one its rank had not read yet"
            recv[dst][half][i] = word
            continue
        r = rng.choice(list(progs))
        try:
            next(progs[r])
        except StopIteration:
            del progs[r]
    assert seq == [calls] * world


@pytest.mark.parametrize("world", [2, 4, 8])
def test_word_protocol_is_safe_and_live(world):
    for seed in range(8):
        run_model(world, rows_per_rank=3, calls=9, seed=seed * 104729 + world)


def test_model_catches_a_single_half_receive_array():
    """Planted mistake (in the model only): one half for every call instead of two by
    parity; a fast rank's next call then overwrites words a slow rank still has to
    read, and the model must report it."""
    import inspect

    src = inspect.getsource(run_model).replace("half = call & 1", "half = 0")
    ns = {}
    exec(compile("import random\n" + inspect.getsource(value) + src, "<model>", "exec"), ns)
    with pytest.raises(AssertionError):
        for seed in range(60):
            ns["run_model"](4, 2, 8, seed=seed)
