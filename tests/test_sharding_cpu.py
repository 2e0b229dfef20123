"""Row sharding, host side (no GPU): partition arithmetic, a 2-rank gloo run whose
all-gathered shards equal the unsharded result, handle exchange, and a rank
failure that the others detect instead of hanging."""
from __future__ import annotations

import ctypes as C
import os
import socket

import numpy as np
import pytest
import torch.distributed as dist
import torch.multiprocessing as mp

import oracle
import qraf_b200 as qb


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


@pytest.mark.parametrize("rows,world", [(4096, 2), (4096, 8), (151936, 8), (128256, 8), (7, 4), (3, 8)])
def test_shard_partition_covers_rows_exactly(rows, world):
    lib = qb.lib
    full = qb.qraf_weight_t()
    fake = 0x10000000   # never dereferenced: sharding is pointer arithmetic
    rb = qb.row_bytes(qb.Q4_0, 4096)
    full.data, full.bytes, full.row_bytes = fake, rb * rows, rb
    full.dtype, full.block_size, full.rows, full.cols = qb.Q4_0, 32, rows, 4096
    covered = 0
    for r in range(world):
        sh = qb.qraf_weight_t()
        assert lib.qraf_cuda_weight_shard(C.byref(full), world, r, C.byref(sh)) == qb.OK
        assert sh.data == fake + covered * rb
        assert sh.bytes == sh.rows * rb and sh.owned == 0
        covered += sh.rows
    assert covered == rows
    bad = qb.qraf_weight_t()
    assert lib.qraf_cuda_weight_shard(C.byref(full), world, world, C.byref(bad)) == qb.ERR_INVALID


def _rank_main(rank, world, port, q, n, k, x, want, mode, out):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    import datetime
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=30))
    try:
        if mode == "fail" and rank == 1:
            raise SystemExit(3)            # a rank that leaves before the collective
        r0, r1 = n * rank // world, n * (rank + 1) // world
        rb = q.size // n
        mine = oracle.Oracle().matvec(oracle.Q4_0, q[r0 * rb:r1 * rb], r1 - r0, k, x)
        parts = [None] * world
        dist.all_gather_object(parts, (r0, mine.tobytes()))
        y = np.zeros(n, np.float32)
        for (a, b) in parts:
            v = np.frombuffer(b, np.float32)
            y[a:a + v.size] = v
        handles = qb.torch_all_gather_bytes()(bytes([rank]) * qb.COMM_HANDLE_BYTES)
        ok = y.tobytes() == want.tobytes() and [h[0] for h in handles] == list(range(world)) and \
            all(len(h) == qb.COMM_HANDLE_BYTES for h in handles)
        out.put((rank, ok))
    except SystemExit:
        raise
    except Exception as e:   # the surviving rank reports the failure it saw
        out.put((rank, f"error: {type(e).__name__}"))
    finally:
        try:
            dist.destroy_process_group()
        except Exception:
            pass


def _run(world, mode, q, n, k, x, want, timeout=90):
    ctx = mp.get_context("spawn")
    out = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_rank_main, args=(r, world, port, q, n, k, x, want, mode, out)) for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout)
    alive = [p for p in procs if p.is_alive()]
    for p in alive:
        p.kill()
    res = {}
    while not out.empty():
        r, v = out.get()
        res[r] = v
    return res, alive, [p.exitcode for p in procs]


def _case():
    orc = oracle.Oracle()
    n, k = 96, 256
    w = qb.fill_normal(42, 0.0, 0.02, n * k).reshape(n, k)
    q = orc.quantize_rows(oracle.Q4_0, w).reshape(-1)
    x = qb.fill_normal(43, 0.0, 1.0, k)
    return q, n, k, x, orc.matvec(oracle.Q4_0, q, n, k, x)


def test_two_rank_gloo_sharded_equals_unsharded():
    q, n, k, x, want = _case()
    res, alive, codes = _run(2, "ok", q, n, k, x, want)
    assert not alive and res == {0: True, 1: True}, (res, codes)


def test_rank_failure_is_detected_not_hung():
    q, n, k, x, want = _case()
    res, alive, codes = _run(2, "fail", q, n, k, x, want, timeout=120)
    assert not alive, "a rank hung after its peer left"
    assert codes[1] == 3
    assert 0 in res and isinstance(res[0], str) and res[0].startswith("error"), res
