"""Row-sharded matvec with the all-gather fused into the kernel (peer stores over
NVLink + bounded flag waits).  In EXACT and FAST sharding never changes a row's
arithmetic, so the gathered y must be bit-identical to the unsharded one; in TC
each rank's rows are its shard's own TC bits (the tile splits K among CTAs by the
shard's size), gathered unchanged."""
from __future__ import annotations

import os
import socket

import numpy as np
import pytest

import qraf_b200 as qb

pytestmark = pytest.mark.gpu


def _weight(torch, dev, dt, n, k, seed=42):
    wf = torch.from_numpy(qb.fill_normal(seed, 0.0, 0.02, n * k)).to(dev).reshape(n, k)
    return qb.quantize_rows(dt, wf).reshape(-1)


@pytest.mark.parametrize("dt", [qb.Q8_0, qb.Q4_0])
@pytest.mark.parametrize("mode", [qb.MODE_EXACT, qb.MODE_FAST])
def test_single_rank_group_equals_plain_matvec(cuda, dt, mode):
    import torch

    n, k = 1024, 2048
    q = _weight(torch, cuda, dt, n, k)
    w = qb.Weight.from_device(q, dt, n, k)
    comm = qb.Comm(1, 0, 7 * n)
    qb.Comm.open_local([comm])
    for m in (1, 2, 5) if mode == qb.MODE_FAST else (1, 3, 7):
        x = torch.from_numpy(qb.fill_normal(43 + m, 0.0, 1.0, m * k)).to(cuda).reshape(m, k)
        if mode == qb.MODE_FAST:   # sharded FAST runs the row kernel on pairs of vectors
            want = np.concatenate([qb.matvec_q(w, x[m0:m0 + 2].contiguous(), mode=mode).cpu().numpy()
                                   for m0 in range(0, m, 2)])
        else:
            want = qb.matvec_q(w, x, mode=mode).cpu().numpy()
        for _ in range(3):   # the output buffer alternates call by call
            got = comm.matvec_q(w, n, 0, x, mode=mode).cpu().numpy()
            assert got.tobytes() == want.tobytes(), f"M={m}"
    assert qb.device_status() == qb.OK
    comm.destroy()


@pytest.mark.parametrize("dt,n,k", [(qb.Q8_0, 1024, 2048), (qb.Q4_0, 2304, 4096)])
def test_single_rank_group_on_the_tensor_cores(cuda, dt, n, k):
    """TC (and AUTO from three vectors) through a one-rank group: the tile's
    sharded store, call numbering and gather give the plain TC call's bits, for one
    group of vectors and for several (70 vectors: groups of 64 and 6, two numbered
    calls), call after call."""
    import torch

    q = _weight(torch, cuda, dt, n, k)
    w = qb.Weight.from_device(q, dt, n, k)
    comm = qb.Comm(1, 0, 70 * n)
    qb.Comm.open_local([comm])
    for m in (3, 16, 70):
        x = torch.from_numpy(qb.fill_normal(50 + m, 0.0, 1.0, m * k)).to(cuda).reshape(m, k)
        want = qb.matvec_q(w, x, mode=qb.MODE_TC).cpu().numpy()
        for md in (qb.MODE_TC, qb.MODE_AUTO, qb.MODE_TC):
            got = comm.matvec_q(w, n, 0, x, mode=md).cpu().numpy()
            assert got.tobytes() == want.tobytes(), f"M={m} mode {md}"
    assert qb.device_status() == qb.OK
    comm.destroy()


@pytest.mark.parametrize("dt,n,k", [(qb.Q4_0, 8192, 4096), (qb.Q4_0, 2048, 28672), (qb.Q8_0, 2048, 11008),
                                     (qb.Q4_0, 10240, 8192)])
@pytest.mark.parametrize("world", [2, 8])
def test_row_shards_compute_the_unsharded_bits(cuda, dt, n, k, world):
    """On one GPU: each row shard, as a plain matvec, gives exactly the rows of the
    full weight's result in both modes (a row's arithmetic does not depend on how
    rows are spread over CTAs), which is what makes sharded results bit-identical."""
    import torch

    q = _weight(torch, cuda, dt, n, k)
    full = qb.Weight.from_device(q, dt, n, k)
    x = torch.from_numpy(qb.fill_normal(44, 0.0, 1.0, k)).to(cuda)
    for md in (qb.MODE_EXACT, qb.MODE_FAST):
        want = qb.matvec_q(full, x, mode=md).cpu().numpy()
        for r in range(world):
            r0, r1 = n * r // world, n * (r + 1) // world
            got = qb.matvec_q(full.shard(world, r), x, mode=md).cpu().numpy()
            assert got.tobytes() == want[r0:r1].tobytes(), f"mode {md} shard {r}/{world}"
    assert qb.device_status() == qb.OK


def test_missing_peer_times_out_and_is_reported(cuda):
    """Rank 0 of a 2-rank group runs alone: its wait for rank 1's signal (a flag
    nothing sets) must end after its time limit with an error status, leaving the
    GPU usable.  One launch only; no second kernel waits on it."""
    import torch

    n, k = 512, 1024
    q = _weight(torch, cuda, qb.Q8_0, n, k)
    full = qb.Weight.from_device(q, qb.Q8_0, n, k)
    c0, c1 = qb.Comm(2, 0, n), qb.Comm(2, 1, n)
    qb.Comm.open_local([c0, c1])
    x = torch.from_numpy(qb.fill_normal(5, 0.0, 1.0, k)).to(cuda)
    shard0 = full.shard(2, 0)
    y0 = c0.matvec_q(shard0, n, 0, x, mode=qb.MODE_EXACT)
    assert qb.device_status(clear=True) == qb.ERR_TIMEOUT
    want = qb.matvec_q(full, x, mode=qb.MODE_EXACT).cpu().numpy()
    assert y0.cpu().numpy()[0, :n // 2].tobytes() == want[:n // 2].tobytes()   # its own rows arrived anyway
    again = qb.matvec_q(full, x, mode=qb.MODE_EXACT).cpu().numpy()            # the context is still usable
    assert again.tobytes() == want.tobytes()
    assert qb.device_status() == qb.OK
    c0.destroy()
    c1.destroy()


def test_missing_peer_times_out_on_the_tensor_cores(cuda):
    """The tile's gather, as the row kernel's: rank 0 of a 2-rank group runs alone,
    its wait for rank 1's rows ends after the time limit with QRAF_ERR_TIMEOUT, its
    own rows are in y and the GPU stays usable.  One launch pair; nothing else
    waits on it."""
    import torch

    n, k, m = 512, 2048, 16
    q = _weight(torch, cuda, qb.Q8_0, n, k)
    full = qb.Weight.from_device(q, qb.Q8_0, n, k)
    c0, c1 = qb.Comm(2, 0, m * n), qb.Comm(2, 1, m * n)
    qb.Comm.open_local([c0, c1])
    x = torch.from_numpy(qb.fill_normal(6, 0.0, 1.0, m * k)).to(cuda).reshape(m, k)
    shard0 = full.shard(2, 0)
    y0 = c0.matvec_q(shard0, n, 0, x, mode=qb.MODE_TC)
    assert qb.device_status(clear=True) == qb.ERR_TIMEOUT
    want = qb.matvec_q(shard0, x, mode=qb.MODE_TC).cpu().numpy()
    assert y0.cpu().numpy()[:, :n // 2].tobytes() == want.tobytes()   # its own rows arrived anyway
    again = qb.matvec_q(shard0, x, mode=qb.MODE_TC).cpu().numpy()     # the context is still usable
    assert again.tobytes() == want.tobytes()
    assert qb.device_status() == qb.OK
    c0.destroy()
    c1.destroy()


@pytest.mark.parametrize("dt,n,k", [(qb.Q4_0, 8192, 4096), (qb.Q8_0, 2048, 11008)])
def test_single_process_multi_gpu_group(cuda, dt, n, k):
    import torch

    ngpu = torch.cuda.device_count()
    if ngpu < 2:
        pytest.skip("needs 2 GPUs")
    world = min(ngpu, 8)
    q_full = _weight(torch, cuda, dt, n, k)
    full = qb.Weight.from_device(q_full, dt, n, k)
    m = 3   # three vectors: two launches per sharded FAST call (pairs), one in EXACT
    x0 = torch.from_numpy(qb.fill_normal(43, 0.0, 1.0, m * k)).reshape(m, k)
    want = {qb.MODE_EXACT: qb.matvec_q(full, x0.to(cuda), mode=qb.MODE_EXACT).cpu().numpy(),
            qb.MODE_FAST: np.concatenate([qb.matvec_q(full, x0[m0:m0 + 2].contiguous().to(cuda),
                                                      mode=qb.MODE_FAST).cpu().numpy() for m0 in (0, 2)])}
    comms, shards, xs, offs = [], [], [], []
    rb = q_full.numel() // n
    for r in range(world):
        torch.cuda.set_device(r)
        qb.init(r)
        r0, r1 = n * r // world, n * (r + 1) // world
        dev = torch.device("cuda", r)
        qs = q_full[r0 * rb:r1 * rb].to(dev)
        shards.append(qb.Weight.from_device(qs, dt, r1 - r0, k))
        xs.append(x0.to(dev))
        offs.append(r0)
        comms.append(qb.Comm(world, r, m * n))
    qb.Comm.open_local(comms)
    for md in (qb.MODE_EXACT, qb.MODE_FAST):
        outs = []
        for r in range(world):   # every rank's kernel is in flight before any finishes
            torch.cuda.set_device(r)
            outs.append(comms[r].matvec_q(shards[r], n, offs[r], xs[r], mode=md))
        for r in range(world):
            torch.cuda.set_device(r)
            assert outs[r].cpu().numpy().tobytes() == want[md].tobytes(), f"rank {r} mode {md}"
            assert qb.device_status() == qb.OK
    # TC: every rank's y holds each shard's own TC bits (16 vectors, one group)
    mt = 16
    xt0 = torch.from_numpy(qb.fill_normal(47, 0.0, 1.0, mt * k)).reshape(mt, k)
    want_tc, xts = [], []
    for r in range(world):
        torch.cuda.set_device(r)
        xts.append(xt0.to(torch.device("cuda", r)))
        want_tc.append(qb.matvec_q(shards[r], xts[r], mode=qb.MODE_TC).cpu().numpy())
    want_tc = np.concatenate(want_tc, axis=1)
    tcomms = []
    for r in range(world):
        torch.cuda.set_device(r)
        tcomms.append(qb.Comm(world, r, mt * n))
    qb.Comm.open_local(tcomms)
    for md in (qb.MODE_TC, qb.MODE_AUTO):
        outs = []
        for r in range(world):
            torch.cuda.set_device(r)
            outs.append(tcomms[r].matvec_q(shards[r], n, offs[r], xts[r], mode=md))
        for r in range(world):
            torch.cuda.set_device(r)
            assert outs[r].cpu().numpy().tobytes() == want_tc.tobytes(), f"rank {r} mode {md}"
            assert qb.device_status() == qb.OK
    for r in range(world):
        torch.cuda.set_device(r)
        comms[r].destroy()
        tcomms[r].destroy()
    torch.cuda.set_device(0)


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _ipc_rank(rank, world, port, dt, n, k, out):
    import datetime

    import torch
    import torch.distributed as dist

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60),
                            device_id=dev)
    try:
        qb.init(rank)
        q_full = _weight(torch, dev, dt, n, k)
        full = qb.Weight.from_device(q_full, dt, n, k)
        x = torch.from_numpy(qb.fill_normal(43, 0.0, 1.0, k)).to(dev)
        r0, r1 = n * rank // world, n * (rank + 1) // world
        shard = full.shard(world, rank)
        comm = qb.make_comm(world, rank, n, qb.torch_all_gather_bytes())
        ok = True
        for md in (qb.MODE_EXACT, qb.MODE_FAST):
            want = qb.matvec_q(full, x, mode=md)
            for _ in range(3):
                got = comm.matvec_q(shard, n, r0, x, mode=md)
                torch.cuda.synchronize()
                ok &= bool(torch.equal(got[0], want))
            # NCCL all-gather of the local rows: the baseline the fused kernel replaces
            local = qb.matvec_q(shard, x, mode=md)
            gathered = torch.empty(n, device=dev)
            dist.all_gather_into_tensor(gathered, local)
            ok &= bool(torch.equal(gathered, want))
        ok &= qb.device_status() == qb.OK
        ok &= _captured_chain_matches(torch, dev, dist, world, rank)
        dist.barrier()
        comm.destroy()
        out.put((rank, ok))
    finally:
        dist.destroy_process_group()


def _captured_chain_matches(torch, dev, dist, world, rank, n=4096, steps=8):
    """A chain of sharded calls (each input is the previous call's gathered output,
    or the one three calls back) captured in a CUDA graph and replayed: the calls
    are numbered on the device, so replays stay in step across ranks and give the
    unsharded chain's bits every time."""
    q_full = _weight(torch, dev, qb.Q8_0, n, n, seed=7)
    full = qb.Weight.from_device(q_full, qb.Q8_0, n, n)
    shard = full.shard(world, rank)
    r0 = n * rank // world
    x0 = torch.from_numpy(qb.fill_normal(11, 0.0, 1.0, n)).to(dev)
    outs, want = [x0], [x0]
    for i in range(steps):
        src = want[-3] if i % 4 == 3 else want[-1]
        want.append(qb.matvec_q(full, src, mode=qb.MODE_FAST))
    comm = qb.make_comm(world, rank, n, qb.torch_all_gather_bytes())
    s = torch.cuda.Stream(dev)

    def chain():
        got = [x0]
        for i in range(steps):
            src = got[-3] if i % 4 == 3 else got[-1]
            got.append(comm.matvec_q(shard, n, r0, src, mode=qb.MODE_FAST | qb.MODE_FLAG_OVERLAP)[0])
        return got

    with torch.cuda.stream(s):
        chain()                       # eager once (first-use set-up happens outside the capture)
    torch.cuda.synchronize(dev)
    dist.barrier()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g, stream=s):
        got = chain()
    ok = True
    for _ in range(3):
        g.replay()
        torch.cuda.synchronize(dev)
        # the last QRAF_COMM_BUFFERS outputs are still in their buffers
        ok &= all(bool(torch.equal(a, b)) for a, b in zip(got[-qb.COMM_BUFFERS:], want[-qb.COMM_BUFFERS:]))
    ok &= qb.device_status() == qb.OK
    dist.barrier()
    del g
    comm.destroy()
    return ok


@pytest.mark.parametrize("dt,n,k", [(qb.Q4_0, 10240, 8192)])
def test_multi_process_ipc_group(cuda, dt, n, k):
    import torch
    import torch.multiprocessing as mp

    ngpu = torch.cuda.device_count()
    if ngpu < 2:
        pytest.skip("needs 2 GPUs")
    world = min(ngpu, 8)
    ctx = mp.get_context("spawn")
    out = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_ipc_rank, args=(r, world, port, dt, n, k, out)) for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(240)
    for p in procs:
        if p.is_alive():
            p.kill()
    res = {}
    while not out.empty():
        r, v = out.get()
        res[r] = v
    assert res == {r: True for r in range(world)}, res
