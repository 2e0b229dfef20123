"""The batch-1 tensor-core kernel (qmv_tc1_kernel: tcgen05 kind::i8, weights
rewritten into MMA tiles before the dependency wait).

It serves one vector under QRAF_MODE_TC where K is a multiple of 1024 up to
4096 and the weight's 32-row CTAs fit one wave.  Its per-block sums
are the FAST path's exact integers, so it is held to the FAST bar against the
reference's result (EXACT mode = the reference's bits) and the fp64 value, and
to strict allclose on the 4096 x 4096 configurations.  Every call goes through
the C ABI."""
from __future__ import annotations

import numpy as np
import pytest

import qraf_b200 as qb
from test_gpu_parity import assert_fast_ok, strict_misses

pytestmark = pytest.mark.gpu

SHAPES = [(qb.Q4_0, 4096, 4096), (qb.Q8_0, 4096, 4096), (qb.Q4_0, 100, 1024), (qb.Q8_0, 4736, 3072),
          (qb.Q4_0, 33, 2048), (qb.Q8_0, 2048, 2048), (qb.Q8_0, 256, 2048), (qb.Q4_0, 4736, 4096),
          (qb.Q8_0, 1, 1024)]


def _weight(dt, n, k, seed, cuda):
    import torch

    wf = torch.from_numpy(qb.fill_normal(seed, 0.0, 0.02, n * k)).to(cuda).reshape(n, k)
    q = qb.quantize_rows(dt, wf).reshape(-1)
    return qb.Weight.from_device(q, dt, n, k), q


@pytest.mark.parametrize("dt,n,k", SHAPES)
def test_tc1_against_the_reference(cuda, oracle_lib, dt, n, k):
    import torch

    w, q = _weight(dt, n, k, 42, cuda)
    x = torch.from_numpy(qb.fill_normal(43, 0.0, 1.0, k)).to(cuda)
    y_tc = qb.matvec_q(w, x, mode=qb.MODE_TC).cpu().numpy()
    y_ref = qb.matvec_q(w, x, mode=qb.MODE_EXACT).cpu().numpy()      # the reference's bits
    y64 = oracle_lib.matvec_f64(dt, q.cpu().numpy(), n, k, x.cpu().numpy())
    assert_fast_ok(y_tc, y_ref, y64, f"tc1 {dt} {n}x{k}")
    if n == 4096 and k == 4096:   # BASELINE configs 0 and 1: strictly within allclose
        assert strict_misses(y_tc, y_ref) == 0
    again = qb.matvec_q(w, x, mode=qb.MODE_TC).cpu().numpy()
    assert again.tobytes() == y_tc.tobytes(), "deterministic"
    assert qb.device_status() == qb.OK


def test_tc1_special_blocks(cuda, oracle_lib):
    """Zero, huge, tiny and non-finite activation blocks: the same outputs as the
    FAST row kernel where finite (within the bar), NaN where it gives NaN."""
    import torch

    n, k = 320, 2048
    for dt in (qb.Q8_0, qb.Q4_0):
        w, q = _weight(dt, n, k, 7, cuda)
        xh = qb.fill_normal(8, 0.0, 1.0, k)
        xh[0:32] = 0.0
        xh[32:64] *= 1e30
        xh[64:96] *= 1e-30
        xh[96:128] *= 1e-42      # subnormal
        x = torch.from_numpy(xh).to(cuda)
        y_tc = qb.matvec_q(w, x, mode=qb.MODE_TC).cpu().numpy()
        y_ref = qb.matvec_q(w, x, mode=qb.MODE_EXACT).cpu().numpy()
        y64 = oracle_lib.matvec_f64(dt, q.cpu().numpy(), n, k, xh)
        assert_fast_ok(y_tc, y_ref, y64, f"special blocks {dt}")
        xh[200] = np.nan
        y_nan = qb.matvec_q(w, torch.from_numpy(xh).to(cuda), mode=qb.MODE_TC).cpu().numpy()
        y_fast = qb.matvec_q(w, torch.from_numpy(xh).to(cuda), mode=qb.MODE_FAST).cpu().numpy()
        assert np.array_equal(np.isnan(y_nan), np.isnan(y_fast)) and np.isnan(y_nan).all()
    assert qb.device_status() == qb.OK


def test_tc1_dependent_chain_and_graph(cuda):
    """A chain y1 = W1 x, y2 = W2 y1, y3 = W1 y2 with programmatic dependent
    launch gives the bits of the same calls without it, eagerly and replayed
    from a CUDA graph."""
    import torch

    k = 4096
    w1, _ = _weight(qb.Q4_0, k, k, 11, cuda)
    w2, _ = _weight(qb.Q8_0, k, k, 12, cuda)
    x = torch.from_numpy(qb.fill_normal(13, 0.0, 1.0, k)).to(cuda)
    ys = [torch.empty(k, device=cuda) for _ in range(3)]

    def chain(flags):
        qb.matvec_q(w1, x, ys[0], mode=qb.MODE_TC | flags)
        qb.matvec_q(w2, ys[0], ys[1], mode=qb.MODE_TC | flags)
        qb.matvec_q(w1, ys[1], ys[2], mode=qb.MODE_TC | flags)

    chain(0)
    torch.cuda.synchronize(cuda)
    want = [y.cpu().numpy().copy() for y in ys]
    for y in ys:
        y.fill_(float("nan"))
    chain(qb.MODE_FLAG_OVERLAP)
    torch.cuda.synchronize(cuda)
    assert all(a.tobytes() == y.cpu().numpy().tobytes() for a, y in zip(want, ys))
    s = torch.cuda.Stream(cuda)
    g = torch.cuda.CUDAGraph()
    with torch.cuda.stream(s):
        chain(qb.MODE_FLAG_OVERLAP)      # warm-up on the capture stream
        s.synchronize()
        with torch.cuda.graph(g, stream=s):
            chain(qb.MODE_FLAG_OVERLAP)
    for y in ys:
        y.fill_(float("nan"))
    for _ in range(3):
        g.replay()
    torch.cuda.synchronize(cuda)
    assert all(a.tobytes() == y.cpu().numpy().tobytes() for a, y in zip(want, ys))
    assert qb.device_status() == qb.OK


def test_tc1_projections_of_one_input_in_one_launch(cuda):
    """qraf_cuda_matvec_q_multi under TC with one vector: the rows of up to four
    weights as one tensor-core launch, bitwise equal to separate calls."""
    import torch

    k = 2048
    ws = [_weight(qb.Q8_0, n, k, 20 + i, cuda)[0] for i, n in enumerate((2048, 256, 256, 40))]
    x = torch.from_numpy(qb.fill_normal(21, 0.0, 1.0, k)).to(cuda)
    got = qb.matvec_q_multi(ws, x.reshape(1, k), mode=qb.MODE_TC)
    for i, w in enumerate(ws):
        want = qb.matvec_q(w, x, mode=qb.MODE_TC)
        assert got[i].reshape(-1).cpu().numpy().tobytes() == want.cpu().numpy().tobytes(), f"weight {i}"
    assert qb.device_status() == qb.OK
