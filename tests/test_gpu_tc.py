"""Tensor-core path (MODE_TC; MODE_AUTO takes it for M >= 3): the tcgen05 tile
against the oracle's reference-order result, with the FAST bar (assert_fast_ok):
every output within allclose(rtol 1e-5, atol 1e-6) of the reference, or no
farther from the fp64 value than the reference's own worst error.  Shapes cover
ragged row tiles, tiles split across CTAs (stream-K partial sums), groups of
more than 64 vectors, and the BASELINE continuous-batching shapes."""
from __future__ import annotations

import numpy as np
import pytest

import qraf_b200 as qb
from test_gpu_parity import assert_fast_ok

pytestmark = pytest.mark.gpu


def _setup(torch, dev, dt, n, k, m, seed=42):
    wf = torch.from_numpy(qb.fill_normal(seed, 0.0, 0.02, n * k)).to(dev).reshape(n, k)
    q = qb.quantize_rows(dt, wf).reshape(-1)
    x = torch.from_numpy(qb.fill_normal(seed + 1, 0.0, 1.0, m * k)).to(dev).reshape(m, k)
    return q, qb.Weight.from_device(q, dt, n, k), x


def _check(oracle_lib, dt, q, n, k, x, y, label):
    qh, xh = q.cpu().numpy(), x.cpu().numpy()
    y_ref = np.stack([oracle_lib.matvec(dt, qh, n, k, xh[j]) for j in range(xh.shape[0])])
    y64 = np.stack([oracle_lib.matvec_f64(dt, qh, n, k, xh[j]) for j in range(xh.shape[0])])
    assert_fast_ok(y, y_ref, y64, label)


@pytest.mark.parametrize("dt", [qb.Q8_0, qb.Q4_0])
@pytest.mark.parametrize("n,k,m", [
    (1000, 512, 16),     # ragged last tile, few units per tile
    (256, 8192, 32),     # 2 tiles, each split over many CTAs (stream-K combine)
    (640, 2048, 64),
    (384, 1024, 1),      # one vector through the tile (MODE_TC forced)
    (300, 1024, 17),     # 17 vectors: 32-wide tile, 15 padding rows
    (128, 256 * 3, 130),  # three launch pairs (64 + 64 + 2)
])
def test_tc_matches_reference(cuda, oracle_lib, dt, n, k, m):
    import torch

    if dt == qb.Q4_0 and k % 256:
        pytest.skip("Q4_0 tiles need K % 256 == 0")
    q, w, x = _setup(torch, cuda, dt, n, k, m)
    y = qb.matvec_q(w, x, mode=qb.MODE_TC).cpu().numpy()
    assert qb.device_status() == qb.OK
    _check(oracle_lib, dt, q, n, k, x, y, f"TC dt={dt} {n}x{k} M={m}")


@pytest.mark.parametrize("dt,n,k", [(qb.Q8_0, 11008, 2048), (qb.Q4_0, 2048, 11008)])
def test_tc_batching_shapes(cuda, oracle_lib, dt, n, k):
    """BASELINE config 4 shapes at M = 16, 32, 64 through MODE_AUTO (which takes
    the tensor cores for M >= 3); outputs checked on a sample of rows."""
    import torch

    q, w, x = _setup(torch, cuda, dt, n, k, 64)
    rows = np.arange(0, n, 7)
    qh = q.cpu().numpy().reshape(n, -1)[rows].reshape(-1)
    for m in (16, 32, 64):
        y = qb.matvec_q(w, x[:m].contiguous(), mode=qb.MODE_AUTO).cpu().numpy()
        y_tc = qb.matvec_q(w, x[:m].contiguous(), mode=qb.MODE_TC).cpu().numpy()
        assert y.tobytes() == y_tc.tobytes()
        xh = x[:m].cpu().numpy()
        y_ref = np.stack([oracle_lib.matvec(dt, qh, rows.size, k, xh[j]) for j in range(m)])
        y64 = np.stack([oracle_lib.matvec_f64(dt, qh, rows.size, k, xh[j]) for j in range(m)])
        assert_fast_ok(y[:, rows], y_ref, y64, f"AUTO dt={dt} {n}x{k} M={m}")
    assert qb.device_status() == qb.OK


def test_auto_switches_to_the_tile_at_three_vectors(cuda, oracle_lib):
    """MODE_AUTO: the row kernel (FAST) for one or two vectors, the tensor-core tile
    from three; both against the reference."""
    import torch

    q, w, x = _setup(torch, cuda, qb.Q4_0, 640, 2048, 8)
    for m in (1, 2, 3, 8):
        xm = x[:m].contiguous()
        y = qb.matvec_q(w, xm, mode=qb.MODE_AUTO)
        want = qb.matvec_q(w, xm, mode=qb.MODE_TC if m >= 3 else qb.MODE_FAST)
        assert torch.equal(y, want), f"M={m}"
        _check(oracle_lib, qb.Q4_0, q, 640, 2048, xm, y.cpu().numpy(), f"AUTO M={m}")
    assert qb.device_status() == qb.OK


def test_tc_is_deterministic_and_nan_propagates(cuda):
    import torch

    q, w, x = _setup(torch, cuda, qb.Q4_0, 512, 4096, 24)
    a = qb.matvec_q(w, x, mode=qb.MODE_TC)
    b = qb.matvec_q(w, x, mode=qb.MODE_TC)
    assert torch.equal(a, b)
    x2 = x.clone()
    x2[3, 100] = float("nan")
    y = qb.matvec_q(w, x2, mode=qb.MODE_TC)
    assert torch.isnan(y[3]).all()
    assert torch.equal(y[:3], a[:3]) and torch.equal(y[4:], a[4:])
    assert qb.device_status() == qb.OK


@pytest.mark.filterwarnings("ignore:The CUDA Graph is empty")   # the refused second capture records nothing
def test_tc_graph_capture_after_first_call(cuda):
    """The first call on a stream sizes its scratch; later calls of that size can be
    captured and replayed.  A capture that would need more scratch is refused with
    an error instead of allocating inside the capture."""
    import torch

    q, w, x = _setup(torch, cuda, qb.Q8_0, 768, 1024, 32)
    s = torch.cuda.Stream(cuda)
    y = torch.empty(32, 768, device=cuda)
    with torch.cuda.stream(s):
        qb.matvec_q(w, x, y, mode=qb.MODE_TC)
    torch.cuda.synchronize()
    want = y.clone()
    y.zero_()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g, stream=s):
        qb.matvec_q(w, x, y, mode=qb.MODE_TC)
    g.replay()
    torch.cuda.synchronize()
    assert torch.equal(y, want)
    del g
    s2 = torch.cuda.Stream(cuda)
    g2 = torch.cuda.CUDAGraph()
    with pytest.raises(qb.QrafError) as e:
        with torch.cuda.graph(g2, stream=s2):
            qb.matvec_q(w, x, y, mode=qb.MODE_TC)
    assert e.value.code == qb.ERR_UNSUPPORTED
    torch.cuda.synchronize()
    assert qb.device_status() == qb.OK


def test_tc_rejects_ineligible_weights(cuda):
    import torch

    q, w, x = _setup(torch, cuda, qb.Q4_0, 64, 384, 16)   # K % 256 != 0
    with pytest.raises(qb.QrafError) as e:
        qb.matvec_q(w, x, mode=qb.MODE_TC)
    assert e.value.code == qb.ERR_UNSUPPORTED
    y = qb.matvec_q(w, x, mode=qb.MODE_AUTO)   # AUTO falls back to the FAST kernels
    assert torch.isfinite(y).all()
