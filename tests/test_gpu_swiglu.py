"""qraf_cuda_matvec_q_swiglu: silu(W_gate x) * (W_up x) in one launch (FAST, one
or two vectors) or as the reference's separate steps (other modes).

The fused launch computes each gate and up row with the FAST path's arithmetic,
bit for bit the rows of separate FAST calls, then silu and the product in fp32;
it is checked against those separate calls (a few ulp for expf and the division)
and, like every FAST output, against the reference's pipeline (the oracle's
dispatch_matvec_q outputs, then silu and the product as src/nn/ops.cpp:218-221
and src/nn/attention.cpp:172-179 compute them in fp32) and the fp64 value."""
from __future__ import annotations

import numpy as np
import pytest

import qraf_b200 as qb
from test_gpu_parity import assert_fast_ok

pytestmark = pytest.mark.gpu

CASES = [(qb.Q8_0, 11008, 2048), (qb.Q4_0, 2048, 8192), (qb.Q4_0, 333, 4096), (qb.Q4_0, 640, 28672),
         (qb.Q8_0, 7, 1024)]


def _silu_mul32(g, u):
    g = np.asarray(g, np.float32)
    return (g / (np.float32(1.0) + np.exp(-g))) * np.asarray(u, np.float32)


def _pair(dt, n, k, cuda):
    import torch

    ws, qs = [], []
    for i in range(2):
        wf = torch.from_numpy(qb.fill_normal(60 + i, 0.0, 0.02, n * k)).to(cuda).reshape(n, k)
        q = qb.quantize_rows(dt, wf).reshape(-1)
        ws.append(qb.Weight.from_device(q, dt, n, k))
        qs.append(q)
    return ws, qs


@pytest.mark.parametrize("dt,n,k", CASES)
def test_fused_swiglu(cuda, oracle_lib, dt, n, k):
    import torch

    (wg, wu), (qg, qu) = _pair(dt, n, k, cuda)
    for m in (1, 2):
        x = torch.from_numpy(qb.fill_normal(70 + m, 0.0, 1.0, m * k)).to(cuda).reshape(m, k)
        h = qb.matvec_q_swiglu(wg, wu, x, mode=qb.MODE_FAST).cpu().numpy()
        g = qb.matvec_q(wg, x, mode=qb.MODE_FAST).cpu().numpy()
        u = qb.matvec_q(wu, x, mode=qb.MODE_FAST).cpu().numpy()
        want = _silu_mul32(g, u)
        assert np.allclose(h, want, rtol=1e-6, atol=1e-30), f"{dt} {n}x{k} M={m}: fused differs from FAST + silu"
        # against the reference pipeline
        xh = x.cpu().numpy()
        gh, uh = qg.cpu().numpy(), qu.cpu().numpy()
        g_ref = np.stack([oracle_lib.matvec(dt, gh, n, k, xh[j]) for j in range(m)])
        u_ref = np.stack([oracle_lib.matvec(dt, uh, n, k, xh[j]) for j in range(m)])
        g64 = np.stack([oracle_lib.matvec_f64(dt, gh, n, k, xh[j]) for j in range(m)])
        u64 = np.stack([oracle_lib.matvec_f64(dt, uh, n, k, xh[j]) for j in range(m)])
        h64 = (g64 / (1.0 + np.exp(-g64))) * u64
        assert_fast_ok(h, _silu_mul32(g_ref, u_ref), h64, f"swiglu {dt} {n}x{k} M={m}")
        h_auto = qb.matvec_q_swiglu(wg, wu, x, mode=qb.MODE_AUTO).cpu().numpy()
        assert h_auto.tobytes() == h.tobytes()
    assert qb.device_status() == qb.OK


def test_unfused_modes(cuda, oracle_lib):
    """EXACT: the reference's bits for both projections, then silu and the product
    on the GPU; TC with four vectors: the tensor-core tile twice, then the same."""
    import torch

    dt, n, k = qb.Q8_0, 1024, 2048
    (wg, wu), (qg, qu) = _pair(dt, n, k, cuda)
    x = torch.from_numpy(qb.fill_normal(80, 0.0, 1.0, 4 * k)).to(cuda).reshape(4, k)
    h = qb.matvec_q_swiglu(wg, wu, x[:1].contiguous(), mode=qb.MODE_EXACT).cpu().numpy()
    g = qb.matvec_q(wg, x[:1].contiguous(), mode=qb.MODE_EXACT).cpu().numpy()
    u = qb.matvec_q(wu, x[:1].contiguous(), mode=qb.MODE_EXACT).cpu().numpy()
    assert np.allclose(h, _silu_mul32(g, u), rtol=1e-6, atol=1e-30)
    h4 = qb.matvec_q_swiglu(wg, wu, x, mode=qb.MODE_TC).cpu().numpy()
    g4 = qb.matvec_q(wg, x, mode=qb.MODE_TC).cpu().numpy()
    u4 = qb.matvec_q(wu, x, mode=qb.MODE_TC).cpu().numpy()
    assert np.allclose(h4, _silu_mul32(g4, u4), rtol=1e-6, atol=1e-30)
    assert qb.device_status() == qb.OK


def test_swiglu_rejects_mismatched_weights(cuda):
    import torch

    (wg, _), _ = _pair(qb.Q8_0, 64, 1024, cuda)
    (wu, _), _ = _pair(qb.Q8_0, 32, 1024, cuda)
    x = torch.zeros(1024, device=cuda)
    with pytest.raises(qb.QrafError) as e:
        qb.matvec_q_swiglu(wg, wu, x)
    assert e.value.code == qb.ERR_INVALID
