"""Fusions around the projections (qraf_cuda_matvec_q_multi_ex, qraf_cuda_matvec_q_swiglu_ex):
RMSNorm of the input folded into the projections' launch, biases added to their
outputs.  EXACT gives the bits of the reference's own steps (dispatch_rms_norm,
then dispatch_matvec_q, then dispatch_add: src/nn/transformer.cpp:588-590,
src/nn/attention.cpp:92-102), here the oracle's restatement of them, which the
CPU suite pins to the reference library; FAST and TC meet the FAST bar against
that pipeline and its fp64 value."""
from __future__ import annotations

import numpy as np
import pytest

import qraf_b200 as qb
from test_gpu_parity import assert_fast_ok

pytestmark = pytest.mark.gpu
EPS = 1e-6


def _weights(dt, rows, k, seed, cuda):
    import torch

    ws, qs = [], []
    for i, n in enumerate(rows):
        wf = torch.from_numpy(qb.fill_normal(seed + i, 0.0, 0.02, n * k)).to(cuda).reshape(n, k)
        q = qb.quantize_rows(dt, wf).reshape(-1)
        ws.append(qb.Weight.from_device(q, dt, n, k))
        qs.append(q.cpu().numpy())
    return ws, qs


def _reference(oracle_lib, dt, qs, rows, k, xh, gamma, biases, f64=False):
    """Per vector: RMSNorm, then each projection, then its bias (fp32 add)."""
    outs = [[] for _ in rows]
    for j in range(xh.shape[0]):
        xn = oracle_lib.rms_norm(xh[j], gamma, EPS) if gamma is not None else xh[j]
        for i, (q, n) in enumerate(zip(qs, rows)):
            y = oracle_lib.matvec_f64(dt, q, n, k, xn) if f64 else oracle_lib.matvec(dt, q, n, k, xn)
            if biases is not None and biases[i] is not None:
                y = y + biases[i].astype(np.float64 if f64 else np.float32)
            outs[i].append(y)
    return [np.stack(o) for o in outs]


CASES = [(qb.Q8_0, (2048, 256, 256), 2048),    # Qwen2-3B Q, K, V with biases
         (qb.Q4_0, (4096,), 4096),              # one weight: RMSNorm and bias
         (qb.Q4_0, (640, 700), 28672)]          # long rows: the limb-prep kernel normalises


@pytest.mark.parametrize("dt,rows,k", CASES)
def test_norm_and_bias(cuda, oracle_lib, dt, rows, k):
    import torch

    ws, qs = _weights(dt, rows, k, 90, cuda)
    rng = np.random.default_rng(3)
    gamma = rng.normal(1.0, 0.2, size=k).astype(np.float32)
    biases = [rng.normal(0.0, 0.1, size=n).astype(np.float32) if i != 1 else None for i, n in enumerate(rows)]
    g_dev = torch.from_numpy(gamma).to(cuda)
    b_dev = [torch.from_numpy(b).to(cuda) if b is not None else None for b in biases]
    for mode, ms in ((qb.MODE_EXACT, (1, 3)), (qb.MODE_FAST, (1, 2)), (qb.MODE_TC, (1, 4))):
        if mode == qb.MODE_TC and (k % 256) != 0:
            continue
        for m in ms:
            xh = (qb.fill_normal(100 + m, 0.0, 3.0, m * k)).reshape(m, k)
            x = torch.from_numpy(xh).to(cuda)
            got = qb.matvec_q_multi(ws, x, mode=mode, norm_w=g_dev, norm_eps=EPS, biases=b_dev)
            assert np.array_equal(x.cpu().numpy(), xh), "x is not modified"
            want = _reference(oracle_lib, dt, qs, rows, k, xh, gamma, biases)
            want64 = _reference(oracle_lib, dt, qs, rows, k, xh, gamma, biases, f64=True)
            for i in range(len(rows)):
                y = got[i].cpu().numpy()
                if mode == qb.MODE_EXACT:
                    assert y.tobytes() == want[i].astype(np.float32).tobytes(), f"EXACT M={m} weight {i}"
                else:
                    assert_fast_ok(y, want[i], want64[i], f"mode {mode} M={m} weight {i}")
    assert qb.device_status() == qb.OK


def test_bias_only_keeps_exact_bits(cuda, oracle_lib):
    import torch

    dt, n, k = qb.Q8_0, 2048, 2048
    ws, qs = _weights(dt, (n,), k, 95, cuda)
    b = np.random.default_rng(4).normal(0.0, 0.5, size=n).astype(np.float32)
    xh = qb.fill_normal(7, 0.0, 1.0, k).reshape(1, k)
    y = qb.matvec_q_multi(ws, torch.from_numpy(xh).to(cuda), mode=qb.MODE_EXACT,
                          biases=[torch.from_numpy(b).to(cuda)])[0].cpu().numpy()
    want = oracle_lib.matvec(dt, qs[0], n, k, xh[0]) + b
    assert y.tobytes() == want.astype(np.float32).reshape(1, n).tobytes()


@pytest.mark.parametrize("dt,n,k", [(qb.Q8_0, 11008, 2048), (qb.Q4_0, 640, 28672)])
def test_norm_then_swiglu(cuda, oracle_lib, dt, n, k):
    import torch

    (wg, wu), (qg, qu) = _weights(dt, (n, n), k, 110, cuda)
    gamma = np.random.default_rng(6).normal(1.0, 0.2, size=k).astype(np.float32)
    for mode, m in ((qb.MODE_FAST, 1), (qb.MODE_FAST, 2), (qb.MODE_EXACT, 1)):
        xh = qb.fill_normal(120 + m, 0.0, 2.0, m * k).reshape(m, k)
        h = qb.matvec_q_swiglu(wg, wu, torch.from_numpy(xh).to(cuda), mode=mode,
                               norm_w=torch.from_numpy(gamma).to(cuda), norm_eps=EPS).cpu().numpy()
        gr, ur = _reference(oracle_lib, dt, [qg, qu], (n, n), k, xh, gamma, None)
        g64, u64 = _reference(oracle_lib, dt, [qg, qu], (n, n), k, xh, gamma, None, f64=True)
        want = (gr / (np.float32(1.0) + np.exp(-gr))) * ur
        want64 = (g64 / (1.0 + np.exp(-g64))) * u64
        assert_fast_ok(h, want, want64, f"norm + swiglu mode {mode} M={m}")
    assert qb.device_status() == qb.OK
