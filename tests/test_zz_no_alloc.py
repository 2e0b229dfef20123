"""qraf_cuda_matmul_tc_noalloc: the tensor-core path for callers that may not
allocate device memory (an engine that handed all device memory to its own pool,
or a thread that must not take cudaMalloc's implicit synchronisation), with its
scratch in the library's fixed device array.  Called through the C ABI on a
fresh stream and checked bit for bit against the allocating entry point
(qraf_cuda_matvec_q, MODE_TC: the same kernels, a deterministic combine) on two
calls in a row, once against the oracle at the FAST / TC bar, and shown to leave
the device's free memory unchanged.  Kept in a file of its own that pytest
collects last; it sets up everything it needs, so it also passes alone in a
fresh process."""
from __future__ import annotations

import ctypes as C

import numpy as np
import pytest

import qraf_b200 as qb
from test_gpu_parity import assert_fast_ok

pytestmark = pytest.mark.gpu


def _noalloc(lib, w, x, y, m, stream):
    return lib.qraf_cuda_matmul_tc_noalloc(C.byref(w.desc), C.c_void_p(x.data_ptr()), C.c_void_p(y.data_ptr()), m, 0,
                                           qb._stream(stream))


@pytest.mark.parametrize("dt,n,k,m", [(qb.Q8_0, 1000, 2048, 16), (qb.Q4_0, 2048, 4096, 40), (qb.Q8_0, 640, 1024, 70)])
def test_noalloc_matches_the_allocating_entry(cuda, oracle_lib, dt, n, k, m):
    import torch

    lib = qb._get_lib()
    wf = torch.from_numpy(qb.fill_normal(42, 0.0, 0.02, n * k)).to(cuda).reshape(n, k)
    q = qb.quantize_rows(dt, wf).reshape(-1)
    del wf
    w = qb.Weight.from_device(q, dt, n, k)
    x = torch.from_numpy(qb.fill_normal(43, 0.0, 1.0, m * k)).to(cuda).reshape(m, k)
    want = qb.matvec_q(w, x, mode=qb.MODE_TC).cpu().numpy()   # loads the kernels; allocates its own scratch
    s = torch.cuda.Stream(cuda)                                 # a stream the library has never seen
    ys = [torch.full((m, n), float("nan"), device=cuda) for _ in range(2)]
    torch.cuda.synchronize(cuda)
    free_before = torch.cuda.mem_get_info(cuda)[0]
    for call in range(2):
        rc = _noalloc(lib, w, x, ys[call], m, s)
        assert rc == qb.OK, qb.last_error()
    s.synchronize()
    free_after = torch.cuda.mem_get_info(cuda)[0]
    assert free_after == free_before, f"device free memory changed by {free_before - free_after} bytes"
    for call in range(2):
        got = ys[call].cpu().numpy()
        assert got.tobytes() == want.tobytes(), f"call {call}: differs from the allocating entry"
    if dt == qb.Q4_0:   # one case against the oracle too
        qh, xh = q.cpu().numpy(), x.cpu().numpy()
        y_ref = np.stack([oracle_lib.matvec(dt, qh, n, k, xh[j]) for j in range(m)])
        y64 = np.stack([oracle_lib.matvec_f64(dt, qh, n, k, xh[j]) for j in range(m)])
        assert_fast_ok(ys[1].cpu().numpy(), y_ref, y64, "no-allocation entry against the oracle")
    assert qb.device_status() == qb.OK


def test_noalloc_rejects_scratch_beyond_its_array(cuda):
    """20000 x 28672 Q4_0 with 64 vectors needs about 17.3 MB of scratch, more than
    the 16 MiB array: the call is refused with a clear message and runs nothing."""
    import torch

    lib = qb._get_lib()
    n, k, m = 20000, 28672, 64
    q = torch.zeros(n * qb.row_bytes(qb.Q4_0, k), dtype=torch.uint8, device=cuda)
    w = qb.Weight.from_device(q, qb.Q4_0, n, k)
    x = torch.zeros(m, k, device=cuda)
    y = torch.full((m, n), 7.0, device=cuda)
    rc = _noalloc(lib, w, x, y, m, None)
    assert rc == qb.ERR_INVALID
    msg = qb.last_error()
    assert "scratch" in msg and str(16 << 20) in msg, msg
    assert torch.all(y == 7.0)
    assert qb.device_status() == qb.OK
