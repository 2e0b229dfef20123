"""qraf_cuda_matmul_tc_noalloc: the tensor-core path with its scratch in the
library's fixed device array (no allocation).  Called through the C ABI and
checked against the allocating entry point (qraf_cuda_matvec_q, MODE_TC) on two
calls in a row, with the tolerance the FAST / TC tests use.  Kept in a file of
its own that pytest collects last; it sets up everything it needs, so it also
passes alone in a fresh process."""
from __future__ import annotations

import ctypes as C

import numpy as np
import pytest

import qraf_b200 as qb

pytestmark = pytest.mark.gpu

RTOL, ATOL = 1e-5, 1e-6


def _noalloc(lib, w, x, y, m):
    return lib.qraf_cuda_matmul_tc_noalloc(C.byref(w.desc), C.c_void_p(x.data_ptr()), C.c_void_p(y.data_ptr()), m, 0,
                                           qb._stream(None))


@pytest.mark.parametrize("dt,n,k,m", [(qb.Q8_0, 1000, 2048, 16), (qb.Q4_0, 2048, 4096, 40), (qb.Q8_0, 640, 1024, 70)])
def test_noalloc_matches_the_allocating_entry(cuda, dt, n, k, m):
    import torch

    lib = qb._get_lib()
    wf = torch.from_numpy(qb.fill_normal(42, 0.0, 0.02, n * k)).to(cuda).reshape(n, k)
    q = qb.quantize_rows(dt, wf).reshape(-1)
    w = qb.Weight.from_device(q, dt, n, k)
    x = torch.from_numpy(qb.fill_normal(43, 0.0, 1.0, m * k)).to(cuda).reshape(m, k)
    want = qb.matvec_q(w, x, mode=qb.MODE_TC).cpu().numpy()
    for call in range(2):
        y = torch.full((m, n), float("nan"), device=cuda)
        rc = _noalloc(lib, w, x, y, m)
        assert rc == qb.OK, qb.last_error()
        got = y.cpu().numpy()
        assert np.isfinite(got).all(), f"call {call}: outputs left unwritten"
        np.testing.assert_allclose(got, want, rtol=RTOL, atol=ATOL, err_msg=f"call {call}")
    assert qb.device_status() == qb.OK


def test_noalloc_rejects_scratch_beyond_its_array(cuda):
    """8192 x 28672 Q4_0 with 64 vectors needs about 17.3 MB of scratch, more than
    the 16 MiB array: the call is refused with a clear message and runs nothing."""
    import torch

    lib = qb._get_lib()
    n, k, m = 20000, 28672, 64
    q = torch.zeros(n * qb.row_bytes(qb.Q4_0, k), dtype=torch.uint8, device=cuda)
    w = qb.Weight.from_device(q, qb.Q4_0, n, k)
    x = torch.zeros(m, k, device=cuda)
    y = torch.full((m, n), 7.0, device=cuda)
    rc = _noalloc(lib, w, x, y, m)
    assert rc == qb.ERR_INVALID
    msg = qb.last_error()
    assert "scratch" in msg and str(16 << 20) in msg, msg
    assert torch.all(y == 7.0)
    assert qb.device_status() == qb.OK
