"""The drop-in, end to end: the reference's own code calling the CUDA path.

oracle/_ref/libqraf_ref_cuda.so is the reference's sources linked the way a QRAF
maintainer links the library (backend.cpp's scalar dispatch_matvec_q renamed, the
shim qraf_b200/shim/dispatch_matvec_q_cuda.cpp in its place).  The reference's
unmodified SwiGLU MLP (src/nn/attention.cpp:159-186: gate, up and down
projections through do_matvec -> dispatch_matvec_q) must give bit-identical
results on the GPU (default EXACT mode) and on the reference's CPU build.
"""
from __future__ import annotations

import ctypes as C
import os

import numpy as np
import pytest

import oracle

pytestmark = pytest.mark.gpu

REF_CUDA_SO = os.path.join(os.path.dirname(oracle.REF_SO), "libqraf_ref_cuda.so")


def _mlp_lib(path):
    lib = C.CDLL(path)
    f = lib.qref_mlp_forward
    f.restype = None
    f.argtypes = [C.c_void_p, C.c_void_p, C.c_void_p, C.c_void_p, C.c_void_p, C.c_uint64, C.c_uint64, C.c_uint32,
                  C.c_int, C.c_uint32, C.c_uint32]
    return lib


@pytest.mark.skipif(not (oracle.reference_available() and os.path.exists(REF_CUDA_SO)),
                    reason="reference builds (oracle/_ref) not present")
@pytest.mark.parametrize("dtype", [oracle.Q8_0, oracle.Q4_0])
@pytest.mark.parametrize("hidden,inter", [(512, 1376), (2048, 11008)])
def test_reference_mlp_on_cuda_is_bit_identical(cuda, dtype, hidden, inter):
    import qraf_b200 as qb

    ref = oracle.Reference()
    cpu, gpu = _mlp_lib(oracle.REF_SO), _mlp_lib(REF_CUDA_SO)
    seed = 1000 + hidden + dtype
    wg = ref.quantize_rows(dtype, qb.fill_normal(seed, 0.0, 0.02, inter * hidden).reshape(inter, hidden))
    wu = ref.quantize_rows(dtype, qb.fill_normal(seed + 1, 0.0, 0.02, inter * hidden).reshape(inter, hidden))
    wd = ref.quantize_rows(dtype, qb.fill_normal(seed + 2, 0.0, 0.02, hidden * inter).reshape(hidden, inter))
    x = qb.fill_normal(seed + 3, 0.0, 1.0, hidden)
    outs = []
    for lib in (cpu, gpu):
        for _ in range(2):      # the second call runs on cached device weights
            out = np.zeros(hidden, dtype=np.float32)
            lib.qref_mlp_forward(out.ctypes.data, x.ctypes.data, wg.ctypes.data, wu.ctypes.data, wd.ctypes.data,
                                 wg.nbytes, wd.nbytes, dtype, 32, hidden, inter)
            outs.append(out)
    assert outs[0].tobytes() == outs[1].tobytes()
    assert outs[2].tobytes() == outs[0].tobytes(), "the reference's MLP on the CUDA drop-in is not bit-identical"
    assert outs[3].tobytes() == outs[0].tobytes()
