"""The tensor-core tile's arithmetic (qraf_b200/csrc/matmul_tc.cuh: tc_prep_kernel's limbs
and factors, the exact per-block sums of the kind::f16 MMAs, the epilogue's fold),
restated in numpy and held to the FAST bar against the oracle on BASELINE config-4
and 70B shapes (a sample of rows, several activation vectors).  This pins the
design independently of the GPU: the limbs fit fp16 exactly, every per-block sum
is an integer below 2^24 (so fp32 accumulation in the tensor core is exact), and
the one rounding of each block sum plus the fp32 fold keep the result within the
tolerance the GPU tests apply.  Summation runs block by block in K order here; the
kernel's stream-K split only regroups the same per-block terms."""
from __future__ import annotations

import numpy as np
import pytest

import qraf_b200 as qb
from test_gpu_parity import assert_fast_ok

F32, F64 = np.float32, np.float64


def blocks(q, dt, n, k):
    """Block scales (fp32, [n, nb]) and codes (int64, [n, nb, 32], element order)."""
    nb = k // 32
    if dt == qb.Q8_0:
        b = q.reshape(n, nb, 36)
        s = b[:, :, :4].copy().view(np.float32)[:, :, 0]
        v = b[:, :, 4:].view(np.int8).astype(np.int64)
    else:
        b = q.reshape(n, nb, 18)
        s = b[:, :, :2].copy().view(np.float16)[:, :, 0].astype(np.float32)   # exact fp16 -> fp32
        lo = (b[:, :, 2:] & 15).astype(np.int64) - 8
        hi = (b[:, :, 2:] >> 4).astype(np.int64) - 8
        v = np.stack([lo, hi], -1).reshape(n, nb, 32)
    return s, v


def tc_limbs(x):
    """tc_prep_kernel: e from the exponent bits of the block's max |x| (2^e > max),
    X = rint(x 2^(23-e)) (ties to even), hi = (X + 2048) >> 12, lo = X - 4096 hi,
    factor 2^(e-23)."""
    xb = x.reshape(-1, 32).astype(F32)
    mx = np.abs(xb).max(1)
    ex = ((mx.view(np.uint32) >> 23) & 0xFF).astype(np.int64)
    e = np.where(ex == 0, 1, ex) - 126
    X = np.rint(xb.astype(F64) * np.exp2(23.0 - e)[:, None]).astype(np.int64)
    hi = (X + 2048) >> 12
    lo = X - 4096 * hi
    return hi, lo, np.exp2(e - 23.0).astype(F32)


def tc_matvec(s, v, x):
    hi, lo, fac_x = tc_limbs(x)
    assert np.abs(hi).max() <= 2048 and np.abs(lo).max() <= 2048, "a limb is not exact in fp16"
    dh = np.einsum("nbi,bi->nb", v, hi)
    dl = np.einsum("nbi,bi->nb", v, lo)
    assert np.abs(dh).max() < 2 ** 24 and np.abs(dl).max() < 2 ** 24, "a per-block sum is not exact in fp32"
    t = (4096.0 * dh.astype(F64) + dl.astype(F64)).astype(F32)    # fma(D_hi, 4096, D_lo): one rounding
    fac = (s * fac_x[None, :]).astype(F32)                           # scale x 2^(e-23), exact
    acc = np.zeros(s.shape[0], F32)
    for b in range(s.shape[1]):                                      # acc = fma(t, fac, acc)
        acc = (t[:, b].astype(F64) * fac[:, b].astype(F64) + acc.astype(F64)).astype(F32)
    return acc


@pytest.mark.parametrize("dt,n,k,rows", [
    (qb.Q8_0, 11008, 2048, 384), (qb.Q4_0, 11008, 2048, 384),   # config 4 gate/up
    (qb.Q8_0, 2048, 11008, 256), (qb.Q4_0, 2048, 11008, 256),   # config 4 down
    (qb.Q4_0, 28672, 8192, 128), (qb.Q4_0, 8192, 28672, 96),    # 70B gate/up and down
])
def test_tile_arithmetic_meets_the_fast_bar(oracle_lib, dt, n, k, rows):
    w = qb.fill_normal(42, 0.0, 0.02, rows * k).reshape(rows, k)   # the first rows of the seeded weight
    q = oracle_lib.quantize_rows(dt, w)
    s, v = blocks(q, dt, rows, k)
    for m in range(3):
        x = qb.fill_normal(43 + m, 0.0, 1.0, k)
        y = tc_matvec(s, v, x)
        y_ref = oracle_lib.matvec(dt, q, rows, k, x)
        y64 = oracle_lib.matvec_f64(dt, q, rows, k, x)
        assert_fast_ok(y, y_ref, y64, f"tile arithmetic dt={dt} {n}x{k} vector {m}")


def test_limbs_of_special_blocks():
    """Zero, subnormal-range and mixed-magnitude blocks: limbs stay in range and the
    reconstruction 4096 hi + lo reproduces X."""
    rng = np.random.default_rng(5)
    x = np.concatenate([np.zeros(32), rng.normal(0, 1e-39, 32), rng.normal(0, 1, 32) * 10.0 ** rng.integers(-20, 20, 32),
                        np.full(32, 3.4e38), -np.full(32, 1.0)]).astype(F32)
    hi, lo, fac = tc_limbs(x)
    assert np.abs(hi).max() <= 2048 and np.abs(lo).max() <= 2048
    X = 4096 * hi + lo
    xb = x.reshape(-1, 32).astype(F64)
    assert np.all(np.abs(X * fac[:, None].astype(F64) - xb) <= fac[:, None].astype(F64) * 0.5 + 1e-300)
