"""The CPU oracle, pinned against the reference's own outputs (no GPU needed).

The oracle (oracle/qraf_oracle.c) restates src/tensor/quantize.cpp,
src/tensor/dtype.cpp and src/nn/backend.cpp.  These tests hold it to the
golden fixtures that tests/golden/make_golden.py produced with the reference's
compiled sources, and, where oracle/_ref is built, to the reference directly.
"""
from __future__ import annotations

import hashlib
import os

import numpy as np
import pytest

import oracle
from conftest import GOLDEN

Q8, Q4 = oracle.Q8_0, oracle.Q4_0


def sha(a):
    return hashlib.sha256(np.ascontiguousarray(a).tobytes()).hexdigest()


# ── the reference's own unit tests (tests/test_quantize.cpp:7-50) ─────────
def test_reference_unit_cases(oracle_lib):
    u = np.load(os.path.join(GOLDEN, "ref_unit_cases.npz"))
    q8 = oracle_lib.quantize(Q8, u["data"], 8)
    q4 = oracle_lib.quantize(Q4, u["data"], 8)
    assert q8.tobytes() == u["q8"].tobytes()
    assert q4.tobytes() == u["q4"].tobytes()
    d8 = oracle_lib.dequantize_block(Q8, q8, 8)
    d4 = oracle_lib.dequantize_block(Q4, q4, 8)
    assert d8.tobytes() == u["q8_deq"].tobytes()
    assert d4.tobytes() == u["q4_deq"].tobytes()
    # The reference's own tolerances (test_quantize.cpp:20, :35, :48).
    assert np.all(np.abs(d8 - u["data"]) <= 0.02)
    assert np.all(np.abs(d4 - u["data"]) <= 0.3)
    qa = oracle_lib.quantize(Q8, u["dot_a"], 4)
    assert qa.tobytes() == u["dot_q8"].tobytes()
    r = oracle_lib.dot(Q8, qa, u["dot_b"], 4, 4)
    assert np.float32(r).tobytes() == u["dot_result"].tobytes()
    assert abs(r - 5.0) <= 0.1


# ── seeded small cases: bytes, outputs and per-block partials bit-exact ──
def test_small_cases_bit_exact(oracle_lib, small_cases):
    for i, c in enumerate(small_cases):
        dt, bs, n, k = c["dtype"], c["bs"], c["n"], c["k"]
        if "w" in c:
            q = oracle_lib.quantize_rows(dt, c["w"], bs)
            assert q.tobytes() == c["q"].tobytes(), f"case {i}: quantized bytes differ"
        y = oracle_lib.matmul(dt, c["q"], n, k, c["x"], bs)
        assert y.tobytes() == c["y"].tobytes(), f"case {i}: y differs"
        p = oracle_lib.block_partials(dt, c["q"], n, k, c["x"][0], bs)
        assert p.tobytes() == c["partials"].tobytes(), f"case {i}: partials differ"


def test_unknown_dtype_zero_fills(oracle_lib):
    # dispatch_matvec_q zero-fills y for a dtype it has no kernel for (backend.cpp:195-198).
    y = oracle_lib.matvec(30, np.zeros(64, np.uint8), 4, 32, np.ones(32, np.float32))
    assert np.all(y == 0)


def test_fp16_truncating_encoder(oracle_lib):
    # fp32_to_fp16 truncates (dtype.cpp:52): 1 + 2^-11 + 2^-12 rounds down, not up.
    assert oracle_lib.fp32_to_fp16(1.0 + 2.0 ** -11 + 2.0 ** -12) == 0x3C00
    assert oracle_lib.fp32_to_fp16(float("nan")) == 0x7C00            # NaN -> inf
    assert oracle_lib.fp32_to_fp16(1e-5) == 0x0000                    # below 2^-14 -> 0
    assert oracle_lib.fp32_to_fp16(-65520.0) == 0xFBFF                # truncation keeps it finite
    assert oracle_lib.fp16_to_fp32(0x0001) == 2.0 ** -24              # subnormal decode is exact


# ── full-size configuration digests (the cheap ones run here) ────────────
@pytest.mark.parametrize("name", ["cfg1_q8_4096x4096", "cfg2_q4_4096x4096", "cfg3_q8_kv", "cfg3_q8_qo"])
def test_config_digests_oracle(oracle_lib, digests, name):
    import qraf_b200

    d = digests[name]
    w = qraf_b200.fill_normal(d["seed_w"], 0.0, 0.02, d["n"] * d["k"])
    q = oracle_lib.quantize(d["dtype"], w, d["block_size"])
    assert sha(q) == d["sha_q"]
    x = qraf_b200.fill_normal(d["seed_x"], 0.0, 1.0, d["k"])
    y = oracle_lib.matvec(d["dtype"], q, d["n"], d["k"], x, d["block_size"])
    assert sha(y[None, :]) == d["y"]["1"]


# ── direct cross-check with the reference's compiled code, where built ────
@pytest.mark.skipif(not oracle.reference_available(), reason="oracle/_ref not built here")
def test_oracle_matches_reference_randomised(oracle_lib):
    ref = oracle.Reference()
    rng = np.random.default_rng(7)
    for trial in range(60):
        dt = (Q8, Q4)[trial % 2]
        bs = int(rng.choice([1, 2, 3, 4, 7, 8, 16, 32, 33, 64]))
        if dt == Q4 and bs < 2:
            bs = 2
        n, k = int(rng.integers(1, 9)), int(rng.integers(1, 300))
        w = (rng.standard_normal((n, k)) * 10.0 ** rng.integers(-6, 4)).astype(np.float32)
        x = rng.standard_normal(k).astype(np.float32)
        qa, qb = oracle_lib.quantize_rows(dt, w, bs), ref.quantize_rows(dt, w, bs)
        assert qa.tobytes() == qb.tobytes()
        assert oracle_lib.matvec(dt, qa, n, k, x, bs).tobytes() == ref.matvec(dt, qb, n, k, x, bs).tobytes()
    for h in range(0, 65536, 7):
        a = np.float32(oracle_lib.fp16_to_fp32(h))
        b = np.float32(ref.lib.qref_fp16_to_fp32(h))
        assert a.tobytes() == b.tobytes() or (np.isnan(a) and np.isnan(b))


def _block_scales(dt, q, n, k):
    nb = k // 32
    raw = np.asarray(q, np.uint8).reshape(n, nb, 36 if dt == 10 else 18)
    if dt == 10:
        return raw[:, :, :4].copy().view(np.float32)[:, :, 0].astype(np.float64)
    return raw[:, :, :2].copy().view(np.float16)[:, :, 0].astype(np.float64)


@pytest.mark.parametrize("dt", [10, 20])
def test_limb_partials_reconstruct_the_dot(oracle_lib, dt):
    """The integer restatement of the FAST path: sum_b scale_b c_b sum_j 2^(8(3-j)) D_j
    matches the fp64 dot up to the rounding of X_i (half a unit of c_b per element),
    including blocks of zeros, of tiny (subnormal-range) and of huge values."""
    n, k = 16, 512
    rng = np.random.default_rng(7)
    w = rng.normal(0.0, 0.02, (n, k)).astype(np.float32)
    x = rng.normal(0.0, 1.0, k).astype(np.float32)
    x[32:64] = 0.0
    x[64:96] *= np.float32(1e-40)
    x[96:128] *= np.float32(1e30)
    x[130] = np.float32(3e-42)
    q = oracle_lib.quantize_rows(dt, w)
    d, c = oracle_lib.limb_partials(dt, q, n, k, x)
    assert c[1] == 0.0 and not d[:, 1].any()
    ints = (d.astype(np.int64) * np.array([1 << 24, 1 << 16, 1 << 8, 1], np.int64)).sum(-1)
    sc = _block_scales(dt, q, n, k)
    rec = (sc * c.astype(np.float64)[None, :] * ints).sum(1)
    y64 = oracle_lib.matvec_f64(dt, q, n, k, x)
    qmax = 127.0 if dt == 10 else 8.0
    bound = (np.abs(sc) * c.astype(np.float64)[None, :] * 0.5 * 32 * qmax).sum(1) * (1 + 1e-12) + 1e-300
    assert (np.abs(rec - y64) <= bound).all(), (np.abs(rec - y64) / bound).max()


def test_limb_partials_known_block(oracle_lib):
    """Block max 0.75 (t = 0.75 (1 + 2^-8) < 1, so e = 0, c = 2^-30 and X_i = rint(x_i 2^30))
    against codes all 1; every digit within [-128, 127]."""
    k = 32
    raw = np.zeros(36, np.uint8)
    raw[:4] = np.frombuffer(np.float32(1.0).tobytes(), np.uint8)
    raw[4:] = 1
    x = (np.arange(1, 33, dtype=np.float32) / np.float32(64.0)) * np.float32(0.98)
    x[-1] = np.float32(0.75)
    d, c = oracle_lib.limb_partials(10, raw, 1, k, x)
    assert c[0] == np.float32(2.0 ** -30)
    ints = int((d[0, 0].astype(np.int64) * np.array([1 << 24, 1 << 16, 1 << 8, 1])).sum())
    assert ints == int(sum(int(np.rint(float(v) * 2.0 ** 30)) for v in x))


@pytest.mark.skipif(not oracle.reference_available(), reason="oracle/_ref not built (no reference tree)")
def test_rms_norm_matches_the_reference(oracle_lib):
    """qo_rms_norm is ops::rms_norm_inplace (src/nn/ops.cpp:107-118) bit for bit."""
    ref = oracle.Reference()
    rng = np.random.default_rng(5)
    for size, scale, eps in ((2048, 1.0, 1e-6), (4096, 30.0, 1e-5), (8192, 1e-3, 1e-6), (37, 1.0, 0.0),
                             (28672, 5.0, 1e-6)):
        x = (rng.normal(size=size) * scale).astype(np.float32)
        w = rng.normal(1.0, 0.1, size=size).astype(np.float32)
        assert oracle_lib.rms_norm(x, w, eps).tobytes() == ref.rms_norm(x, w, eps).tobytes(), (size, eps)


def test_kv_int8_quantizer_is_the_reference():
    """The reference's QuantizedKVCache::store (include/nn/kv_cache_quant.h:61-94),
    restated: per head scale = max |x| / 127 (a NaN is never the max), codes
    clamp(round-half-away(x * (1 / scale)), -127, 127), 0 for an all-zero head."""
    import oracle

    if not oracle.reference_available():
        pytest.skip("oracle/_ref not built")
    rng = np.random.default_rng(21)
    kv_heads, hd = 4, 32
    k = rng.normal(0, 2, kv_heads * hd).astype(np.float32)
    v = rng.normal(0, 0.5, kv_heads * hd).astype(np.float32)
    k[hd:2 * hd] = 0.0                    # an all-zero head
    v[5] = np.nan                         # NaN is skipped by the max and clamps to 127
    k[3 * hd] = np.float32(0.5) * np.float32(np.abs(k[3 * hd + 1:4 * hd]).max())   # ordinary value
    kq, vq, ks, vs = oracle.Reference().kv_quantize(k, v, kv_heads, hd)

    def restate(x):
        codes, scales = np.empty(x.size, np.int8), np.empty(kv_heads, np.float32)
        for h in range(kv_heads):
            seg = x[h * hd:(h + 1) * hd]
            finite = seg[~np.isnan(seg)]
            mx = np.float32(np.abs(finite).max()) if finite.size else np.float32(0)
            sc = np.float32(mx / np.float32(127.0))
            inv = np.float32(np.float32(1.0) / sc) if sc > 0 else np.float32(0)
            prod = (seg * inv).astype(np.float32)
            r = np.where(np.isnan(prod), 127.0, np.sign(prod) * np.floor(np.abs(prod).astype(np.float64) + 0.5))
            codes[h * hd:(h + 1) * hd] = np.clip(r, -127, 127).astype(np.int8)
            scales[h] = sc
        return codes, scales

    want_kq, want_ks = restate(k)
    want_vq, want_vs = restate(v)
    assert np.array_equal(kq, want_kq) and np.array_equal(ks, want_ks)
    assert np.array_equal(vq, want_vq) and np.array_equal(vs, want_vs)
    assert (kq[hd:2 * hd] == 0).all() and ks[1] == 0 and vq[5] == 127
