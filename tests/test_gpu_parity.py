"""GPU parity: the sm_100a kernels against the oracle's and the reference's outputs.

Bar: quantized payloads bit-exact; EXACT mode output
bit-exact; FAST mode within allclose(rtol=1e-5, atol=1e-6) of the reference's
fp32 result wherever the reference itself is that close to the exact value
(see assert_fast_ok).  Every call goes through the C ABI of libqraf_cuda.so.
"""
from __future__ import annotations

import ctypes as C
import hashlib
import os

import numpy as np
import pytest

import qraf_b200 as qb
from conftest import GOLDEN

pytestmark = pytest.mark.gpu

RTOL, ATOL = 1e-5, 1e-6


def assert_fast_ok(y, y_ref, y64, label):
    """FAST / TC bar.  Every output is within allclose(RTOL, ATOL) of the
    reference's result, or no farther from the fp64 value of the same dequantized
    product than the reference's own worst error on that tensor (plus RTOL
    relative).  At long K the reference's serial fp32 chains miss the fp64 value
    by more than ATOL on some near-zero outputs, and any fp32 sum in another
    order carries rounding noise of the same size, so no such sum can stay
    inside ATOL of the reference there: EXACT mode is the bit-identical one."""
    y = np.asarray(y, np.float64)
    y_ref = np.asarray(y_ref, np.float64)
    ref_err = float(np.max(np.abs(y_ref - y64))) if y64.size else 0.0
    close = np.abs(y - y_ref) <= ATOL + RTOL * np.abs(y_ref)
    bounded = np.abs(y - y64) <= ref_err + RTOL * np.abs(y64)
    bad = ~(close | bounded)
    assert not bad.any(), (f"{label}: {int(bad.sum())} outputs outside allclose of the reference and beyond the "
                           f"reference's own worst error {ref_err:.3g}; worst |d|={np.abs(y - y_ref)[bad].max():.3g}")


def sha(a):
    return hashlib.sha256(np.ascontiguousarray(a).tobytes()).hexdigest()


def to_dev(a, torch, dev):
    return torch.from_numpy(np.ascontiguousarray(a)).to(dev)


# ── quantizer ────────────────────────────────────────────────────────────
def test_quantizer_small_cases_byte_exact(cuda, small_cases):
    import torch

    n_checked = 0
    for i, c in enumerate(small_cases):
        if "w" not in c:
            continue
        w = to_dev(c["w"], torch, cuda)
        q = qb.quantize_rows(c["dtype"], w, c["bs"]).cpu().numpy()
        assert q.tobytes() == c["q"].tobytes(), f"case {i}"
        n_checked += 1
    assert n_checked >= 10


def test_reference_unit_cases_on_gpu(cuda):
    import torch

    u = np.load(os.path.join(GOLDEN, "ref_unit_cases.npz"))
    data = to_dev(u["data"], torch, cuda)
    assert qb.quantize(qb.Q8_0, data, 8).cpu().numpy().tobytes() == u["q8"].tobytes()
    assert qb.quantize(qb.Q4_0, data, 8).cpu().numpy().tobytes() == u["q4"].tobytes()
    d8 = qb.dequantize(qb.Q8_0, to_dev(u["q8"], torch, cuda), 8, 8).cpu().numpy()
    d4 = qb.dequantize(qb.Q4_0, to_dev(u["q4"], torch, cuda), 8, 8).cpu().numpy()
    assert d8.tobytes() == u["q8_deq"].tobytes() and d4.tobytes() == u["q4_deq"].tobytes()
    r = qb.dot_q8_0_f32(to_dev(u["dot_q8"], torch, cuda), to_dev(u["dot_b"], torch, cuda), 4, 4).cpu().numpy()
    assert r.tobytes() == u["dot_result"].tobytes()
    assert abs(float(r[0]) - 5.0) <= 0.1


def test_quantizer_special_values(cuda, oracle_lib):
    import torch

    vals = [np.nan, np.inf, -np.inf, 0.0, -0.0, 1e-40, 6e-5, 65504.0, 7e4, -3e-8, 1e30, -1e-30]
    for dt in (qb.Q8_0, qb.Q4_0):
        for v in vals:
            w = np.full(32, v, dtype=np.float32)
            w[3], w[9] = 0.5, -0.25
            q = qb.quantize(dt, to_dev(w, torch, cuda)).cpu().numpy()
            assert q.tobytes() == oracle_lib.quantize(dt, w).tobytes(), (dt, v)
    # ragged and odd block sizes
    rng = np.random.default_rng(3)
    for dt in (qb.Q8_0, qb.Q4_0):
        for bs, count in [(32, 33), (7, 50), (5, 23), (64, 1000), (3, 2), (32, 1)]:
            x = rng.standard_normal(count).astype(np.float32)
            q = qb.quantize(dt, to_dev(x, torch, cuda), bs).cpu().numpy()
            assert q.tobytes() == oracle_lib.quantize(dt, x, bs).tobytes(), (dt, bs, count)
            deq = qb.dequantize(dt, to_dev(q, torch, cuda), count, bs).cpu().numpy()
            want = np.zeros(count, np.float32)
            nb = (count + bs - 1) // bs
            bb = 4 + bs if dt == qb.Q8_0 else 2 + bs // 2
            for b in range(nb):
                n = min(bs, count - b * bs)
                blk = oracle_lib.dequantize_block(dt, q[b * bb:(b + 1) * bb], bs)
                m = n if dt == qb.Q8_0 else 2 * (n // 2)
                want[b * bs:b * bs + m] = blk[:m]
            assert deq.tobytes() == want.tobytes(), (dt, bs, count)


# ── matvec on the golden small cases ─────────────────────────────────────
def test_matvec_exact_small_cases(cuda, small_cases):
    import torch

    for i, c in enumerate(small_cases):
        w = qb.Weight.from_device(to_dev(c["q"], torch, cuda).reshape(-1), c["dtype"], c["n"], c["k"], c["bs"])
        x = to_dev(c["x"], torch, cuda)
        y = qb.matvec_q(w, x, mode=qb.MODE_EXACT).cpu().numpy()
        assert y.tobytes() == c["y"].tobytes(), f"case {i} ({c['dtype']}, bs={c['bs']}, {c['n']}x{c['k']}, M={c['m']})"


def test_matvec_fast_small_cases(cuda, small_cases, oracle_lib):
    import torch

    for i, c in enumerate(small_cases):
        w = qb.Weight.from_device(to_dev(c["q"], torch, cuda).reshape(-1), c["dtype"], c["n"], c["k"], c["bs"])
        x = to_dev(c["x"], torch, cuda)
        y = qb.matvec_q(w, x, mode=qb.MODE_FAST).cpu().numpy()
        y64 = np.stack([oracle_lib.matvec_f64(c["dtype"], c["q"], c["n"], c["k"], c["x"][j], c["bs"])
                        for j in range(c["m"])])
        assert_fast_ok(y, c["y"], y64, f"case {i}")


def test_overlap_flag_gives_identical_results(cuda, small_cases):
    import torch

    for i, c in enumerate(small_cases):
        w = qb.Weight.from_device(to_dev(c["q"], torch, cuda).reshape(-1), c["dtype"], c["n"], c["k"], c["bs"])
        x = to_dev(c["x"], torch, cuda)
        for mode in (qb.MODE_EXACT, qb.MODE_FAST):
            a = qb.matvec_q(w, x, mode=mode).cpu().numpy()
            # several launches back to back so that overlapped launches actually overlap
            outs = [qb.matvec_q(w, x, mode=mode | qb.MODE_FLAG_OVERLAP) for _ in range(4)]
            for o in outs:
                assert o.cpu().numpy().tobytes() == a.tobytes(), f"case {i} mode {mode}"


def test_block_partials_bit_exact(cuda, small_cases):
    import torch

    for i, c in enumerate(small_cases):
        w = qb.Weight.from_device(to_dev(c["q"], torch, cuda).reshape(-1), c["dtype"], c["n"], c["k"], c["bs"])
        p = qb.block_partials(w, to_dev(c["x"][0], torch, cuda)).cpu().numpy()
        assert p.tobytes() == c["partials"].tobytes(), f"case {i}"


@pytest.mark.parametrize("dt", [qb.Q8_0, qb.Q4_0])
@pytest.mark.parametrize("n,k", [(64, 4096), (8, 28672), (300, 2048)])
def test_limb_partials_bit_exact(cuda, oracle_lib, dt, n, k):
    """The FAST kernels' per-block integer partial sums D_j (and the block factors)
    equal the oracle's integer restatement bit for bit, on ordinary blocks and on
    blocks of zeros, tiny (subnormal-range), huge and non-finite values."""
    import torch

    wf = torch.from_numpy(qb.fill_normal(42, 0.0, 0.02, n * k)).to(cuda).reshape(n, k)
    q = qb.quantize_rows(dt, wf).reshape(-1)
    w = qb.Weight.from_device(q, dt, n, k)
    x = qb.fill_normal(43, 0.0, 1.0, k)
    x[32:64] = 0.0
    x[64:96] *= np.float32(1e-40)
    x[96:128] *= np.float32(1e30)
    x[130] = np.float32(3e-42)
    x[200] = np.float32("nan")
    x[290] = np.float32("inf")
    d, c = qb.limb_partials(w, torch.from_numpy(x).to(cuda))
    d_ref, c_ref = oracle_lib.limb_partials(dt, q.cpu().numpy(), n, k, x)
    assert np.array_equal(d.cpu().numpy(), d_ref)
    assert np.array_equal(c.cpu().numpy(), c_ref, equal_nan=True)
    assert qb.device_status() == qb.OK


def test_unaligned_pointers_take_the_generic_path(cuda, small_cases):
    import torch

    c = next(c for c in small_cases if c["k"] == 4096)
    raw = torch.zeros(c["q"].size + 16, dtype=torch.uint8, device=cuda)
    raw[4:4 + c["q"].size] = to_dev(c["q"].reshape(-1), torch, cuda)
    w = qb.Weight.from_device(raw[4:4 + c["q"].size], c["dtype"], c["n"], c["k"], c["bs"])
    xr = torch.zeros(c["k"] + 4, dtype=torch.float32, device=cuda)
    xr[1:1 + c["k"]] = to_dev(c["x"][0], torch, cuda)
    y = qb.matvec_q(w, xr[1:1 + c["k"]], mode=qb.MODE_EXACT).cpu().numpy()
    assert y.tobytes() == c["y"][0].tobytes()


def test_empty_shapes(cuda):
    import torch

    q = torch.zeros(64, dtype=torch.uint8, device=cuda)
    w = qb.Weight.from_device(q, qb.Q8_0, 0, 32)
    y = torch.full((1, 0), 5.0, device=cuda)
    qb.matvec_q(w, torch.ones(32, device=cuda), y=y)
    w = qb.Weight.from_device(q, qb.Q8_0, 3, 0)
    y = torch.full((1, 3), 5.0, device=cuda)
    qb.matvec_q(w, torch.ones(4, device=cuda)[:0].reshape(1, 0).contiguous(), y=y, mode=qb.MODE_EXACT)
    assert torch.all(y == 0)


def test_errors_are_reported(cuda):
    import torch

    q = torch.zeros(36 * 4, dtype=torch.uint8, device=cuda)
    w = qb.Weight.from_device(q, qb.Q8_0, 4, 32)
    with pytest.raises(qb.QrafError) as e:
        qb.matvec_q(w, torch.ones(32, device=cuda), mode=7)
    assert e.value.code == qb.ERR_INVALID
    with pytest.raises(qb.QrafError):
        qb.Weight.from_device(q[:100], qb.Q8_0, 4, 32)


# ── the host-pointer drop-in entry ────────────────────────────────────────
def test_host_entry_matches_reference(cuda, small_cases, oracle_lib):
    for i, c in enumerate(small_cases):
        q = np.ascontiguousarray(c["q"]).reshape(-1)
        for mode in (qb.MODE_EXACT, qb.MODE_FAST):
            y = np.zeros((c["m"], c["n"]), np.float32)
            qb.dispatch_matvec_q(q, q.size, c["dtype"], c["bs"], c["n"], c["k"], np.ascontiguousarray(c["x"]), y,
                                 m=c["m"], mode=mode)
            if mode == qb.MODE_EXACT:
                assert y.tobytes() == c["y"].tobytes(), f"case {i}"
            else:
                y64 = np.stack([oracle_lib.matvec_f64(c["dtype"], c["q"], c["n"], c["k"], c["x"][j], c["bs"])
                                for j in range(c["m"])])
                assert_fast_ok(y, c["y"], y64, f"host case {i}")
    qb.host_cache_clear()


def test_host_entry_repeated_calls(cuda, oracle_lib):
    """Repeated host-entry calls with one weight replay a cached graph of the call's
    device work: every call still reads its own x and returns its own exact result,
    for the row kernel, the long-K path with limb prep, and the tensor cores."""
    for dt, n, k, m, mode in [(qb.Q8_0, 512, 4096, 1, qb.MODE_EXACT), (qb.Q4_0, 96, 28672, 1, qb.MODE_FAST),
                              (qb.Q8_0, 640, 2048, 20, qb.MODE_TC)]:
        w = qb.fill_normal(42, 0.0, 0.02, n * k).reshape(n, k)
        q = oracle_lib.quantize_rows(dt, w).reshape(-1)
        for call in range(4):
            x = qb.fill_normal(100 + call, 0.0, 1.0, m * k).reshape(m, k)
            y = np.zeros((m, n), np.float32)
            qb.dispatch_matvec_q(q, q.size, dt, 32, n, k, x, y, m=m, mode=mode)
            y_ref = np.stack([oracle_lib.matvec(dt, q, n, k, x[j]) for j in range(m)])
            if mode == qb.MODE_EXACT:
                assert y.tobytes() == y_ref.tobytes(), f"call {call}"
            else:
                y64 = np.stack([oracle_lib.matvec_f64(dt, q, n, k, x[j]) for j in range(m)])
                assert_fast_ok(y, y_ref, y64, f"dt={dt} mode={mode} call {call}")
    qb.host_cache_clear()
    assert qb.device_status() == qb.OK


def _host_check(oracle_lib, dt, q, n, k, x, y, mode, label):
    m = x.shape[0]
    y_ref = np.stack([oracle_lib.matvec(dt, q, n, k, x[j]) for j in range(m)])
    if mode == qb.MODE_EXACT:
        assert y.tobytes() == y_ref.tobytes(), label
    else:
        y64 = np.stack([oracle_lib.matvec_f64(dt, q, n, k, x[j]) for j in range(m)])
        assert_fast_ok(y, y_ref, y64, label)


def test_host_entry_shapes_that_grow_the_scratch(cuda, oracle_lib):
    """The host entry replays a cached CUDA graph per (weight, M, mode), and those
    graphs hold the stream's scratch address.  A later call that needs more scratch
    must not free memory an earlier graph still writes: the 70B sequence QKV
    (10240 x 8192, activation limbs in scratch) -> down (8192 x 28672, more
    scratch) -> QKV again, then on the tensor cores M = 16 on a small weight ->
    M = 64 on a large one -> M = 16 on the small one again; every call against the
    oracle, twice per step so that the second call of a step replays its graph."""
    seq = [("qkv", qb.Q4_0, 10240, 8192, 1, qb.MODE_FAST), ("down", qb.Q4_0, 8192, 28672, 1, qb.MODE_FAST),
           ("qkv", qb.Q4_0, 10240, 8192, 1, qb.MODE_FAST),
           ("small", qb.Q8_0, 640, 2048, 16, qb.MODE_TC), ("large", qb.Q4_0, 4096, 8192, 64, qb.MODE_TC),
           ("small", qb.Q8_0, 640, 2048, 16, qb.MODE_TC)]
    weights = {}
    for step, (name, dt, n, k, m, mode) in enumerate(seq):
        if name not in weights:
            w = qb.fill_normal(42, 0.0, 0.02, n * k).reshape(n, k)
            weights[name] = oracle_lib.quantize_rows(dt, w).reshape(-1)
        q = weights[name]
        for call in range(2):
            x = qb.fill_normal(100 + 10 * step + call, 0.0, 1.0, m * k).reshape(m, k)
            y = np.zeros((m, n), np.float32)
            qb.dispatch_matvec_q(q, q.size, dt, 32, n, k, x, y, m=m, mode=mode)
            _host_check(oracle_lib, dt, q, n, k, x, y, mode, f"step {step} ({name}) call {call}")
    qb.host_cache_clear()
    assert qb.device_status() == qb.OK


def test_host_entry_reports_an_expired_device_wait(cuda, oracle_lib):
    """The host entry reads the device's status word with the copy of y: a bounded
    wait that ran out on the device (here: a 2-rank fused all-gather with no second
    rank, a flag nothing sets) comes back as QRAF_ERR_TIMEOUT from the next host
    call instead of a silently incomplete y; the word is taken, so the call after
    that is clean again."""
    import torch

    n, k = 256, 1024
    qd = torch.from_numpy(oracle_lib.quantize_rows(qb.Q8_0, qb.fill_normal(7, 0.0, 0.02, n * k).reshape(n, k)))
    full = qb.Weight.from_device(qd.to(cuda).reshape(-1), qb.Q8_0, n, k)
    c0, c1 = qb.Comm(2, 0, n), qb.Comm(2, 1, n)
    qb.Comm.open_local([c0, c1])
    c0.matvec_q(full.shard(2, 0), n, 0, torch.ones(k, device=cuda), mode=qb.MODE_EXACT)
    torch.cuda.synchronize()
    q = qd.numpy().reshape(-1)
    x = qb.fill_normal(8, 0.0, 1.0, k).reshape(1, k)
    y = np.zeros((1, n), np.float32)
    with pytest.raises(qb.QrafError) as e:
        qb.dispatch_matvec_q(q, q.size, qb.Q8_0, 32, n, k, x, y, m=1, mode=qb.MODE_EXACT)
    assert e.value.code == qb.ERR_TIMEOUT
    qb.dispatch_matvec_q(q, q.size, qb.Q8_0, 32, n, k, x, y, m=1, mode=qb.MODE_EXACT)
    _host_check(oracle_lib, qb.Q8_0, q, n, k, x, y, qb.MODE_EXACT, "after the reported timeout")
    assert qb.device_status() == qb.OK
    qb.host_cache_clear()
    c0.destroy()
    c1.destroy()


# ── full-size configurations ──────────────────
_W_CACHE = {}
_Q_HOST = {}


def weight_for(name, d, torch, dev):
    """Quantize the config's seeded weight on the GPU and check its digest."""
    if name in _W_CACHE:
        return _W_CACHE[name]
    _W_CACHE.clear()
    wf = qb.fill_normal(d["seed_w"], 0.0, 0.02, d["n"] * d["k"])
    wd = torch.from_numpy(wf).to(dev).reshape(d["n"], d["k"])
    del wf
    q = qb.quantize_rows(d["dtype"], wd, d["block_size"])
    del wd
    q_host = q.cpu().numpy()
    assert sha(q_host) == d["sha_q"], f"{name}: quantized payload differs from the reference"
    _Q_HOST.clear()
    _Q_HOST[name] = q_host.reshape(-1)
    w = qb.Weight.from_device(q.reshape(-1), d["dtype"], d["n"], d["k"], d["block_size"])
    _W_CACHE[name] = w
    return w


def config_names(digests):
    """Every BASELINE configuration shape, the two LM heads (151936 x 2048 Q8_0,
    128256 x 8192 Q4_0) included."""
    return sorted(digests)


# Outputs outside strict allclose(RTOL, ATOL) of the reference, per (config, M,
# mode): printed at the end of the session, written as JSON where
# QRAF_PARITY_REPORT names a file.  Configurations 1 and 2 (4096 x 4096) must
# have none.
STRICT_MISSES = {}
STRICT_REQUIRED = ("cfg1_q8_4096x4096", "cfg2_q4_4096x4096")


def strict_misses(y, y_ref):
    y, y_ref = np.asarray(y, np.float64), np.asarray(y_ref, np.float64)
    return int((np.abs(y - y_ref) > ATOL + RTOL * np.abs(y_ref)).sum())


@pytest.fixture(scope="module", autouse=True)
def _strict_report():
    yield
    if not STRICT_MISSES:
        return
    import json

    print("\nstrict allclose(1e-5, 1e-6) misses per config, M and mode (outputs):")
    for key, v in sorted(STRICT_MISSES.items()):
        print(f"  {key}: {v['misses']} of {v['outputs']}")
    path = os.environ.get("QRAF_PARITY_REPORT")
    if path:
        with open(path, "w") as f:
            json.dump(STRICT_MISSES, f, indent=1, sort_keys=True)


def pytest_generate_tests(metafunc):
    if "config_name" in metafunc.fixturenames:
        from conftest import load_digests

        metafunc.parametrize("config_name", config_names(load_digests()))


def test_config_exact_and_fast(cuda, digests, config_name, oracle_lib):
    import torch

    d = digests[config_name]
    w = weight_for(config_name, d, torch, cuda)
    q_host = np.ascontiguousarray(_Q_HOST[config_name])
    mmax = max(int(m) for m in d["y"])
    xall = torch.from_numpy(qb.fill_normal(d["seed_x"], 0.0, 1.0, mmax * d["k"])).to(cuda).reshape(mmax, d["k"])
    ys = np.load(os.path.join(GOLDEN, "config_y.npz"))
    for ms, digest in d["y"].items():
        m = int(ms)
        y_exact = qb.matvec_q(w, xall[:m].contiguous(), mode=qb.MODE_EXACT).cpu().numpy()
        assert sha(y_exact) == digest, f"{config_name} M={m}: EXACT output differs from the reference"
        y_fast = qb.matvec_q(w, xall[:m].contiguous(), mode=qb.MODE_FAST).cpu().numpy()
        xh = xall[:m].cpu().numpy()
        y64 = np.stack([oracle_lib.matvec_f64(d["dtype"], q_host, d["n"], d["k"], xh[j]) for j in range(m)])
        assert_fast_ok(y_fast, y_exact, y64, f"{config_name} M={m}")
        STRICT_MISSES[f"{config_name} M={m} FAST"] = {"misses": strict_misses(y_fast, y_exact), "outputs": y_fast.size}
        if config_name in STRICT_REQUIRED:
            assert STRICT_MISSES[f"{config_name} M={m} FAST"]["misses"] == 0, f"{config_name}: FAST not strictly close"
        if d["k"] % (256 if d["dtype"] == qb.Q4_0 else 128) == 0:
            y_tc = qb.matvec_q(w, xall[:m].contiguous(), mode=qb.MODE_TC).cpu().numpy()
            assert_fast_ok(y_tc, y_exact, y64, f"{config_name} M={m} tensor cores")
            STRICT_MISSES[f"{config_name} M={m} TC"] = {"misses": strict_misses(y_tc, y_exact), "outputs": y_tc.size}
        if m == 1 and config_name in ys.files:
            assert y_exact[0].tobytes() == ys[config_name].tobytes()
    assert qb.device_status() == qb.OK


# ── several projections of one input in one launch ───────────────────────
@pytest.mark.parametrize("dt,rows,k", [
    (qb.Q8_0, (2048, 256, 256), 2048),      # Qwen2-3B Q, K, V (config 3)
    (qb.Q4_0, (3000, 3000), 4096),          # gate and up
    (qb.Q4_0, (5, 3, 7, 1), 8192),          # tiny weights: stages span several of them
    (qb.Q4_0, (640, 700), 28672),           # long rows: pieces of K, limb prep
])
def test_multi_weight_launch_equals_separate_calls(cuda, dt, rows, k):
    """qraf_cuda_matvec_q_multi gives the bits of one qraf_cuda_matvec_q call per
    weight, in EXACT (1 and 3 vectors), FAST (1 and 2) and TC (1: the batch-1
    tensor-core kernel, fused where all rows fit one wave, else weight by weight)."""
    import torch

    ws = []
    for i, n in enumerate(rows):
        wf = torch.from_numpy(qb.fill_normal(42 + i, 0.0, 0.02, n * k)).to(cuda).reshape(n, k)
        ws.append(qb.Weight.from_device(qb.quantize_rows(dt, wf).reshape(-1), dt, n, k))
    for mode, ms in ((qb.MODE_EXACT, (1, 3)), (qb.MODE_FAST, (1, 2)), (qb.MODE_TC, (1,))):
        for m in ms:
            x = torch.from_numpy(qb.fill_normal(50 + m, 0.0, 1.0, m * k)).to(cuda).reshape(m, k)
            got = qb.matvec_q_multi(ws, x, mode=mode)
            for i, w in enumerate(ws):
                want = qb.matvec_q(w, x, mode=mode)
                assert got[i].cpu().numpy().tobytes() == want.cpu().numpy().tobytes(), f"mode {mode} M={m} weight {i}"
    assert qb.device_status() == qb.OK
