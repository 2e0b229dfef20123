"""Generate the golden fixtures from the reference's OWN compiled code.

Run in a container that has the reference tree (it builds oracle/_ref first):

    python tests/golden/make_golden.py            # small cases + unit cases + config digests
    python tests/golden/make_golden.py --skip-big # without the 70B LM-head digest

Outputs (committed):
  ref_unit_cases.npz   the reference's own test_quantize.cpp cases (tests/test_quantize.cpp:7-50)
                       evaluated by the reference code: bytes, dequantized values, dot result
  small_cases.npz      seeded small matvec cases (many block sizes, ragged K, specials):
                       fp32 weight, quantized bytes, x, y = dispatch_matvec_q(...) per vector,
                       and the per-block partial products
  config_digests.json  for every BASELINE.json configuration shape: seeds, the SHA-256 of the
                       reference quantizer's bytes and of dispatch_matvec_q's output
  config_y.npz         the reference's y for the M = 1 configuration shapes (fast-mode tolerance)

Inputs: W ~ N(0, 0.02) from std::mt19937(42) drawn row-major [N][K] and X ~ N(0, 1) from
std::mt19937(43) drawn row-major [M][K], both with std::normal_distribution<float>.
"""
from __future__ import annotations

import argparse
import hashlib
import json
import os
import sys
import time

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, ROOT)

import oracle  # noqa: E402

Q8, Q4 = oracle.Q8_0, oracle.Q4_0
SEED_W, SEED_X = 42, 43

# (dtype, N, K, M list) — BASELINE.json configs 1-5, expanded to (out, in) shapes.
CONFIGS = [
    ("cfg1_q8_4096x4096", Q8, 4096, 4096, [1]),
    ("cfg2_q4_4096x4096", Q4, 4096, 4096, [1]),
    ("cfg3_q8_qo", Q8, 2048, 2048, [1]),
    ("cfg3_q8_kv", Q8, 256, 2048, [1]),
    ("cfg3_q8_gate_up", Q8, 11008, 2048, [1]),
    ("cfg3_q8_down", Q8, 2048, 11008, [1]),
    ("cfg3_q8_lm_head", Q8, 151936, 2048, [1]),
    ("cfg4_q8_11008x2048", Q8, 11008, 2048, [1, 4, 16, 32, 64]),
    ("cfg4_q8_2048x11008", Q8, 2048, 11008, [1, 4, 16, 32, 64]),
    ("cfg4_q4_11008x2048", Q4, 11008, 2048, [1, 4, 16, 32, 64]),
    ("cfg4_q4_2048x11008", Q4, 2048, 11008, [1, 4, 16, 32, 64]),
    ("cfg5_q4_gate_up", Q4, 28672, 8192, [1, 32]),
    ("cfg5_q4_down", Q4, 8192, 28672, [1, 32]),
    ("cfg5_q4_qkv", Q4, 10240, 8192, [1, 32]),
    ("cfg5_q4_lm_head", Q4, 128256, 8192, [1]),
]


def sha(a: np.ndarray) -> str:
    return hashlib.sha256(np.ascontiguousarray(a).tobytes()).hexdigest()


def small_cases(ref: oracle.Reference, orc: oracle.Oracle):
    rng = np.random.default_rng(2024)
    cases = []
    shapes = [
        # (dtype, bs, N, K, M)
        *[(dt, 32, n, k, m) for dt in (Q8, Q4) for (n, k, m) in [
            (1, 32, 1), (7, 64, 1), (33, 96, 2), (5, 33, 1), (3, 1, 1), (24, 4096, 1), (37, 256, 3),
            (6, 11008, 1), (96, 2048, 3), (150, 512, 16), (41, 1024, 2), (4, 8192, 5), (2, 28672, 1)]],
        (Q8, 8, 7, 64, 1), (Q4, 8, 7, 64, 1), (Q8, 4, 3, 12, 2), (Q4, 4, 3, 12, 2),
        (Q4, 7, 5, 50, 1), (Q8, 7, 5, 50, 1), (Q8, 64, 4, 200, 1), (Q4, 64, 4, 200, 1),
        (Q4, 5, 6, 23, 1), (Q8, 1, 4, 9, 1), (Q4, 2, 4, 9, 1), (Q8, 33, 3, 100, 1), (Q4, 33, 3, 100, 1),
    ]
    for i, (dt, bs, n, k, m) in enumerate(shapes):
        w = (rng.standard_normal((n, k)) * 0.02).astype(np.float32)
        x = rng.standard_normal((m, k)).astype(np.float32)
        if i % 3 == 0 and n * k > 40:   # specials: a zero block, huge, tiny and negative-zero values
            flat = w.ravel()
            flat[: min(bs, flat.size)] = 0.0
            flat[min(flat.size - 1, bs + 1)] = 3.0e4
            flat[min(flat.size - 1, bs + 5)] = -1.0e-30
            flat[min(flat.size - 1, bs + 6)] = -0.0
            x.ravel()[:: max(1, k // 7)] = 0.0
        q = ref.quantize_rows(dt, w, bs)
        y = np.stack([ref.matvec(dt, q, n, k, x[j], bs) for j in range(m)])
        y_or = orc.matmul(dt, q, n, k, x, bs)
        assert y.tobytes() == y_or.tobytes(), f"oracle disagrees with reference on case {i}"
        part = orc.block_partials(dt, q, n, k, x[0], bs)
        c = dict(dtype=dt, bs=bs, n=n, k=k, m=m, q=q, x=x, y=y, partials=part)
        if n * k <= 16384:      # keep the fixture small: fp32 weights only where the quantizer is pinned
            c["w"] = w
        cases.append(c)
    return cases


def unit_cases(ref: oracle.Reference):
    data = np.array([1.0, -0.5, 0.3, -1.0, 0.7, -0.2, 0.1, 0.9], dtype=np.float32)
    q8 = ref.quantize(Q8, data, 8)
    q4 = ref.quantize(Q4, data, 8)
    a = np.array([1.0, 2.0, 3.0, 4.0], dtype=np.float32)
    b = np.full(4, 0.5, dtype=np.float32)
    qa = ref.quantize(Q8, a, 4)
    return dict(
        data=data, q8=q8, q8_deq=ref.dequantize_block(Q8, q8, 8), q4=q4, q4_deq=ref.dequantize_block(Q4, q4, 8),
        dot_a=a, dot_b=b, dot_q8=qa, dot_result=np.array([ref.dot(Q8, qa, b, 4, 4)], dtype=np.float32))


def config_digests(ref: oracle.Reference, skip_big: bool):
    out, ys = {}, {}
    for name, dt, n, k, ms in CONFIGS:
        if skip_big and n * k > 400_000_000:
            continue
        t0 = time.time()
        w = ref.fill_normal(SEED_W, 0.0, 0.02, n * k)
        q = ref.quantize(dt, w, 32)          # K % 32 == 0: identical to per-row quantization
        del w
        mmax = max(ms)
        xall = ref.fill_normal(SEED_X, 0.0, 1.0, mmax * k).reshape(mmax, k)
        entry = dict(dtype=int(dt), n=n, k=k, block_size=32, seed_w=SEED_W, seed_x=SEED_X,
                     w_bytes=int(q.size), sha_q=sha(q), y={})
        threads = os.cpu_count() or 1
        for m in ms:
            y = np.stack([ref.matvec(dt, q, n, k, xall[j], 32, threads=threads) for j in range(m)])
            entry["y"][str(m)] = sha(y)
            if m == 1 and n <= 32768:
                ys[name] = y[0]
        out[name] = entry
        print(f"{name}: {time.time() - t0:.1f}s", flush=True)
    return out, ys


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--skip-big", action="store_true")
    args = ap.parse_args()
    oracle.build(with_ref=True)
    ref, orc = oracle.Reference(), oracle.Oracle()

    u = unit_cases(ref)
    np.savez_compressed(os.path.join(HERE, "ref_unit_cases.npz"), **u)

    cases = small_cases(ref, orc)
    flat = {}
    for i, c in enumerate(cases):
        for key, v in c.items():
            flat[f"c{i}_{key}"] = np.asarray(v)
    flat["ncases"] = np.array(len(cases))
    np.savez_compressed(os.path.join(HERE, "small_cases.npz"), **flat)

    dig, ys = config_digests(ref, args.skip_big)
    with open(os.path.join(HERE, "config_digests.json"), "w") as f:
        json.dump(dig, f, indent=1, sort_keys=True)
    np.savez_compressed(os.path.join(HERE, "config_y.npz"), **ys)


if __name__ == "__main__":
    main()
