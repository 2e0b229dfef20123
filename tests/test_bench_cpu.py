"""bench.py host logic on the CPU: workload names, the algorithmic byte counts the
roofline divides by, the launch count rule, and the reference arm's JSON line
(the driver's contract) on a small workload."""
from __future__ import annotations

import json
import os
import subprocess
import sys

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path.insert(0, ROOT)

import bench  # noqa: E402


def test_workload_names():
    assert bench.parse_workload("q4_4096x4096") == (bench.Q4, 4096, 4096, 1)
    assert bench.parse_workload("q8_11008x2048_m16") == (bench.Q8, 11008, 2048, 16)
    assert bench.parse_workload("q4_28672x8192_shard") == (bench.Q4, 28672, 8192, 1)
    assert bench.parse_workload("q4_28672x8192_m2_shard") == (bench.Q4, 28672, 8192, 2)
    assert bench.is_shard_workload("q4_28672x8192_shard")
    assert not bench.is_shard_workload("q4_4096x4096")
    assert bench.parse_token_workload("llama70b_token") == ("llama70b", 1)
    assert bench.parse_token_workload("qwen3b_token_m16") == ("qwen3b", 16)
    assert bench.parse_token_workload("q4_4096x4096") is None
    assert bench.resolve_workload(None, 1) == "q4_4096x4096"
    assert bench.resolve_workload(None, 8) == "q4_28672x8192_shard"       # the sharded 70B projection
    assert bench.resolve_workload("q8_4096x4096", 8) == "q8_4096x4096"


def test_algorithmic_bytes_match_the_measurement_plan():
    """Per-call bytes = weights + x + y (configs 1 and 2 of the measurement plan)."""
    assert bench.alg_bytes(bench.Q8, 4096, 4096, 1) == 18_907_136
    assert bench.alg_bytes(bench.Q4, 4096, 4096, 1) == 9_469_952
    # config 4, weights only: Q8 25,362,432 B and Q4 12,681,216 B for 11008 x 2048
    assert bench.alg_bytes(bench.Q8, 11008, 2048, 16) - 4 * 16 * (2048 + 11008) == 25_362_432
    assert bench.alg_bytes(bench.Q4, 2048, 11008, 16) - 4 * 16 * (2048 + 11008) == 12_681_216


def test_launch_count_rule():
    """The limb-prep kernel runs for rows of >= 320 blocks when a CTA gets <= 96 rows."""
    assert bench.launches_per_call(4096, 4096, 148) == 1        # 128 blocks per row
    assert bench.launches_per_call(10240, 8192, 148) == 1       # 256 blocks per row
    assert bench.launches_per_call(2048, 11008, 148) == 2       # 344 blocks per row
    assert bench.launches_per_call(8192, 28672, 148) == 2       # 896 blocks, 56 rows per CTA
    assert bench.launches_per_call(28672, 28672, 148) == 1      # 194 rows per CTA


def test_reference_arm_prints_the_contract_line():
    """The reference arm's line has every contract key and the same config as our
    arm, and the process never maps the product library (its inputs come from the
    reference library's own std::mt19937 draws)."""
    env = dict(os.environ, CUDA_VISIBLE_DEVICES="")
    code = ("import sys, runpy; sys.argv = ['bench.py', '--impl', 'reference', '--workload', 'q8_256x512', "
            "'--steps', '2', '--warmup', '1']; runpy.run_path('bench.py', run_name='__main__'); "
            "maps = open('/proc/self/maps').read(); print('PRODUCT_SO_MAPPED', 'libqraf_cuda' in maps)")
    out = subprocess.run([sys.executable, "-c", code], capture_output=True, text=True, env=env, timeout=300, cwd=ROOT)
    assert out.returncode == 0, out.stderr[-2000:]
    lines = [ln for ln in out.stdout.splitlines() if ln.startswith("{")]
    assert len(lines) == 1, out.stdout
    d = json.loads(lines[0])
    for key in ("impl", "metric", "value", "unit", "n_gpus", "steps", "warmup", "ms_per_step", "higher_is_better",
                "scaling", "vs_baseline", "dtype", "data", "config", "cpu_baseline", "e2e"):
        assert key in d, key
    assert d["impl"] == "reference" and d["metric"] == bench.METRIC and d["unit"] == "GB/s"
    assert d["value"] > 0 and d["higher_is_better"] is True
    assert d["cpu_baseline"]["kind"] in ("reference", "port") and d["cpu_baseline"]["cores"] >= 1
    assert d["e2e"] == {"value": d["value"], "unit": "GB/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}
    assert d["config"] == {"workload": "q8_256x512", "N": 256, "K": 512, "M": 1, "block": 32, "quant": "Q8_0",
                           "mode": "fast"}
    assert "PRODUCT_SO_MAPPED False" in out.stdout


def test_decode_workload_names_and_bytes():
    assert bench.parse_decode_workload("qwen3b_decode") == ("qwen3b", 1, 512, False)
    assert bench.parse_decode_workload("qwen3b_decode_m8_c1024") == ("qwen3b", 8, 1024, False)
    assert bench.parse_decode_workload("qwen3b_decode_c4096_kv8") == ("qwen3b", 1, 4096, True)
    total8, _ = bench.decode_bytes_per_step("qwen3b", 1, 512, kv8=True)
    # 513 positions read + 1 written per layer: 2 x 4 x 256 bytes each in f32, 2 x (256 + 2 x 4) in int8
    assert total8 == bench.decode_bytes_per_step("qwen3b", 1, 512)[0] - 514 * 36 * (2 * 4 * 256 - 2 * (256 + 2 * 4))
    assert bench.parse_decode_workload("qwen3b_token") is None
    total, weights = bench.decode_bytes_per_step("qwen3b", 1, 512)
    # 36 layers of Q8_0 projections (q, k, v, o, gate, up, down) + the 151936 x 2048 head
    assert weights == 36 * (2048 * 2048 * 2 + 256 * 2048 * 2 + 11008 * 2048 * 3) * 36 // 32 + 151936 * 64 * 36
    kv = 36 * 513 * 256 * 4 * 2 + 36 * 256 * 4 * 2
    small = 4 * (73 * 2048 + 36 * (2048 + 512))
    assert total == weights + kv + small + 2048 * 4


def test_decode_file_runs_in_the_reference_transformer(tmp_path, monkeypatch):
    """The bench's model file (a smaller model of the same layout) loads in the
    reference's Transformer and decodes: the CPU baseline's path."""
    import numpy as np

    import oracle

    if not oracle.reference_available():
        import pytest

        pytest.skip("oracle/_ref not built")
    monkeypatch.setitem(bench.TOKEN_MODELS, "tiny", {"dtype": bench.Q4, "layers": 2, "hidden": 256, "vocab": 300,
                                                     "projs": []})
    monkeypatch.setitem(bench.DECODE_MODELS, "tiny", {"arch": "qwen2", "heads": 4, "kv_heads": 2, "inter": 512})
    ref = oracle.Reference()
    path = str(tmp_path / "tiny.qraf")
    n = bench.write_decode_file("tiny", path, lambda seed, std, k: bench.host_normal(seed, std, k),
                                lambda dt, w: ref.quantize(dt, np.ascontiguousarray(w).reshape(-1), 32), max_seq=9)
    assert n == os.path.getsize(path)
    cpu = bench.decode_cpu_baseline("tiny", 8, 0.05, path)
    assert cpu["kind"] == "reference" and cpu["value"] > 0


def test_sharded_call_kernel_count():
    """A sharded call's kernels: the tile pair per 64 vectors in TC (AUTO from three
    vectors), the row kernel in pairs of vectors in FAST (with the limb prep for
    long K and few rows per CTA), one launch in EXACT."""
    import bench

    assert bench.shard_call_kernels("auto", 14336, 8192, 16, 148) == ("qmm_tc_kernel", 2)
    assert bench.shard_call_kernels("tc", 14336, 8192, 70, 148) == ("qmm_tc_kernel", 4)
    assert bench.shard_call_kernels("auto", 14336, 8192, 2, 148) == ("qmv_rows_kernel", 1)   # 97 rows per CTA
    assert bench.shard_call_kernels("fast", 14336, 8192, 5, 148) == ("qmv_rows_kernel", 3)
    assert bench.shard_call_kernels("fast", 7168, 28672, 5, 148) == ("qmv_rows_kernel", 6)   # 49 rows: limb prep
    assert bench.shard_call_kernels("fast", 3584, 28672, 1, 148) == ("qmv_rows_kernel", 2)
    assert bench.shard_call_kernels("exact", 14336, 8192, 4, 148) == ("qmv_rows_kernel", 1)
