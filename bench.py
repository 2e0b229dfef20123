#!/usr/bin/env python
"""bench.py — QRAF's quantized matvec on B200 (BASELINE.json metric: "Q8/Q4 matvec HBM GB/s").

Default workload on one GPU: BASELINE.json configs[1], the Q4_0 4096x4096
batch-1 matvec.  Weight W ~ N(0, 0.02) from std::mt19937(42) (the reference's
seeding idiom), quantized on the GPU by the byte-exact Q4_0 quantizer;
activation x ~ N(0, 1) from std::mt19937(43).

A STEP is one pass over a pool of R distinct copies of the quantized weight
(R = ceil(4 x L2 / weight bytes)), one matvec launch per copy: every launch
reads its weight cold from HBM (inputs larger than L2, so no flush is needed).
The step is captured once as a CUDA graph and replayed; consecutive launches
overlap their ramps (programmatic dependent launch), as a decode chain of
matvecs runs.  value = algorithmic bytes (N*K/32*block_bytes + 4K + 4N per
matvec) of every launch of every rank / max-over-ranks device time of the K
timed steps; roofline.achieved is the same bytes per launch over the average
launch duration in that timed region.

  python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
                  [--workload q4_4096x4096|q8_4096x4096|<q4|q8>_<N>x<K>[_m<M>][_shard]|<model>_token[_m<M>]
                             |qwen3b_decode[_m<M>][_c<context>]]
                  [--mode fast|exact|tc|auto]

Under torch.distributed.run (WORLD_SIZE > 1) the default workload is the
row-sharded 70B gate/up projection (q4_28672x8192_shard
configs[4]): one weight split by output rows over the ranks, every call
all-gathering its rows inside the kernel (NVLink peer stores): "scaling":
"strong".  --impl reference times the reference's own CPU code (oracle/_ref:
dispatch_matvec_q's per-row dot, fanned out over all host threads) on the same
workload; under torchrun only rank 0 runs it.
"""
from __future__ import annotations

import argparse
import json
import math
import os
import statistics
import sys
import threading
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

Q8, Q4 = 10, 20
DEFAULT_WORKLOAD = "q4_4096x4096"
DEFAULT_SHARDED = "q4_28672x8192_shard"    # the 70B gate/up projection, row-sharded
BLOCK_BYTES = {Q8: 36, Q4: 18}
METRIC = "Q8/Q4 matvec HBM GB/s"


def parse_workload(name: str):
    """'q4_4096x4096' -> (dtype, N, K, M); an optional '_m<M>' suffix sets the batch
    (a trailing '_shard' is read by is_shard_workload)."""
    parts = [p for p in name.split("_") if p != "shard"]
    dt = {"q4": Q4, "q8": Q8}[parts[0]]
    n, k = (int(v) for v in parts[1].split("x"))
    m = int(parts[2][1:]) if len(parts) > 2 and parts[2].startswith("m") else 1
    return dt, n, k, m


def resolve_workload(name, world: int) -> str:
    """The workload a run without --workload measures: configs[1] on one GPU, the
    row-sharded 70B gate/up projection across torchrun ranks."""
    if name:
        return name
    return DEFAULT_SHARDED if world > 1 else DEFAULT_WORKLOAD


def is_shard_workload(name: str) -> bool:
    return name.endswith("_shard")


def uses_tc1(mode_name, n, k, m, sm_count):
    """Whether one matvec runs the batch-1 tensor-core kernel (qmv_tc1_kernel): one
    vector under TC, K a multiple of 1024 up to 4096, and every 32-row CTA
    resident in one wave (capi.cu plan_tc1)."""
    return m == 1 and mode_name == "tc" and k % 1024 == 0 and k <= 4096 and -(-n // 32) <= sm_count


def launches_per_call(n_rows, k, sm_count):
    """Kernels one FAST M <= 2 matvec launches: the activation-limb prep kernel runs
    when a row has at least 320 blocks and a CTA gets at most 96 rows (capi.cu)."""
    return 2 if k // 32 >= 320 and -(-n_rows // sm_count) <= 96 else 1


def shard_call_kernels(mode, n_rows, k, m, sm_count):
    """(kernel timed, kernels launched) for one call of a row-sharded or plain
    projection of m vectors: the tensor-core tile in TC, and in AUTO from three
    vectors (a prep and a tile launch per group of up to 64 vectors); else the row
    kernel, FAST in launches of two vectors (each with its limb prep where
    launches_per_call says so), EXACT in one launch."""
    if mode == "tc" or (mode == "auto" and m >= 3):
        return "qmm_tc_kernel", 2 * -(-m // 64)
    groups = 1 if mode == "exact" else -(-m // 2)
    return "qmv_rows_kernel", groups * launches_per_call(n_rows, k, sm_count)


def alg_bytes(dt, n, k, m):
    return n * (k // 32) * BLOCK_BYTES[dt] + 4 * m * k + 4 * m * n


def measured_peaks():
    path = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(path):
        with open(path) as f:
            p = json.load(f)
        return float(p["hbm_gbs"]), "measured (MEASURED_PEAKS.json hbm_gbs)"
    return 6650.0, "fallback (6.65 TB/s, profiling recipe)"


def profiled_traffic(kernel, dt, n, k, m=1):
    """DRAM bytes per launch from the committed ncu summary of the same kernel and shape, if present."""
    stem = {"qmm_tc_kernel": "matmul_tc", "qmv_tc1_kernel": "matvec_tc1"}.get(kernel, "matvec_rows")
    name = f"{stem}_{'q4' if dt == Q4 else 'q8'}_{n}x{k}{f'_m{m}' if m > 1 else ''}.md"
    path = os.path.join(ROOT, "profiles", name)
    if not os.path.exists(path):
        return None
    for line in open(path):
        if line.strip().startswith("traffic_bytes_per_launch:"):
            try:
                return int(line.split(":", 1)[1].strip().split()[0])
            except ValueError:
                return None
    return None


# ── clocks during the timed region (NVML, what nvidia-smi reads) ───────────
class ClockSampler:
    REASONS = {0x4: "sw_power_cap", 0x8: "hw_slowdown", 0x20: "sw_thermal_slowdown",
               0x40: "hw_thermal_slowdown", 0x80: "hw_power_brake_slowdown", 0x2: "applications_clocks_setting",
               0x1: "gpu_idle", 0x10: "sync_boost"}

    def __init__(self, torch_device_index: int, period_s: float = 0.005):
        self.samples, self.reasons = [], set()
        self.ok = False
        self.period = period_s
        self._stop = threading.Event()
        try:
            import pynvml

            pynvml.nvmlInit()
            import torch

            props = torch.cuda.get_device_properties(torch_device_index)
            h = None
            uuid = getattr(props, "uuid", None)
            if uuid is not None:
                try:
                    h = pynvml.nvmlDeviceGetHandleByUUID(("GPU-" + str(uuid)).encode())
                except Exception:
                    h = None
            if h is None:
                vis = os.environ.get("CUDA_VISIBLE_DEVICES")
                idx = int(vis.split(",")[torch_device_index]) if vis and vis.split(",")[0].isdigit() else torch_device_index
                h = pynvml.nvmlDeviceGetHandleByIndex(idx)
            self.nvml, self.h = pynvml, h
            self.sm_max = pynvml.nvmlDeviceGetMaxClockInfo(h, pynvml.NVML_CLOCK_SM)
            self.ok = True
        except Exception as e:  # no NVML: report that instead of clocks
            self.err = str(e)

    def _reasons_now(self):
        fn = getattr(self.nvml, "nvmlDeviceGetCurrentClocksEventReasons", None) or \
            self.nvml.nvmlDeviceGetCurrentClocksThrottleReasons
        return int(fn(self.h))

    def _run(self):
        while not self._stop.is_set():
            try:
                self.samples.append(self.nvml.nvmlDeviceGetClockInfo(self.h, self.nvml.NVML_CLOCK_SM))
                bits = self._reasons_now()
                for b, name in self.REASONS.items():
                    if bits & b and name != "gpu_idle":
                        self.reasons.add(name)
            except Exception:
                pass
            time.sleep(self.period)

    def start(self):
        if self.ok:
            self.t = threading.Thread(target=self._run, daemon=True)
            self.t.start()

    def stop(self):
        if self.ok:
            self._stop.set()
            self.t.join()

    def summary(self):
        if not self.ok:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": [], "note": "NVML unavailable: " + self.err}
        return {"sm_mhz": statistics.median(self.samples) if self.samples else None, "sm_max_mhz": self.sm_max,
                "reasons": sorted(self.reasons), "samples": len(self.samples)}


# ── the reference's CPU path ──────────────────────────────────────────────
def cpu_reference(dt, n, k, m, q_host, x_host, threads, budget_s, max_ops=None):
    """Time the reference's own dispatch_matvec_q code (oracle/_ref) on host cores."""
    import oracle

    if oracle.reference_available():
        ref, kind = oracle.Reference(), "reference"

        def op():
            for j in range(m):
                ref.matvec(dt, q_host, n, k, x_host[j], 32, threads=threads)
    else:   # the C restatement, rows fanned out over threads (ctypes releases the GIL)
        from concurrent.futures import ThreadPoolExecutor

        orc, kind = oracle.Oracle(), "port"
        rb = q_host.size // n
        pool = ThreadPoolExecutor(max(1, threads))
        bounds = [(n * t // threads, n * (t + 1) // threads) for t in range(threads)]

        def op():
            for j in range(m):
                list(pool.map(lambda b: orc.matvec(dt, q_host[b[0] * rb:b[1] * rb], b[1] - b[0], k, x_host[j]),
                              bounds))
    op()   # warm
    t0 = time.perf_counter()
    ops = 0
    while True:
        op()
        ops += 1
        el = time.perf_counter() - t0
        if el >= budget_s or (max_ops is not None and ops >= max_ops):
            break
    return ops, el, kind


def base_config(args, dt, n, k, m):
    """The workload's identity, the same in both arms' JSON lines."""
    return {"workload": args.workload, "N": n, "K": k, "M": m, "block": 32,
            "quant": "Q4_0" if dt == Q4 else "Q8_0", "mode": args.mode}


def host_normal(seed, std, n):
    """Seeded synthetic values with the reference's idiom (std::mt19937(seed),
    std::normal_distribution<float>), drawn by the reference library built in
    oracle/_ref (so the reference arm loads nothing of the product)."""
    import oracle

    if oracle.reference_available():
        return oracle.Reference().fill_normal(seed, 0.0, std, n)
    return np.random.default_rng(seed).normal(0.0, std, n).astype(np.float32)


def run_reference_arm(args, dt, n, k, m):
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    import oracle

    w = host_normal(42, 0.02, n * k).reshape(n, k)
    q_host = (oracle.Reference() if oracle.reference_available() else oracle.Oracle()).quantize(dt, w.ravel(), 32)
    del w
    x_host = host_normal(43, 1.0, m * k).reshape(m, k)
    threads = os.cpu_count() or 1
    # Each step is one full matvec of the workload; warm-up is bounded to keep the run short.
    for _ in range(min(args.warmup, 3)):
        cpu_reference(dt, n, k, m, q_host, x_host, threads, 0.0, max_ops=1)
    ops, el, kind = cpu_reference(dt, n, k, m, q_host, x_host, threads, budget_s=1e9, max_ops=args.steps)
    gbs = ops * alg_bytes(dt, n, k, m) / el / 1e9
    sample = (f"{ops} full {n}x{k} {'Q4_0' if dt == Q4 else 'Q8_0'} matvecs (M={m}) through the reference's "
              f"dot_{'q4' if dt == Q4 else 'q8'}_0_f32, rows split over {threads} threads "
              f"(the reference's own row fan-out, backend.cpp:145-151)")
    line = {"impl": "reference", "metric": METRIC, "value": gbs, "unit": "GB/s", "n_gpus": args.gpus,
            "steps": ops, "warmup": args.warmup, "ms_per_step": el / ops * 1e3, "higher_is_better": True,
            "scaling": "strong" if is_shard_workload(args.workload) else "weak", "vs_baseline": None,
            "dtype": "f32", "data": "synthetic", "config": base_config(args, dt, n, k, m),
            "cpu_baseline": {"value": gbs, "unit": "GB/s", "cores": threads, "kind": kind, "sample": sample},
            "e2e": {"value": gbs, "unit": "GB/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


# ── our arm ───────────────────────────────────────────────────────────────
def run_ours(args, dt, n, k, m):
    import torch

    import qraf_b200 as qb

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    dist = None
    if world > 1:
        import datetime

        import torch.distributed as dist

        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120), device_id=dev)
    qb.init(local)
    mode = {"exact": qb.MODE_EXACT, "fast": qb.MODE_FAST, "tc": qb.MODE_TC, "auto": qb.MODE_AUTO}[args.mode]
    use_tc = args.mode == "tc" or (args.mode == "auto" and m >= 3)   # AUTO's switch (every bench shape qualifies)
    sm_count = torch.cuda.get_device_properties(dev).multi_processor_count
    if uses_tc1(args.mode, n, k, m, sm_count):
        kernel = "qmv_tc1_kernel"
    else:
        kernel = "qmm_tc_kernel" if use_tc else ("qmv_rows_kernel" if m <= 2 or args.mode == "exact"
                                                 else "qmv_stream_kernel")

    # Seeded weight, quantized on the GPU (byte-exact with the reference quantizer).
    wf = torch.from_numpy(qb.fill_normal(42, 0.0, 0.02, n * k)).to(dev).reshape(n, k)
    q = qb.quantize_rows(dt, wf, 32).reshape(-1)
    del wf
    wbytes = q.numel()
    props = torch.cuda.get_device_properties(dev)
    l2 = props.L2_cache_size
    free, _ = torch.cuda.mem_get_info(dev)
    R = max(2, math.ceil(4 * l2 / wbytes))
    R = max(2, min(R, int(0.5 * free // wbytes)))
    pool = torch.empty((R, wbytes), dtype=torch.uint8, device=dev)
    pool[:] = q
    weights = [qb.Weight.from_device(pool[r], dt, n, k) for r in range(R)]
    x = torch.from_numpy(qb.fill_normal(43, 0.0, 1.0, m * k)).to(dev).reshape(m, k)
    y = torch.empty((R, m, n), dtype=torch.float32, device=dev)

    payload_ok = None
    dg = os.path.join(ROOT, "tests", "golden", "config_digests.json")
    if os.path.exists(dg) and (n, k) == (4096, 4096):
        import hashlib

        key = "cfg2_q4_4096x4096" if dt == Q4 else "cfg1_q8_4096x4096"
        want = json.load(open(dg))[key]["sha_q"]
        payload_ok = hashlib.sha256(q.cpu().numpy().tobytes()).hexdigest() == want

    # One step = one launch per weight copy, captured as a CUDA graph.  Launches
    # may overlap their ramps (programmatic dependent launch) unless --no-overlap.
    # A second graph of the same launches strictly one after another gives the
    # average duration of one launch (for the roofline): its replay is bracketed
    # by CUDA events on the launching stream, right after the timed steps.
    launch_mode = mode | (qb.MODE_FLAG_OVERLAP if args.overlap else 0)
    s = torch.cuda.Stream(dev)
    with torch.cuda.stream(s):
        for r in range(R):
            qb.matvec_q(weights[r], x, y[r], mode=launch_mode)
    torch.cuda.synchronize(dev)
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g, stream=s):
        for r in range(R):
            qb.matvec_q(weights[r], x, y[r], mode=launch_mode)
    g_seq = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g_seq, stream=s):
        for r in range(R):
            qb.matvec_q(weights[r], x, y[r], mode=mode)
    for _ in range(max(3, args.warmup)):
        g.replay()
    g_seq.replay()
    torch.cuda.synchronize(dev)

    clocks = ClockSampler(local)
    t0, t1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    t2, t3 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    seq_reps = max(3, min(50, args.steps // 10))
    if dist:
        dist.barrier()
    torch.cuda.synchronize(dev)
    clocks.start()
    with torch.cuda.stream(s):
        t0.record()
        for _ in range(args.steps):
            g.replay()
        t1.record()
        t2.record()         # average launch duration, right after the timed steps
        for _ in range(seq_reps):
            g_seq.replay()
        t3.record()
    torch.cuda.synchronize(dev)
    clocks.stop()
    if dist:
        dist.barrier()
    elapsed_ms = t0.elapsed_time(t1)
    kern_ms = t2.elapsed_time(t3) / (seq_reps * R)
    if dist:
        t = torch.tensor([elapsed_ms, kern_ms], device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        elapsed_ms, kern_ms = float(t[0]), float(t[1])
    per_launch = alg_bytes(dt, n, k, m)
    value = world * args.steps * R * per_launch / (elapsed_ms / 1e3) / 1e9
    peak, peak_src = measured_peaks()
    launch_ms = elapsed_ms / (args.steps * R)              # average launch duration in the timed region
    achieved = per_launch / (launch_ms / 1e3) / 1e9
    achieved_alone = per_launch / (kern_ms / 1e3) / 1e9
    status = qb.device_status()

    # e2e: the reference-facing host entry (host x in, host y out, synchronous), same pool.
    q_host = q.cpu().numpy()
    host_copies = [q_host.copy() for _ in range(R)]
    x_host = x.cpu().numpy()
    y_host = np.empty((m, n), dtype=np.float32)
    for r in range(R):   # first call per copy uploads it into the device weight cache
        qb.dispatch_matvec_q(host_copies[r], wbytes, dt, 32, n, k, x_host, y_host, m=m, mode=mode)
    e2e_steps = max(3, min(args.steps, 100))
    if dist:
        dist.barrier()
    te = time.perf_counter()
    for _ in range(e2e_steps):
        for r in range(R):
            qb.dispatch_matvec_q(host_copies[r], wbytes, dt, 32, n, k, x_host, y_host, m=m, mode=mode)
    e2e_s = time.perf_counter() - te
    if dist:
        t = torch.tensor([e2e_s], device=dev, dtype=torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        e2e_s = float(t[0])
    e2e = {"value": world * e2e_steps * R * per_launch / e2e_s / 1e9, "unit": "GB/s",
           "h2d_bytes_per_step": R * m * k * 4, "d2h_bytes_per_step": R * m * n * 4, "steps": e2e_steps,
           "path": "qraf_cuda_matvec_q_host (drop-in body of qraf::dispatch_matvec_q): pinned staging, H2D x and "
                   "D2H y by SM copy kernels over the mapped pinned buffers, the matvec kernel, stream sync per call "
                   "(one cached CUDA graph per weight, M and mode); weights cached on the device after their first "
                   "call"}
    qb.host_cache_clear()

    cpu = None
    if rank == 0 and world == 1:
        ops, el, kind = cpu_reference(dt, n, k, m, q_host, x_host.reshape(m, k), 1, budget_s=args.cpu_seconds)
        cpu = {"value": ops * per_launch / el / 1e9, "unit": "GB/s", "cores": 1, "kind": kind,
               "sample": f"{ops} full {n}x{k} matvecs (M={m}) through dispatch_matvec_q's scalar Linux path "
                         f"(single-threaded, as the reference runs it), {el:.1f} s of {os.cpu_count()} host threads' "
                         f"worth of cores used: 1"}

    if rank == 0:
        line = {
            "metric": METRIC, "value": value, "unit": "GB/s", "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": elapsed_ms / args.steps, "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
            "config": base_config(args, dt, n, k, m),
            "setup": {"parallelism": f"independent weights per rank x{world}" if world > 1 else "single GPU",
                      "pool_copies": R, "pool_bytes": R * wbytes, "l2_bytes": l2,
                      "l2_policy": "inputs larger than L2: rotating pool of weight copies >= 4x L2",
                      "step": f"{R} matvec launches, one per L2-cold weight copy (CUDA graph replay)",
                      "launch_overlap": "programmatic dependent launch (weights prefetched before the previous "
                                        "launch ends)" if args.overlap else "none",
                      "weights": "N(0,0.02) std::mt19937(42), quantized on GPU (byte-exact Q*_0)",
                      "payload_sha_matches_reference": payload_ok, "arith": "exact int32 block sums, fp32 accumulate"},
            "e2e": e2e,
            "gpu_launches": args.steps * R * launches_per_call(n, k, props.multi_processor_count)
            if kernel == "qmv_rows_kernel" and m <= 2 and args.mode != "exact" else args.steps * R,
            "roofline": {"bound": "hbm", "achieved": achieved, "peak": peak, "unit": "GB/s",
                         "frac": achieved / peak, "traffic": profiled_traffic(kernel, dt, n, k, m),
                         "peak_source": peak_src, "kernel": kernel,
                         "kernel_us": launch_ms * 1e3,
                         "kernel_timing": "average launch duration in the timed region (CUDA events on the "
                                          "launching stream around the K steps of overlapping launches)",
                         "kernel_us_alone": kern_ms * 1e3, "achieved_alone": achieved_alone,
                         "frac_alone": achieved_alone / peak,
                         "alone_timing": "the same launches strictly one after another, without overlap (CUDA "
                                         "events around a graph of them, inter-launch gaps included)",
                         "alg_bytes_per_launch": per_launch},
            "clocks": clocks.summary(),
            "cpu_baseline": cpu,
            "device_status": status,
        }
        print(json.dumps(line), flush=True)
    del g, g_seq
    if dist:
        dist.barrier()
        dist.destroy_process_group()

# ── decode-token workloads: BASELINE.json configs 3 and 5 ─────────────────
# Per layer, the projections in call order: (name, N out, K in, input).  The
# input is the output of an earlier projection of the token ("h" = the layer's
# input, which is the previous layer's "down" output).  Attention, norms and
# SwiGLU are not on the path: O consumes the Q projection's output and down
# consumes gate's (same widths), so every matvec reads a real predecessor.
TOKEN_MODELS = {
    # Qwen2-style 3B (config 3): hidden 2048, 16 Q / 2 KV heads of 128, FFN 11008, tied LM head 151936, Q8_0.
    "qwen3b": {"dtype": Q8, "layers": 36, "hidden": 2048, "vocab": 151936,
               "projs": [("q", 2048, 2048, "h"), ("k", 256, 2048, "h"), ("v", 256, 2048, "h"),
                         ("o", 2048, 2048, "q"), ("gate", 11008, 2048, "o"), ("up", 11008, 2048, "o"),
                         ("down", 2048, 11008, "gate")],
               # projections of one input in the model (attention.cpp:92-97, :172-174): one launch each
               "groups": [("q", "k", "v"), ("gate", "up")],
               # RMSNorm before the attention and MLP inputs (transformer.cpp:588-590, :596-597);
               # Qwen2's Q, K and V biases (attention.cpp:100-102)
               "norm_before": ("q", "gate"), "biased": ("q", "k", "v")},
    # 70B shapes (config 5), Q4_0: fused QKV 10240, gate/up 28672, down, LM head 128256.
    "llama70b": {"dtype": Q4, "layers": 80, "hidden": 8192, "vocab": 128256,
                 "projs": [("qkv", 10240, 8192, "h"), ("gate", 28672, 8192, "h"), ("up", 28672, 8192, "h"),
                           ("down", 8192, 28672, "gate")],
                 "groups": [("gate", "up")],
                 "norm_before": ("qkv", "gate"), "biased": ()},
}
# The payload digests of the reference quantizer (tests/golden/config_digests.json)
# for each projection shape of the token workloads.
TOKEN_DIGEST_KEYS = {
    "qwen3b": {(2048, 2048): "cfg3_q8_qo", (256, 2048): "cfg3_q8_kv", (11008, 2048): "cfg3_q8_gate_up",
               (2048, 11008): "cfg3_q8_down", (151936, 2048): "cfg3_q8_lm_head"},
    "llama70b": {(10240, 8192): "cfg5_q4_qkv", (28672, 8192): "cfg5_q4_gate_up", (8192, 28672): "cfg5_q4_down",
                 (128256, 8192): "cfg5_q4_lm_head"},
}
TOKEN_METRIC = "projection-only decode tokens/s"


def parse_token_workload(name: str):
    """'llama70b_token' / 'qwen3b_token_m2' -> (model, M), or None for a single-matvec workload."""
    parts = name.split("_")
    if len(parts) < 2 or parts[0] not in TOKEN_MODELS or parts[1] != "token":
        return None
    m = int(parts[2][1:]) if len(parts) > 2 and parts[2].startswith("m") else 1
    return parts[0], m


def token_shapes(spec):
    """Every projection of one token, in order: (name, N, K, input), the LM head last."""
    calls = []
    for _ in range(spec["layers"]):
        calls.extend(spec["projs"])
    return calls + [("lm_head", spec["vocab"], spec["hidden"], "h")]


def token_cpu_seconds(spec, m, time_rows):
    """Seconds for one token of M vectors on the reference's CPU path, from per-row times:
    time_rows(n, k) -> seconds per row of that shape."""
    per_layer = sum(time_rows(n, k) * n for _, n, k, _ in spec["projs"])
    lm = time_rows(spec["vocab"], spec["hidden"]) * spec["vocab"]
    return m * (spec["layers"] * per_layer + lm)


def _sample_rows_timer(spec, threads, budget_s, quantized_rows):
    """Per-row seconds of the reference's dot (oracle/_ref) on a bounded sample of rows of each shape.
    quantized_rows(n, k, rows) -> host bytes of the first `rows` rows of that shape."""
    import oracle

    ref = oracle.Reference() if oracle.reference_available() else None
    orc = None if ref else oracle.Oracle()
    dt = spec["dtype"]
    shapes = sorted({(n, k) for _, n, k, _ in spec["projs"]} | {(spec["vocab"], spec["hidden"])})
    per_row, sampled = {}, []
    x_cache = {}
    for n, k in shapes:
        rows = min(n, max(256, 32 * threads))
        q = quantized_rows(n, k, rows)
        x = x_cache.setdefault(k, qb_fill(43, k))
        t0 = time.perf_counter()
        reps = 0
        while True:
            if ref:
                ref.matvec(dt, q, rows, k, x, 32, threads=threads)
            else:
                orc.matvec(dt, q, rows, k, x)
            reps += 1
            if time.perf_counter() - t0 >= budget_s / len(shapes):
                break
        per_row[(n, k)] = (time.perf_counter() - t0) / (reps * rows)
        sampled.append(f"{reps}x{rows} rows of {n}x{k}")
    kind = "reference" if ref else "port"
    return (lambda n, k: per_row[(n, k)]), kind, "; ".join(sampled)


def qb_fill(seed, n):
    return host_normal(seed, 1.0, n)


def run_shard(args, dt, n, k, m):
    """One projection split by output rows over the N ranks (rank r: rows
    [r N/W, (r+1) N/W)); every call all-gathers the rows into every rank's y,
    inside the kernel (peer stores over NVLink, default) or by NCCL after the
    plain kernel (--allgather nccl).  On one GPU: the unsharded kernel.  A STEP is
    R calls over a pool of shard copies (>= 4x L2 per GPU, R a multiple of 4),
    replayed from a CUDA graph with overlapping launches; single-call latency is
    the same calls one after another.  value = bytes of the WHOLE projection x
    calls / max-over-ranks device time ("strong": the work per call is fixed)."""
    import torch

    import qraf_b200 as qb

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    dist = None
    if world > 1:
        import datetime

        import torch.distributed as dist

        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120), device_id=dev)
    qb.init(local)
    mode = {"exact": qb.MODE_EXACT, "fast": qb.MODE_FAST, "tc": qb.MODE_TC, "auto": qb.MODE_AUTO}[args.mode]
    fused = world > 1 and args.allgather == "fused"
    r0, r1 = n * rank // world, n * (rank + 1) // world
    rows = r1 - r0

    # the shard's rows of the seeded weight (seeded per 1024-row chunk, so every
    # world size draws the same rows), quantized byte-exactly on the device
    gen = torch.Generator(device=dev)
    wf = torch.empty((rows, k), device=dev)
    for c0 in range(r0 // 1024 * 1024, r1, 1024):
        gen.manual_seed(42 * 1_000_003 + c0 // 1024)
        blk = torch.randn((min(1024, n - c0), k), generator=gen, device=dev) * 0.02
        a, b = max(c0, r0), min(c0 + 1024, r1)
        wf[a - r0:b - r0] = blk[a - c0:b - c0]
    q = qb.quantize_rows(dt, wf, 32).reshape(-1)
    del wf
    sbytes = q.numel()
    props = torch.cuda.get_device_properties(dev)
    free, _ = torch.cuda.mem_get_info(dev)
    R = max(4, math.ceil(4 * props.L2_cache_size / sbytes))
    R = min(R, max(4, int(0.5 * free // sbytes)))
    R = (R + 3) // 4 * 4   # whole rounds of the comm's four output buffers
    pool = torch.empty((R, sbytes), dtype=torch.uint8, device=dev)
    pool[:] = q
    weights = [qb.Weight.from_device(pool[i], dt, rows, k) for i in range(R)]
    x = torch.from_numpy(qb.fill_normal(43, 0.0, 1.0, m * k)).to(dev).reshape(m, k)

    # The same projection unsharded on rank 0's GPU alone (the 1-GPU point of this
    # strong-scaling line; the other ranks wait at the barrier).
    one_gpu = None
    if world > 1 and not args.no_1gpu_ref:
        if rank == 0:
            one_gpu = _unsharded_figure(args, dt, n, k, m, mode, dev)
        dist.barrier()

    comm = None
    ys = [torch.empty((m, n), device=dev) for _ in range(R)] if world == 1 else None
    loc = gat = None
    if fused:
        comm = qb.make_comm(world, rank, m * n, qb.torch_all_gather_bytes())
    elif world > 1:
        loc = [torch.empty((m, rows), device=dev) for _ in range(R)]
        gat = [torch.empty((world * m * rows,), device=dev) for _ in range(R)]

    def call(i, flags):
        if world == 1:
            return qb.matvec_q(weights[i], x, ys[i], mode=mode | flags)
        if fused:
            return comm.matvec_q(weights[i], n, r0, x, mode=mode | flags)
        qb.matvec_q(weights[i], x, loc[i], mode=mode | flags)
        dist.all_gather_into_tensor(gat[i], loc[i])
        return gat[i]

    ov = qb.MODE_FLAG_OVERLAP if args.overlap else 0
    s = torch.cuda.Stream(dev)
    with torch.cuda.stream(s):
        for i in range(R):
            call(i, ov)
    torch.cuda.synchronize(dev)
    if dist:
        dist.barrier()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g, stream=s):
        for i in range(R):
            last = call(i, ov)
    g_seq = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g_seq, stream=s):
        for i in range(R):
            call(i, 0)
    for _ in range(max(3, args.warmup)):
        g.replay()
    g_seq.replay()
    torch.cuda.synchronize(dev)
    if qb.device_status() != qb.OK:
        raise SystemExit("device status not OK after warm-up")

    clocks = ClockSampler(local)
    t0, t1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    t2, t3 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    seq_reps = max(3, min(20, args.steps // 10))
    if dist:
        dist.barrier()
    torch.cuda.synchronize(dev)
    clocks.start()
    with torch.cuda.stream(s):
        t0.record()
        for _ in range(args.steps):
            g.replay()
        t1.record()
        t2.record()
        for _ in range(seq_reps):
            g_seq.replay()
        t3.record()
    torch.cuda.synchronize(dev)
    clocks.stop()
    elapsed_ms, call_ms = t0.elapsed_time(t1), t2.elapsed_time(t3) / (seq_reps * R)

    # e2e: the step's x in from pinned host memory, its last call's y out
    x_host = torch.from_numpy(qb.fill_normal(44, 0.0, 1.0, m * k)).reshape(m, k).pin_memory()
    y_host = torch.empty((m, n), dtype=torch.float32).pin_memory()
    e2e_steps = max(3, min(args.steps, 50))
    if dist:
        dist.barrier()
    te = time.perf_counter()
    for _ in range(e2e_steps):
        with torch.cuda.stream(s):
            x.copy_(x_host, non_blocking=True)
            g.replay()
            y_host.copy_(last.reshape(world, m, rows).permute(1, 0, 2).reshape(m, n) if (world > 1 and not fused
                                                                                      and m > 1) else
                         last.reshape(m, n), non_blocking=True)
        s.synchronize()
    e2e_s = time.perf_counter() - te
    status = qb.device_status()
    if dist:
        t = torch.tensor([elapsed_ms, call_ms, e2e_s, float(status != qb.OK)], device=dev, dtype=torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        elapsed_ms, call_ms, e2e_s = float(t[0]), float(t[1]), float(t[2])
        status = status if not float(t[3]) else max(status, 1)

    full = alg_bytes(dt, n, k, m)
    shard = alg_bytes(dt, rows, k, m)
    peak, peak_src = measured_peaks()
    cpu = None
    if rank == 0 and world == 1:
        q_host = q.cpu().numpy()
        xh = x.cpu().numpy()
        ops, el, kind = cpu_reference(dt, n, k, m, q_host, xh, 1, args.cpu_seconds, max_ops=1000)
        cpu = {"value": ops * full / el / 1e9, "unit": "GB/s", "cores": 1, "kind": kind,
               "sample": f"{ops} full {n}x{k} matvecs (M={m}) through dispatch_matvec_q's scalar path, "
                         "single-threaded as the reference runs it on Linux"}
    if rank == 0:
        calls = args.steps * R
        line = {
            "metric": METRIC, "value": calls * full / (elapsed_ms / 1e3) / 1e9, "unit": "GB/s", "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": elapsed_ms / args.steps,
            "higher_is_better": True, "scaling": "strong" if world > 1 else "weak", "vs_baseline": None,
            "dtype": "f32", "data": "synthetic",
            "config": base_config(args, dt, n, k, m),
            "setup": {"parallelism": (f"rows split over {world} GPUs ({rows} per GPU), all-gather "
                                      f"{'fused into the kernel (NVLink peer stores)' if fused else 'by NCCL'}")
                      if world > 1 else "single GPU (unsharded kernel)",
                      "comm_ranks": world,
                      "pool_copies": R, "l2_policy": "inputs larger than L2: rotating pool of shard copies",
                      "step": f"{R} calls (CUDA graph replay, overlapping launches)",
                      "us_per_call_pipelined": elapsed_ms * 1e3 / calls,
                      "us_per_call_alone": call_ms * 1e3,
                      "same_workload_1gpu": one_gpu},
            "e2e": {"value": e2e_steps * R * full / e2e_s / 1e9, "unit": "GB/s", "h2d_bytes_per_step": m * k * 4,
                    "d2h_bytes_per_step": m * n * 4, "steps": e2e_steps,
                    "path": "H2D x from pinned memory, the step's graph, D2H of the last call's y, stream sync"},
            "gpu_launches": calls * shard_call_kernels(args.mode, rows, k, m, props.multi_processor_count)[1],
            "roofline": {"bound": "hbm", "achieved": shard / (call_ms / 1e3) / 1e9, "peak": peak, "unit": "GB/s",
                         "frac": shard / (call_ms / 1e3) / 1e9 / peak, "traffic": None, "peak_source": peak_src,
                         "what": "per GPU: shard bytes of one call / the call's duration alone",
                         "kernel": shard_call_kernels(args.mode, rows, k, m, props.multi_processor_count)[0]},
            "clocks": clocks.summary(),
            "cpu_baseline": cpu,
            "device_status": status,
        }
        print(json.dumps(line), flush=True)
    del g, g_seq
    if dist:
        dist.barrier()
    if comm is not None:
        comm.destroy()
    if dist:
        dist.destroy_process_group()


def _unsharded_figure(args, dt, n, k, m, mode, dev):
    """Pipelined and single-call time of the whole projection on this GPU alone:
    a pool of full-weight copies (>= 4 x L2), one CUDA graph of overlapping calls."""
    import torch

    import qraf_b200 as qb

    gen = torch.Generator(device=dev)
    wf = torch.empty((n, k), device=dev)
    for c0 in range(0, n, 1024):
        gen.manual_seed(42 * 1_000_003 + c0 // 1024)
        wf[c0:c0 + 1024] = torch.randn((min(1024, n - c0), k), generator=gen, device=dev) * 0.02
    q = qb.quantize_rows(dt, wf, 32).reshape(-1)
    del wf
    wb = q.numel()
    R = max(2, math.ceil(4 * torch.cuda.get_device_properties(dev).L2_cache_size / wb))
    pool = torch.empty((R, wb), dtype=torch.uint8, device=dev)
    pool[:] = q
    ws = [qb.Weight.from_device(pool[i], dt, n, k) for i in range(R)]
    x = torch.from_numpy(qb.fill_normal(43, 0.0, 1.0, m * k)).to(dev).reshape(m, k)
    ys = torch.empty((R, m, n), device=dev)
    s = torch.cuda.Stream(dev)
    ov = qb.MODE_FLAG_OVERLAP if args.overlap else 0
    with torch.cuda.stream(s):
        for i in range(R):
            qb.matvec_q(ws[i], x, ys[i], mode=mode | ov)
    torch.cuda.synchronize(dev)
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g, stream=s):
        for i in range(R):
            qb.matvec_q(ws[i], x, ys[i], mode=mode | ov)
    for _ in range(3):
        g.replay()
    torch.cuda.synchronize(dev)
    t0, t1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    reps = max(3, min(20, args.steps))
    with torch.cuda.stream(s):
        t0.record()
        for _ in range(reps):
            g.replay()
        t1.record()
    torch.cuda.synchronize(dev)
    us = t0.elapsed_time(t1) * 1e3 / (reps * R)
    del g
    return {"value": alg_bytes(dt, n, k, m) / (us * 1e-6) / 1e9, "unit": "GB/s", "us_per_call_pipelined": us,
            "what": "the same projection unsharded on one GPU of this box (rank 0 alone), same pool and graph method"}


def run_token(args, model, m):
    """One STEP = one decode token of M vectors through every projection of the model
    (layers x projections + LM head), captured as one CUDA graph and replayed.
    With N > 1 ranks every weight is split by output rows; each call's rows reach
    every rank either through the fused kernel (peer stores over NVLink, the
    default) or through an NCCL all-gather after the plain kernel (--allgather nccl,
    the baseline).  value = M x steps / max-over-ranks device time (tokens/s)."""
    import torch

    import qraf_b200 as qb

    spec = TOKEN_MODELS[model]
    dt, hidden, vocab = spec["dtype"], spec["hidden"], spec["vocab"]
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    dist = None
    if world > 1:
        import datetime

        import torch.distributed as dist

        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120), device_id=dev)
    qb.init(local)
    mode = {"exact": qb.MODE_EXACT, "fast": qb.MODE_FAST, "tc": qb.MODE_TC, "auto": qb.MODE_AUTO}[args.mode]
    fused = world > 1 and args.allgather == "fused"

    # Seeded weights with the reference's idiom: for every projection shape one
    # std::mt19937(42) draw of N(0, 0.02) over the whole [N][K] tensor (the same
    # bytes as the reference's quantizer digests of configs 3 and 5), quantized
    # byte-exactly on the device; each rank keeps its rows, copied into every layer
    # in distinct memory (every matvec reads its weight cold).
    import hashlib

    digests = {}
    dpath = os.path.join(ROOT, "tests", "golden", "config_digests.json")
    if os.path.exists(dpath):
        with open(dpath) as f:
            digests = json.load(f)
    payload_ok = {}
    by_shape = {}

    def shard_bytes(n, k):
        r0, r1 = n * rank // world, n * (rank + 1) // world
        if (n, k) not in by_shape:
            wf = torch.from_numpy(qb.fill_normal(42, 0.0, 0.02, n * k)).reshape(n, k)
            q = qb.quantize_rows(dt, wf.to(dev), 32)
            del wf
            key = TOKEN_DIGEST_KEYS[model].get((n, k))
            if key in digests:
                payload_ok[key] = hashlib.sha256(q.cpu().numpy().tobytes()).hexdigest() == digests[key]["sha_q"]
            by_shape[(n, k)] = q[r0:r1].reshape(-1).clone()
            del q
        return by_shape[(n, k)], r0, r1

    projs = spec["projs"]
    layer_bytes, proto = 0, []
    for name, n, k, _ in projs:
        q, r0, r1 = shard_bytes(n, k)
        proto.append((name, n, k, q, r0, r1, layer_bytes))
        layer_bytes += (q.numel() + 255) // 256 * 256
    store = torch.empty((spec["layers"], layer_bytes), dtype=torch.uint8, device=dev)
    weights = []
    for l in range(spec["layers"]):
        row = []
        for name, n, k, q, r0, r1, off in proto:
            view = store[l, off:off + q.numel()]
            view.copy_(q)
            row.append(qb.Weight.from_device(view, dt, r1 - r0, k))
        weights.append(row)
    q_lm, lm0, lm1 = shard_bytes(vocab, hidden)
    shape_bytes = dict(by_shape)
    w_lm = qb.Weight.from_device(q_lm, dt, lm1 - lm0, hidden)
    shard_weight_bytes = spec["layers"] * sum(p[3].numel() for p in proto) + q_lm.numel()
    total_weight_bytes = spec["layers"] * sum(n * (k // 32) * BLOCK_BYTES[dt] for _, n, k, _ in projs) + \
        vocab * (hidden // 32) * BLOCK_BYTES[dt]
    del proto
    torch.cuda.synchronize(dev)

    h0 = torch.from_numpy(qb.fill_normal(43, 0.0, 1.0, m * hidden)).to(dev).reshape(m, hidden)
    launch_mode = mode | (qb.MODE_FLAG_OVERLAP if args.overlap else 0)
    comm = comm_lm = None
    ybuf, lbuf, gbuf = {}, {}, {}
    if fused:
        gather = qb.torch_all_gather_bytes()
        cap = m * max(n for _, n, _, _ in projs)
        comm = qb.make_comm(world, rank, cap, gather)
        comm_lm = qb.make_comm(world, rank, m * vocab, gather)   # logits: their own buffers
    for name, n, k, _ in projs + [("lm_head", vocab, hidden, "h")]:
        r0, r1 = n * rank // world, n * (rank + 1) // world
        if world == 1:
            ybuf[name] = torch.empty((m, n), device=dev)
        elif not fused:
            lbuf[name] = torch.empty((m, r1 - r0), device=dev)
            gbuf[name] = torch.empty((world * m * (r1 - r0),), device=dev)

    def project(name, n, k, w, x):
        r0 = n * rank // world
        if world == 1:
            return qb.matvec_q(w, x, ybuf[name], mode=launch_mode)
        if fused:
            return (comm_lm if name == "lm_head" else comm).matvec_q(w, n, r0, x, mode=launch_mode)
        loc = qb.matvec_q(w, x, lbuf[name], mode=launch_mode)
        dist.all_gather_into_tensor(gbuf[name], loc)
        rows = n // world
        g = gbuf[name]
        return g.view(1, n) if m == 1 else g.view(world, m, rows).permute(1, 0, 2).reshape(m, n)

    # projections of one input go in one launch (qraf_cuda_matvec_q_multi) on one GPU;
    # gate and up as one SwiGLU launch (qraf_cuda_matvec_q_swiglu: down reads silu(gate) * up);
    # the RMSNorms before them and Qwen2's Q/K/V biases folded into those launches
    multi = world == 1 and args.multi
    first_of = {g[0]: g for g in spec.get("groups", [])} if multi else {}
    in_group = {name for g in first_of.values() for name in g}
    swiglu = multi and args.swiglu
    fuse = swiglu and args.norms
    norms, bias = {}, {}
    if fuse:
        gen = torch.Generator().manual_seed(45)
        for l in range(spec["layers"]):
            for name in spec["norm_before"]:
                norms[(l, name)] = (1.0 + 0.1 * torch.randn(hidden, generator=gen)).to(dev)
            for name, n, k, _ in projs:
                if name in spec["biased"]:
                    bias[(l, name)] = (0.1 * torch.randn(n, generator=gen)).to(dev)

    def token():
        vals = {"h": h0}
        for l in range(spec["layers"]):
            ws = {name: w for (name, _, _, _), w in zip(projs, weights[l])}
            for name, n, k, src in projs:
                nw = norms.get((l, name))
                if name in first_of:
                    g = first_of[name]
                    if swiglu and g == ("gate", "up"):
                        vals["gate"] = qb.matvec_q_swiglu(ws["gate"], ws["up"], vals[src], ybuf["gate"],
                                                          mode=launch_mode, norm_w=nw)
                        continue
                    bs = [bias.get((l, x)) for x in g] if any((l, x) in bias for x in g) else None
                    outs = qb.matvec_q_multi([ws[x] for x in g], vals[src], [ybuf[x] for x in g], mode=launch_mode,
                                             norm_w=nw, biases=bs)
                    vals.update(zip(g, outs))
                elif name not in in_group:
                    if nw is not None or (l, name) in bias:
                        vals[name] = qb.matvec_q_multi([ws[name]], vals[src], [ybuf[name]], mode=launch_mode,
                                                       norm_w=nw, biases=[bias.get((l, name))])[0]
                    else:
                        vals[name] = project(name, n, k, ws[name], vals[src])
            vals["h"] = vals["down"]
        return project("lm_head", vocab, hidden, w_lm, vals["h"])

    s = torch.cuda.Stream(dev)
    with torch.cuda.stream(s):
        token()
    torch.cuda.synchronize(dev)
    if dist:
        dist.barrier()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g, stream=s):
        logits = token()
    for _ in range(max(3, args.warmup)):
        g.replay()
    torch.cuda.synchronize(dev)
    if qb.device_status() != qb.OK:
        raise SystemExit("device status not OK after warm-up")

    clocks = ClockSampler(local)
    t0, t1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    if dist:
        dist.barrier()
    torch.cuda.synchronize(dev)
    clocks.start()
    with torch.cuda.stream(s):
        t0.record()
        for _ in range(args.steps):
            g.replay()
        t1.record()
    torch.cuda.synchronize(dev)
    clocks.stop()
    elapsed_ms = t0.elapsed_time(t1)

    # e2e: every step copies its input hidden state in from pinned host memory and
    # its logits out, around the same graph.
    h_host = torch.from_numpy(qb.fill_normal(44, 0.0, 1.0, m * hidden)).reshape(m, hidden).pin_memory()
    lg_host = torch.empty((m, vocab), dtype=torch.float32).pin_memory()
    e2e_steps = max(3, min(args.steps, 50))
    if dist:
        dist.barrier()
    te = time.perf_counter()
    for _ in range(e2e_steps):
        with torch.cuda.stream(s):
            h0.copy_(h_host, non_blocking=True)
            g.replay()
            lg_host.copy_(logits, non_blocking=True)
        s.synchronize()
    e2e_s = time.perf_counter() - te
    status = qb.device_status()
    if dist:
        t = torch.tensor([elapsed_ms, e2e_s, float(status != qb.OK)], device=dev, dtype=torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        elapsed_ms, e2e_s, bad = float(t[0]), float(t[1]), float(t[2])
        status = status if not bad else max(status, 1)

    calls = (len(projs) - sum(len(g) - 1 for g in first_of.values())) * spec["layers"] + 1
    act_bytes = sum(4 * m * (k + n) for _, n, k, _ in token_shapes(spec))
    per_token_s = elapsed_ms / 1e3 / args.steps
    peak, peak_src = measured_peaks()
    achieved = (shard_weight_bytes + act_bytes) / per_token_s / 1e9   # per GPU
    cpu = None
    if rank == 0 and world == 1:
        def host_rows(n, k, rows):
            return shape_bytes[(n, k)][:rows * (k // 32) * BLOCK_BYTES[dt]].cpu().numpy()

        timer, kind, sample = _sample_rows_timer(spec, 1, args.cpu_seconds, host_rows)
        cpu_tok_s = token_cpu_seconds(spec, m, timer)
        cpu = {"value": m / cpu_tok_s, "unit": "tokens/s", "cores": 1, "kind": kind,
               "sample": f"per-row time of dispatch_matvec_q's scalar path (single-threaded, as the reference runs "
                         f"it on Linux) on {sample}, scaled to every row of one token"}
    if rank == 0:
        line = {
            "metric": TOKEN_METRIC, "value": m * args.steps / (elapsed_ms / 1e3), "unit": "tokens/s",
            "n_gpus": world, "steps": args.steps, "warmup": args.warmup, "ms_per_step": elapsed_ms / args.steps,
            "higher_is_better": True, "scaling": "strong" if world > 1 else "weak", "vs_baseline": None,
            "dtype": "f32", "data": "synthetic",
            "config": {"workload": args.workload, "model_shapes": model, "M": m, "layers": spec["layers"],
                       "quant": "Q4_0" if dt == Q4 else "Q8_0", "mode": args.mode, "calls_per_token": calls,
                       "mlp": "silu(gate) * up fused into the gate/up launch; down reads it" if swiglu
                       else "down reads gate (no activation on the path)",
                       "norms": "RMSNorm folded into the QKV and gate/up launches" + (", Q/K/V biases folded in"
                                                                                     if spec["biased"] else "")
                       if fuse else "none on the path",
                       "weight_bytes_per_token": total_weight_bytes,
                       "parallelism": (f"rows split over {world} GPUs, all-gather "
                                       f"{'fused into the kernel (NVLink peer stores)' if fused else 'by NCCL'}")
                       if world > 1 else "single GPU",
                       "l2_policy": "inputs larger than L2: one distinct weight copy per layer "
                                    f"({shard_weight_bytes / 1e9:.1f} GB per GPU per token)",
                       "weights": "N(0,0.02) std::mt19937(42) over each projection shape, quantized on GPU "
                                  "(byte-exact Q*_0); the same bytes copied into every layer",
                       "payload_sha_matches_reference": payload_ok or None,
                       "one_launch_per_input": [list(g) for g in first_of.values()],
                       "excluded": "attention, norms, SwiGLU, sampling (projection-only)",
                       "step": "one token: every projection of every layer + LM head, one CUDA graph replay"},
            "e2e": {"value": m * e2e_steps / e2e_s, "unit": "tokens/s", "h2d_bytes_per_step": m * hidden * 4,
                    "d2h_bytes_per_step": m * vocab * 4, "steps": e2e_steps,
                    "path": "H2D of the token's hidden state from pinned memory, the token graph, D2H of the "
                            "logits, stream sync, every step"},
            "gpu_launches": args.steps * calls,
            "roofline": {"bound": "hbm", "achieved": achieved, "peak": peak, "unit": "GB/s",
                         "frac": achieved / peak, "traffic": None, "peak_source": peak_src,
                         "what": "per GPU: weight shard + activation bytes of one token / time per token",
                         "us_per_token": per_token_s * 1e6},
            "clocks": clocks.summary(),
            "cpu_baseline": cpu,
            "device_status": status,
        }
        print(json.dumps(line), flush=True)
    del g
    if dist:
        dist.barrier()
    for c in (comm, comm_lm):
        if c is not None:
            c.destroy()
    if dist:
        dist.destroy_process_group()


def run_token_reference(args, model, m):
    """The reference's CPU path on the token workload: per-row times of its dot on a
    bounded sample of rows of every shape, rows fanned out over all host threads."""
    if int(os.environ.get("RANK", "0")) != 0:
        return
    import oracle

    spec = TOKEN_MODELS[model]
    dt = spec["dtype"]
    threads = os.cpu_count() or 1
    qz = oracle.Reference() if oracle.reference_available() else oracle.Oracle()

    def host_rows(n, k, rows, cache={}):
        if (n, k) not in cache:
            w = qb_fill(42, rows * k) * np.float32(0.02)
            cache[(n, k)] = qz.quantize(dt, w, 32)
        return cache[(n, k)]

    budget = max(2.0, min(60.0, 4.0 * args.steps))
    timer, kind, sample = _sample_rows_timer(spec, threads, budget, host_rows)
    tok_s = token_cpu_seconds(spec, m, timer)
    line = {"impl": "reference", "metric": TOKEN_METRIC, "value": m / tok_s, "unit": "tokens/s",
            "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup, "ms_per_step": tok_s * 1e3,
            "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "f32",
            "data": "synthetic", "config": {"workload": args.workload, "model_shapes": model, "M": m},
            "cpu_baseline": {"value": m / tok_s, "unit": "tokens/s", "cores": threads, "kind": kind,
                             "sample": f"per-row time of the reference's dot, rows over {threads} threads, on "
                                       f"{sample}; scaled to every row of one token"},
            "e2e": {"value": m / tok_s, "unit": "tokens/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)



# ── decode workloads: the whole decode step (qraf_cuda_decoder_step) ──────
# BASELINE.json config 3's shapes as a Qwen2 model file: every projection, the
# attention over each slot's KV cache, RoPE, the norms, SwiGLU, the residuals.
DECODE_MODELS = {
    "qwen3b": {"arch": "qwen2", "heads": 16, "kv_heads": 2, "inter": 11008},
}
DECODE_METRIC = "decode tokens/s"


def parse_decode_workload(name: str):
    """'qwen3b_decode' / 'qwen3b_decode_m8_c1024[_kv8]' -> (model, M slots, context length, int8 KV cache),
    else None."""
    parts = name.split("_")
    if len(parts) < 2 or parts[0] not in DECODE_MODELS or parts[1] != "decode":
        return None
    m, ctx, kv8 = 1, 512, False
    for p in parts[2:]:
        if p.startswith("m") and p[1:].isdigit():
            m = int(p[1:])
        elif p.startswith("c") and p[1:].isdigit():
            ctx = int(p[1:])
        elif p == "kv8":
            kv8 = True
        else:
            raise SystemExit(f"unknown decode workload part '{p}' in {name}")
    return parts[0], m, ctx, kv8


def decode_shapes(model):
    tok, dec = TOKEN_MODELS[model], DECODE_MODELS[model]
    hidden, heads, kvh, inter = tok["hidden"], dec["heads"], dec["kv_heads"], dec["inter"]
    hd = hidden // heads
    return {"q_proj": (heads * hd, hidden), "k_proj": (kvh * hd, hidden), "v_proj": (kvh * hd, hidden),
            "o_proj": (hidden, heads * hd), "gate_proj": (inter, hidden), "up_proj": (inter, hidden),
            "down_proj": (hidden, inter)}


def write_decode_file(model, path, fill, quantize, max_seq):
    """The model as a .qraf file that the reference's Transformer loads
    (src/nn/transformer.cpp:96-126, :320-400).  Each projection shape is one
    std::mt19937(42) N(0, 0.02) draw over the whole tensor, quantized once and
    written into every layer; the LM head is the draw of its shape, quantized, and
    the F32 embedding is that same draw; norms 1 + N(0, 0.1) (seed 45) and Qwen2's
    Q/K/V biases N(0, 0.1) (seed 46).  fill(seed, std, n) and quantize(dtype,
    w[n][k]) -> bytes are the caller's.  Returns the file's size in bytes."""
    from qraf_b200 import qraf_file as qf

    tok, dec = TOKEN_MODELS[model], DECODE_MODELS[model]
    dt, hidden, vocab, layers = tok["dtype"], tok["hidden"], tok["vocab"], tok["layers"]
    shapes = decode_shapes(model)
    w = qf.QrafFileWriter()
    for key, v in (("architecture", dec["arch"]), ("vocab_size", vocab), ("hidden_size", hidden),
                   ("num_layers", layers), ("num_heads", dec["heads"]), ("num_kv_heads", dec["kv_heads"]),
                   ("intermediate_size", dec["inter"]), ("max_seq_len", max_seq), ("rope_theta", 1000000.0),
                   ("rms_norm_eps", 1e-6)):
        (w.set_config_string if isinstance(v, str) else w.set_config)(key, v)
    scheme = w.add_quant_scheme(dt, 32, 1)
    qbytes = {}
    for n, k in sorted(set(shapes.values())):
        qbytes[(n, k)] = bytes(quantize(dt, fill(42, 0.02, n * k).reshape(n, k)))
    head = fill(42, 0.02, vocab * hidden).reshape(vocab, hidden)
    w.add_tensor("model.embed_tokens.weight", (vocab, hidden), qf.DTYPE_F32, head.tobytes())
    head_q = bytes(quantize(dt, head))
    del head
    norms = fill(45, 0.1, (2 * layers + 1) * hidden) + np.float32(1.0)
    q_dim, kv_dim = shapes["q_proj"][0], shapes["k_proj"][0]
    biases = fill(46, 0.1, layers * (q_dim + 2 * kv_dim))
    for l in range(layers):
        p = f"model.layers.{l}."
        w.add_tensor(p + "input_layernorm.weight", (hidden,), qf.DTYPE_F32, norms[2 * l * hidden:(2 * l + 1) * hidden])
        for name in ("q_proj", "k_proj", "v_proj", "o_proj"):
            w.add_tensor(p + f"self_attn.{name}.weight", shapes[name], dt, qbytes[shapes[name]], scheme)
        if dec["arch"] == "qwen2":
            off = l * (q_dim + 2 * kv_dim)
            for name, a, b in (("q_proj", 0, q_dim), ("k_proj", q_dim, q_dim + kv_dim),
                               ("v_proj", q_dim + kv_dim, q_dim + 2 * kv_dim)):
                w.add_tensor(p + f"self_attn.{name}.bias", (b - a,), qf.DTYPE_F32, biases[off + a:off + b])
        w.add_tensor(p + "post_attention_layernorm.weight", (hidden,), qf.DTYPE_F32,
                     norms[(2 * l + 1) * hidden:(2 * l + 2) * hidden])
        for name in ("gate_proj", "up_proj", "down_proj"):
            w.add_tensor(p + f"mlp.{name}.weight", shapes[name], dt, qbytes[shapes[name]], scheme)
    w.add_tensor("model.norm.weight", (hidden,), qf.DTYPE_F32, norms[2 * layers * hidden:])
    w.add_tensor("lm_head.weight", (vocab, hidden), dt, head_q, scheme)
    return w.write(path)


def decode_file_path(model):
    """A scratch path for the model file: /dev/shm when it has room, else the temp directory."""
    import shutil
    import tempfile

    tok = TOKEN_MODELS[model]
    need = 3 * tok["vocab"] * tok["hidden"] * 4 + tok["layers"] * 10 ** 8
    d = "/dev/shm" if os.path.isdir("/dev/shm") and shutil.disk_usage("/dev/shm").free > need else \
        tempfile.gettempdir()
    return os.path.join(d, f"qraf_bench_{model}_{os.getpid()}.qraf")


def decode_bytes_per_step(model, m, ctx, kv8=False):
    """Algorithmic HBM bytes of one decode step of M slots at position ctx: every
    quantized weight once, the F32 norms and biases, each slot's embedding row,
    its K and V over ctx + 1 positions of every layer (int8 codes and a scale per
    KV head with kv8), and the step's K/V writes.  Returns (total, weights)."""
    tok = TOKEN_MODELS[model]
    shapes = decode_shapes(model)
    bb = BLOCK_BYTES[tok["dtype"]]
    layers, hidden, vocab = tok["layers"], tok["hidden"], tok["vocab"]
    weights = layers * sum(n * (k // 32) * bb for n, k in shapes.values()) + vocab * (hidden // 32) * bb
    kv_dim = shapes["k_proj"][0]
    small = 4 * ((2 * layers + 1) * hidden + layers * (shapes["q_proj"][0] + 2 * kv_dim))
    kvh = DECODE_MODELS[model]["kv_heads"]
    per_pos = 2 * (kv_dim + 4 * kvh) if kv8 else 2 * 4 * kv_dim
    kv = m * layers * (ctx + 1) * per_pos + m * layers * per_pos
    return weights + small + m * hidden * 4 + kv, weights


def run_decode(args, model, m, ctx, kv8=False):
    """One STEP = one decode token for each of M slots through the whole model
    (qraf_cuda_decoder_step over a .qraf file written here), every slot at
    position ctx with ctx positions of its KV cache filled by earlier steps;
    captured once as a CUDA graph and replayed (every replay recomputes the
    position-ctx token and rewrites its K/V).  value = M x steps / device time."""
    import torch

    import qraf_b200 as qb

    if int(os.environ.get("WORLD_SIZE", "1")) > 1:
        raise SystemExit("decode workloads run on one GPU (replicas only)")
    torch.cuda.set_device(0)
    dev = torch.device("cuda", 0)
    qb.init(0)
    mode = {"exact": qb.MODE_EXACT, "fast": qb.MODE_FAST, "tc": qb.MODE_TC, "auto": qb.MODE_AUTO}[args.mode]

    def fill(seed, std, n):
        return qb.fill_normal(seed, 0.0, std, n)

    def quantize(dtype, w2d):
        return qb.quantize_rows(dtype, torch.from_numpy(w2d).to(dev), 32).cpu().numpy()

    path = decode_file_path(model)
    try:
        t_w = time.perf_counter()
        file_bytes = write_decode_file(model, path, fill, quantize, max_seq=ctx + 1)
        t_w = time.perf_counter() - t_w
        t_o = time.perf_counter()
        dec = qb.Decoder(path, max_slots=m, max_seq=ctx + 1, kv_int8=kv8)
        t_o = time.perf_counter() - t_o
        line = _decode_measure(args, model, m, ctx, dec, mode, kv8)
        line["config"].update({"file_bytes": file_bytes, "write_s": round(t_w, 2), "open_s": round(t_o, 2)})
        dec.close()
        line["cpu_baseline"] = decode_cpu_baseline(model, ctx, args.cpu_seconds, path) if args.cpu_seconds > 0 \
            else None
    finally:
        if os.path.exists(path):
            os.unlink(path)
    print(json.dumps(line), flush=True)


def _decode_measure(args, model, m, ctx, dec, mode, kv8=False):
    import torch

    import qraf_b200 as qb

    dev = torch.device("cuda", 0)
    tok = TOKEN_MODELS[model]
    dt, vocab = tok["dtype"], tok["vocab"]
    rng = np.random.default_rng(47)
    prompt = torch.from_numpy(rng.integers(0, vocab, size=(ctx + 1, m)).astype(np.int32)).to(dev)
    slots = torch.arange(m, dtype=torch.int32, device=dev)
    logits = torch.empty((m, vocab), dtype=torch.float32, device=dev)
    s = torch.cuda.Stream(dev)
    with torch.cuda.stream(s):
        for p in range(ctx):      # fill positions 0 .. ctx-1 of every slot's cache
            pos_p = torch.full((m,), p, dtype=torch.int32, device=dev)
            dec.step(prompt[p], pos_p, slots, mode=mode, logits=logits, stream=s)
    torch.cuda.synchronize(dev)
    tokens = prompt[ctx].clone()
    pos = torch.full((m,), ctx, dtype=torch.int32, device=dev)
    launches0 = qb.launch_count()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g, stream=s):
        dec.step(tokens, pos, slots, mode=mode, logits=logits, stream=s)
    per_step = qb.launch_count() - launches0
    for _ in range(max(3, args.warmup)):
        g.replay()
    torch.cuda.synchronize(dev)
    if qb.device_status() != qb.OK:
        raise SystemExit("device status not OK after warm-up")

    clocks = ClockSampler(0)
    t0, t1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    torch.cuda.synchronize(dev)
    clocks.start()
    with torch.cuda.stream(s):
        t0.record()
        for _ in range(args.steps):
            g.replay()
        t1.record()
    torch.cuda.synchronize(dev)
    clocks.stop()
    elapsed_ms = t0.elapsed_time(t1)

    # e2e: the user's call (Decoder.step, no graph) with the step's tokens copied in
    # from pinned host memory and its logits copied out, every step.
    tok_host = prompt[ctx].cpu().pin_memory()
    lg_host = torch.empty((m, vocab), dtype=torch.float32).pin_memory()
    e2e_steps = max(3, min(args.steps, 50))
    te = time.perf_counter()
    for _ in range(e2e_steps):
        with torch.cuda.stream(s):
            tokens.copy_(tok_host, non_blocking=True)
            dec.step(tokens, pos, slots, mode=mode, logits=logits, stream=s)
            lg_host.copy_(logits, non_blocking=True)
        s.synchronize()
    e2e_s = time.perf_counter() - te
    status = qb.device_status()
    step_s = elapsed_ms / 1e3 / args.steps
    bytes_step, weight_bytes = decode_bytes_per_step(model, m, ctx, kv8)
    peak, peak_src = measured_peaks()
    achieved = bytes_step / step_s / 1e9
    line = {
        "metric": DECODE_METRIC, "value": m * args.steps / (elapsed_ms / 1e3), "unit": "tokens/s", "n_gpus": 1,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": elapsed_ms / args.steps,
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
        "config": {"workload": args.workload, "model_shapes": model, "architecture": DECODE_MODELS[model]["arch"],
                   "M": m, "context": ctx, "layers": tok["layers"], "quant": "Q4_0" if dt == Q4 else "Q8_0",
                   "mode": args.mode, "weight_bytes_per_step": weight_bytes,
                   "kv_cache": "int8 codes + fp32 scale per (position, KV head) (QuantizedKVCache layout)" if kv8
                   else "f32",
                   "l2_policy": f"inputs larger than L2: {weight_bytes / 1e9:.1f} GB of distinct weights per step",
                   "weights": "N(0,0.02) std::mt19937(42) per projection shape, quantized on GPU (byte-exact Q*_0), "
                              "one copy per layer in the file; embedding = the LM head's draw in F32",
                   "step": "one token per slot at position ctx over ctx filled cache positions: embedding, per "
                           "layer RMSNorm+QKV+bias, attention with RoPE and the KV store, O + residual, "
                           "RMSNorm+SwiGLU, down + residual; final RMSNorm + LM head; one CUDA graph replay"},
        "e2e": {"value": m * e2e_steps / e2e_s, "unit": "tokens/s", "h2d_bytes_per_step": m * 4,
                "d2h_bytes_per_step": m * vocab * 4, "steps": e2e_steps,
                "path": "H2D of the step's tokens from pinned memory, Decoder.step (qraf_cuda_decoder_step, no "
                        "graph), D2H of the logits, stream sync, every step"},
        "gpu_launches": args.steps * per_step,
        "launches_per_step": per_step,
        "roofline": {"bound": "hbm", "achieved": achieved, "peak": peak, "unit": "GB/s", "frac": achieved / peak,
                     "traffic": None, "peak_source": peak_src,
                     "what": "weights + norms/biases + embedding rows + each slot's K/V over ctx+1 positions, "
                             "per step / time per step", "bytes_per_step": bytes_step},
        "clocks": clocks.summary(),
        "device_status": status,
    }
    del g
    return line


def decode_cpu_baseline(model, ctx, budget_s, path):
    """The reference's own Transformer::forward (oracle/_ref) on the model file at
    position ctx (its cache zeros below ctx: the cost is the same): forwards for
    about budget_s seconds, at least one."""
    import oracle

    if not oracle.reference_available():
        return None
    ref = oracle.RefTransformer(oracle.Reference(), path, TOKEN_MODELS[model]["vocab"])
    n, t0 = 0, time.perf_counter()
    while True:
        ref.forward(1 + n, ctx)
        n += 1
        if time.perf_counter() - t0 >= budget_s:
            break
    dt_s = time.perf_counter() - t0
    ref.close()
    return {"value": n / dt_s, "unit": "tokens/s", "cores": 1, "kind": "reference",
            "sample": f"{n} forward(token, {ctx}) calls of the reference's Transformer (oracle/_ref, "
                      f"single-threaded, as it runs on Linux) over the same .qraf file, {dt_s:.1f} s"}


def run_decode_reference(args, model, m, ctx, kv8=False):
    """The reference arm: its Transformer over the same file (written with the
    reference's own quantizer and RNG), one request at a time as its scheduler
    runs them; M slots cost M forwards, so tokens/s does not depend on M."""
    if int(os.environ.get("RANK", "0")) != 0:
        return
    import oracle

    if not oracle.reference_available():
        print(json.dumps({"impl": "reference", "unavailable": "oracle/_ref (the reference library) is not built"}))
        return
    qz = oracle.Reference()

    def fill(seed, std, n):
        return host_normal(seed, std, n)

    def quantize(dtype, w2d):
        return qz.quantize(dtype, np.ascontiguousarray(w2d).reshape(-1), 32)

    budget = max(5.0, min(120.0, 10.0 * args.steps))
    path = decode_file_path(model)
    try:
        write_decode_file(model, path, fill, quantize, max_seq=ctx + 1)
        cpu = decode_cpu_baseline(model, ctx, budget, path)
    finally:
        if os.path.exists(path):
            os.unlink(path)
    line = {"impl": "reference", "metric": DECODE_METRIC, "value": cpu["value"], "unit": "tokens/s", "n_gpus": 1,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": 1e3 / cpu["value"],
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
            "config": {"workload": args.workload, "model_shapes": model, "M": m, "context": ctx},
            "cpu_baseline": cpu,
            "e2e": {"value": cpu["value"], "unit": "tokens/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=2000)
    ap.add_argument("--warmup", type=int, default=20)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--workload", default=None,
                    help="default: q4_4096x4096 on one GPU; q4_28672x8192_shard (the 70B gate/up projection split "
                         "over the ranks) under torch.distributed.run")
    ap.add_argument("--no-1gpu-ref", dest="no_1gpu_ref", action="store_true",
                    help="sharded workloads on N > 1 GPUs: skip the unsharded one-GPU figure of the same projection")
    ap.add_argument("--mode", choices=["fast", "exact", "tc", "auto"], default=None,
                    help="projection arithmetic (default: fast; auto for decode workloads, which takes the "
                         "tensor-core tile from three slots)")
    ap.add_argument("--cpu-seconds", type=float, default=10.0)
    ap.add_argument("--no-overlap", dest="overlap", action="store_false",
                    help="launch matvecs strictly one after another (no programmatic dependent launch)")
    ap.add_argument("--no-norms", dest="norms", action="store_false",
                    help="token workloads on one GPU: no RMSNorm / bias folded into the projections")
    ap.add_argument("--no-swiglu", dest="swiglu", action="store_false",
                    help="token workloads on one GPU: gate and up as a plain two-weight launch, down reading gate "
                         "(default: one SwiGLU launch, down reading silu(gate) * up)")
    ap.add_argument("--no-multi", dest="multi", action="store_false",
                    help="token workloads: one launch per projection even where several share an input")
    ap.add_argument("--decode-layers", dest="decode_layers", type=int, default=None,
                    help="decode workloads: this many layers instead of the model's (a small case for profiling)")
    ap.add_argument("--allgather", choices=["fused", "nccl"], default="fused",
                    help="token workloads on N > 1 GPUs: all-gather fused into the kernel, or NCCL after it")
    args = ap.parse_args()
    args.workload = resolve_workload(args.workload, int(os.environ.get("WORLD_SIZE", "1")))
    dec = parse_decode_workload(args.workload)
    if args.mode is None:
        args.mode = "auto" if dec else "fast"
    if dec and args.decode_layers:
        TOKEN_MODELS[dec[0]] = dict(TOKEN_MODELS[dec[0]], layers=args.decode_layers)
    if dec:
        (run_decode_reference if args.impl == "reference" else run_decode)(args, *dec)
        return
    tok = parse_token_workload(args.workload)
    if tok:
        (run_token_reference if args.impl == "reference" else run_token)(args, *tok)
        return
    dt, n, k, m = parse_workload(args.workload)
    if args.impl == "reference":
        run_reference_arm(args, dt, n, k, m)
    elif is_shard_workload(args.workload):
        run_shard(args, dt, n, k, m)
    else:
        run_ours(args, dt, n, k, m)


if __name__ == "__main__":
    main()
