"""Benchmark of the B200 VoxCPM2 per-patch path (one JSON line on rank 0).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

Workload (the headline metric's configuration): one
Q8_0 x bf16 skinny product, M = 22 activation rows, K = 2048, N = 6144,
fp32 accumulation, bf16 output. A step is one product on one of 16 rotating
seeded weight copies (214 MB, larger than the 126 MB L2, so every step reads
its weights from HBM) into that copy's own output, through the product path a
caller of the reference's gemm.hpp takes: Bf16Gemm::Linear on one stream
(vx_gemm_linear_ex), which plans the product itself. Every launch waits for
the previous one (a dependent chain, the reference's own benchmark method);
programmatic dependent launch lets a launch start its weight stream before
the previous one ends. Steps are replayed from CUDA graphs of up to 100
launches (any --steps), so the host's launch rate does not bound the device.
With N > 1 (torchrun, one process per GPU) every rank runs its own products
(replicas, weak scaling); the value is all ranks' bytes over the slowest
rank's time.

`value` is the sustained HBM throughput in GB/s of algorithmic bytes
(weights + activations + bf16 output) of that chain. `stream` is the same
products as independent launches (each skips the programmatic wait, so one
overlaps the next) on the measured stream plan. `e2e` is the same metric
through the C ABI with host buffers: each step copies x from pinned memory,
runs the product and reads y back. `--impl reference` times the reference's
arithmetic on the host cores: the reference (HIP, AMD-only) cannot be built
here, so the CPU oracle port (oracle/, a float32 transcription of its product
kernel) stands in.
"""

from __future__ import annotations

import argparse
import ctypes
import json
import math
import os
import statistics
import subprocess
import sys
import threading
import time
from pathlib import Path

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

ROWS, IN, OUT = 22, 2048, 6144
WEIGHT_BYTES = OUT * IN * 34 // 32          # 13,369,344
X_BYTES = ROWS * IN * 2                     # 90,112
Y_BYTES = ROWS * OUT * 2                    # 270,336 (bf16 output)
STEP_BYTES = WEIGHT_BYTES + X_BYTES + Y_BYTES  # 13,729,792
COPIES = 16
GRAPH_LAUNCHES = 100
E2E_STREAMS = 16  # streams the end-to-end steps rotate over (COPIES % E2E_STREAMS == 0)
E2E_GRAPH_STEPS = 32  # end-to-end steps per stream in one CUDA graph
# Measured best plan for a stream of independent launches of this shape.
STREAM_VARIANT, STREAM_SPLITS = 14, 1
METRIC = "Q8_0 skinny-product HBM GB/s (M=22, K=2048, N=6144, bf16 out)"


def parse():
    p = argparse.ArgumentParser()
    p.add_argument("--gpus", type=int, default=1)
    p.add_argument("--steps", type=int, default=400_000)
    p.add_argument("--warmup", type=int, default=20_000)
    p.add_argument("--impl", choices=["ours", "reference"], default="ours")
    p.add_argument("--case", choices=["product", "dit", "wide", "batch", "matmul", "vae", "step"], default=None,
                   help="run a few launches of one kernel for a profiler and exit (no JSON line)")
    p.add_argument("--max-ctas", type=int, default=0,
                   help="with --case: cap the persistent kernels' CTAs (vx_set_persistent_max_ctas)")
    p.add_argument("--non-cooperative", action="store_true",
                   help="with --case: launch the persistent kernels without the cooperative attribute "
                        "(vx_set_persistent_cooperative(0)), for profilers")
    p.add_argument("--slots", type=int, default=8,
                   help="with --case batch: active slots of the GeneratorBatch (the bench's box_batched runs 16)")
    return p.parse_args()


# ---------------------------------------------------------------- distributed

def init_dist(n_gpus: int):
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world > 1:
        import datetime

        import torch
        import torch.distributed as dist

        torch.cuda.set_device(local)
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                device_id=torch.device("cuda", local))
    return world, rank, local


def barrier(world):
    if world > 1:
        import torch.distributed as dist

        dist.barrier()


def _all_reduce(value: float, op_name: str) -> float:
    """One value reduced over the ranks (a CUDA tensor under NCCL, a host
    tensor under gloo)."""
    import torch
    import torch.distributed as dist

    device = "cpu" if dist.get_backend() == "gloo" else "cuda"
    t = torch.tensor([value], dtype=torch.float64, device=device)
    dist.all_reduce(t, op=getattr(dist.ReduceOp, op_name))
    return float(t.item())


def max_over_ranks(world, value: float) -> float:
    return value if world == 1 else _all_reduce(value, "MAX")


def sum_over_ranks(world, value: float) -> float:
    return value if world == 1 else _all_reduce(value, "SUM")


# ---------------------------------------------------------------- clocks

class ClockSampler:
    """nvidia-smi samples of SM clock and throttle reasons while running."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index: int):
        self.gpu_index = gpu_index
        self.proc = None
        self.lines: list[str] = []
        self.thread = None

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", "-i", str(self.gpu_index), f"--query-gpu={self.FIELDS}",
                 "--format=csv,noheader,nounits", "-lms", "50"],
                stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.thread = threading.Thread(target=self._read, daemon=True)
            self.thread.start()
            time.sleep(0.15)
        except (OSError, FileNotFoundError):
            self.proc = None
        return self

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    def __exit__(self, *exc):
        if self.proc is not None:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()

    def summary(self) -> dict:
        sm, mx, reasons = [], [], set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for line in self.lines:
            parts = [p.strip() for p in line.split(",")]
            if len(parts) < 9:
                continue
            try:
                sm.append(float(parts[1]))
                mx.append(float(parts[2]))
            except ValueError:
                continue
            for name, flag in zip(names, parts[5:9]):
                if flag.lower() == "active":
                    reasons.add(name)
        if not sm:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": [], "samples": 0}
        return {"sm_mhz": statistics.median(sm), "sm_max_mhz": max(mx), "reasons": sorted(reasons),
                "samples": len(sm)}


# ---------------------------------------------------------------- shared

def measured_peak():
    path = ROOT / "MEASURED_PEAKS.json"
    if path.exists():
        data = json.loads(path.read_text())
        return float(data["hbm_gbs"]), "measured"
    return 6650.0, "fallback"


def profiled_traffic():
    """DRAM bytes per launch of the product kernel from the committed ncu
    summary (profiles/traffic.json), or None."""
    path = ROOT / "profiles" / "traffic.json"
    if not path.exists():
        return None
    data = json.loads(path.read_text())
    return data.get("q8_product_m22_k2048_n6144", {}).get("dram_bytes_per_launch")


def cpu_sample(threads: int, budget_s: float):
    """The oracle's float32 product transcription on a slice of config 0,
    repeated for about `budget_s` seconds; returns (GB/s, description)."""
    import numpy as np

    import oracle

    rows_out = 1024
    blocks = oracle.random_q8_0(1, 0, rows_out, IN)
    rng = np.random.default_rng(0)
    x = oracle.bf16_bits(rng.normal(0, 1, (ROWS, IN)).astype(np.float32))
    y = np.zeros((ROWS, rows_out), np.float32)
    oracle.linear(x, oracle.Q8_0, blocks, ROWS, IN, rows_out, y=y, threads=threads)
    start = time.perf_counter()
    reps = 0
    while True:
        oracle.linear(x, oracle.Q8_0, blocks, ROWS, IN, rows_out, y=y, threads=threads)
        reps += 1
        elapsed = time.perf_counter() - start
        if elapsed >= budget_s:
            break
    bytes_per = rows_out * IN * 34 // 32 + X_BYTES + ROWS * rows_out * 2
    return bytes_per * reps / elapsed / 1e9, (
        f"{reps} x (M={ROWS}, K={IN}, N={rows_out} of {OUT}) fp32 per-block transcription, "
        f"{elapsed:.1f} s")


def cpu_model() -> str:
    """The host CPU's model name (from /proc/cpuinfo), or the platform's."""
    try:
        for line in open("/proc/cpuinfo"):
            if line.startswith("model name"):
                return line.split(":", 1)[1].strip()
    except OSError:
        pass
    import platform

    return platform.processor() or platform.machine()


def cpu_host_baselines() -> dict:
    """The host-side references the path's tests check against, timed on
    this box's host cores (reported only):
    - the scalar double-precision product of config 0 on one thread
      (tests/products_test.cpp:117-134);
    - the fp32 per-block transcription of the reference's Q8_0 product
      (kernels/wmma_products.hip:201-214) on a slice of config 0, on one
      thread and on all host threads;
    - one DiT patch of config 2 (12 layers, 10 Euler steps, 9 evaluations,
      CFG 2.0, seeded Q8_0 weights) through the oracle's restatement on all
      cores (generator.cpp:297-324, 424-460);
    - one full per-patch step of config 3 (28-layer LM, 8-layer residual
      LM, 12-layer encoder and DiT, context 512, bf16 cache) through the
      oracle's restatement on all cores (generator.cpp:424-513)."""
    import numpy as np

    import oracle
    from oracle.model import OracleGenerator
    from voxcpm_b200.generator import released_config

    threads = os.cpu_count() or 1
    rng = np.random.default_rng(0)
    blocks = oracle.random_q8_0(1, 0, OUT, IN)
    x = oracle.bf16_bits(rng.normal(0, 1, (ROWS, IN)).astype(np.float32))
    start = time.perf_counter()
    oracle.product_exact(x, oracle.Q8_0, blocks, ROWS, IN, OUT, threads=1)
    product_s = time.perf_counter() - start
    one_value, one_desc = cpu_sample(1, 3.0)
    all_value, all_desc = cpu_sample(threads, 3.0)

    c = released_config()
    c.max_length = 640
    c.vocab = 1024
    ref = OracleGenerator(c, seed=7, threads=threads, bf16_cache=True)
    mu = rng.normal(0, 1, 2 * c.dit.hidden).astype(np.float32)
    cond = rng.normal(0, 1, (c.patch_size, c.feat_dim)).astype(np.float32)
    noise = rng.normal(0, 1, (c.patch_size, c.feat_dim)).astype(np.float32)
    start = time.perf_counter()
    ref.dit_patch(mu, cond, noise, 10, 2.0)
    patch_s = time.perf_counter() - start
    # The step at context 512: caches hold seeded keys and values for the
    # 512 prompt positions (the step's work does not depend on their values).
    for cache in (ref.base_cache, ref.residual_cache):
        cache.k[:, :, :512] = rng.normal(0, 1, cache.k[:, :, :512].shape).astype(np.float32)
        cache.v[:, :, :512] = rng.normal(0, 1, cache.v[:, :, :512].shape).astype(np.float32)
    ref.position = 512
    ref.lm_hidden = rng.normal(0, 1, c.lm.hidden).astype(np.float32)
    ref.residual_hidden = rng.normal(0, 1, c.lm.hidden).astype(np.float32)
    start = time.perf_counter()
    ref.step(noise, 10, 2.0)
    step_s = time.perf_counter() - start
    host = {"cores": threads, "cpu": cpu_model()}
    return {
        "host": host,
        "double_sum_product": {"us": product_s * 1e6, "gbs": STEP_BYTES / product_s / 1e9, "cores": 1,
                               "kind": "port",
                               "sample": f"one full config-0 product (M={ROWS}, K={IN}, N={OUT}), "
                                         "double-precision sums, one thread"},
        "fp32_product_one_thread": {"gbs": one_value, "cores": 1, "kind": "port", "sample": one_desc},
        "fp32_product_all_threads": {"gbs": all_value, "cores": threads, "kind": "port",
                                     "sample": all_desc},
        "dit_patch": {"us": patch_s * 1e6, "cores": threads, "kind": "port",
                      "sample": "one config-2 DiT patch (10 Euler steps, CFG 2.0) through the oracle's "
                                "restatement, all host cores"},
        "step": {"ms": step_s * 1e3, "audio_s_per_s": PATCH_AUDIO_S / step_s, "cores": threads,
                 "kind": "port",
                 "sample": "one config-3 per-patch step at context 512 (bf16 cache) through the "
                           "oracle's restatement, all host cores"},
    }


# ---------------------------------------------------------------- reference arm

def run_reference(args, world, rank):
    if rank != 0:
        return
    import numpy as np

    import oracle

    threads = os.cpu_count() or 1
    # One step = the product on a slice of the output rows, sized so that the
    # whole --warmup + --steps run stays within about a minute.
    probe_rows = 256
    blocks_probe = oracle.random_q8_0(1, 0, probe_rows, IN)
    rng = np.random.default_rng(0)
    x = oracle.bf16_bits(rng.normal(0, 1, (ROWS, IN)).astype(np.float32))
    y = np.zeros((ROWS, probe_rows), np.float32)
    t0 = time.perf_counter()
    oracle.linear(x, oracle.Q8_0, blocks_probe, ROWS, IN, probe_rows, y=y, threads=threads)
    per_row = max((time.perf_counter() - t0) / probe_rows, 1e-9)
    total = max(args.steps + args.warmup, 1)
    rows_out = int(max(16, min(OUT, 60.0 / total / per_row)) // 16 * 16)
    blocks = oracle.random_q8_0(1, 0, rows_out, IN)
    y = np.zeros((ROWS, rows_out), np.float32)
    for _ in range(args.warmup):
        oracle.linear(x, oracle.Q8_0, blocks, ROWS, IN, rows_out, y=y, threads=threads)
    t0 = time.perf_counter()
    for _ in range(args.steps):
        oracle.linear(x, oracle.Q8_0, blocks, ROWS, IN, rows_out, y=y, threads=threads)
    elapsed = time.perf_counter() - t0
    step_bytes = rows_out * IN * 34 // 32 + X_BYTES + ROWS * rows_out * 2
    value = step_bytes * args.steps / elapsed / 1e9
    sample = (f"each step: M={ROWS}, K={IN}, N={rows_out} of {OUT} output rows "
              f"(float32 per-block transcription of the reference's Q8_0 product)")
    line = {
        "impl": "reference", "metric": METRIC, "value": value, "unit": "GB/s", "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": elapsed / max(args.steps, 1) * 1e3, "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "f32", "data": "synthetic (seeded)",
        "config": {"workload": "q8_product_m22_k2048_n6144", "rows": ROWS, "in": IN, "out": OUT},
        "cpu_baseline": {"value": value, "unit": "GB/s", "cores": threads, "kind": "port",
                         "sample": sample},
        "e2e": {"value": value, "unit": "GB/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
        "note": "the reference is HIP for AMD gfx1151 and cannot be built here (no hipcc/ROCm, no "
                "Gufo SDK); this arm times the CPU oracle port of its product on the host cores",
    }
    print(json.dumps(line), flush=True)


# ---------------------------------------------------------------- our arm

def run_ours(args, world, rank, local):
    import numpy as np
    import torch

    from voxcpm_b200 import _lib
    from voxcpm_b200 import kernels as K

    device = torch.device("cuda", local)
    torch.cuda.set_device(device)
    lib = _lib.load()
    stream = torch.cuda.Stream(device)

    # Seeded weight copies (distinct per copy and rank), repacked into tiles.
    tiles = []
    for c in range(COPIES):
        blocks = torch.from_numpy(K.RandomQ8_0(1000 + rank, c, OUT, IN)).to(device)
        t = torch.empty(K.Q8TilesBytes(OUT, IN), dtype=torch.uint8, device=device)
        K.Q8_0ToTiles(blocks, OUT, IN, t, stream=stream)
        tiles.append(t)
        del blocks
    rng = np.random.default_rng(rank)
    x_host = torch.from_numpy(rng.normal(0, 1, (ROWS, IN)).astype(np.float32)).to(torch.bfloat16)
    x = x_host.to(device)
    ys = [torch.empty(ROWS, OUT, dtype=torch.bfloat16, device=device) for _ in range(COPIES)]
    y = ys[0]
    torch.cuda.synchronize()

    s = stream.cuda_stream
    x_ptr = x.data_ptr()
    y_ptrs = [t.data_ptr() for t in ys]
    tile_ptrs = [t.data_ptr() for t in tiles]
    # The product path a caller of the reference's gemm.hpp takes:
    # Bf16Gemm::Linear on the stream (vx_gemm_linear_ex, bf16 output), which
    # plans the product itself (the spread kernel through the gemm's own split
    # scratch); every launch waits for the previous one (a dependent chain).
    gemm = lib.vx_gemm_create(s)
    if not gemm:
        raise RuntimeError(lib.vx_last_error().decode())
    # Beside it, the measured plan for streams of independent launches.
    stream_plan = _lib.WmmaPlan(STREAM_SPLITS, -(-(IN // 32) // STREAM_SPLITS), 0, 0, STREAM_VARIANT)

    def launch(i, mode, x_at=x_ptr, on=s):
        if mode == "chain":
            st = lib.vx_gemm_linear_ex(gemm, x_at, _lib.WEIGHTS_Q8_TILES, tile_ptrs[i % COPIES],
                                       y_ptrs[i % COPIES], _lib.OUT_BF16, ROWS, IN, OUT, 0)
        else:
            st = lib.vx_product_ex(_lib.WEIGHTS_Q8_TILES, x_at, tile_ptrs[i % COPIES], y_ptrs[i % COPIES],
                                   _lib.OUT_BF16, ROWS, IN, OUT, _lib.PRODUCT_INDEPENDENT,
                                   ctypes.byref(stream_plan), on)
        if st != 0:
            raise RuntimeError(lib.vx_last_error().decode())

    # CUDA graphs of the launches (any step count: graphs of GRAPH_LAUNCHES
    # launches and one of the remainder), captured before any timing.
    graphs = {}

    def graph(mode, count):
        key = (mode, count)
        if key not in graphs:
            with torch.cuda.stream(stream):
                for i in range(3):
                    launch(i, mode)
                stream.synchronize()
                g = torch.cuda.CUDAGraph()
                with torch.cuda.graph(g, stream=stream):
                    for i in range(count):
                        launch(i, mode)
            graphs[key] = g
        return graphs[key]

    def run_steps(n, mode):
        full, rest = divmod(n, GRAPH_LAUNCHES)
        with torch.cuda.stream(stream):
            for _ in range(full):
                graph(mode, GRAPH_LAUNCHES).replay()
            if rest:
                graph(mode, rest).replay()

    warmup = max(args.warmup, 3)
    # The stream line's own launch count: at a few launches a stream of
    # independent products measures its ramp, not its rate.
    stream_steps = max(args.steps, STREAM_MIN_LAUNCHES)
    for mode, steps in (("chain", args.steps), ("stream", stream_steps)):
        for n in (warmup, steps):
            full, rest = divmod(n, GRAPH_LAUNCHES)
            if full:
                graph(mode, GRAPH_LAUNCHES)
            if rest:
                graph(mode, rest)
    torch.cuda.synchronize()

    start = torch.cuda.Event(enable_timing=True)
    stop = torch.cuda.Event(enable_timing=True)

    def timed(mode, steps):
        run_steps(warmup, mode)
        torch.cuda.synchronize()
        barrier(world)
        torch.cuda.synchronize()
        with torch.cuda.stream(stream):
            # A device-side pause before the start event, so the host has
            # enqueued the timed graphs by the time the stream reaches it and
            # host submission stays out of the timed region.
            torch.cuda._sleep(200_000)
        start.record(stream)
        run_steps(steps, mode)
        stop.record(stream)
        torch.cuda.synchronize()
        barrier(world)
        return start.elapsed_time(stop)

    visible = os.environ.get("CUDA_VISIBLE_DEVICES")
    sampler = ClockSampler(int(visible.split(",")[local]) if visible else local)
    with sampler:
        ms = timed("chain", args.steps)
    ms_max = max_over_ranks(world, ms)
    total_bytes = sum_over_ranks(world, STEP_BYTES * args.steps)
    value = total_bytes / (ms_max / 1e3) / 1e9
    per_launch_s = ms / 1e3 / max(args.steps, 1)
    achieved = STEP_BYTES / per_launch_s / 1e9
    # The same steps as a stream of independent launches (each skips the
    # programmatic wait, so one overlaps the next) on the measured stream
    # plan.
    extra = {}
    for mode in ("stream",):
        m_ms = max_over_ranks(world, timed(mode, stream_steps))
        extra[mode] = (m_ms, sum_over_ranks(world, STEP_BYTES * stream_steps) / (m_ms / 1e3) / 1e9)
    lib.vx_gemm_destroy(gemm)
    graphs.clear()
    bits = K.DeviceError()
    if bits:
        raise RuntimeError(f"device wait timed out: bits {bits:#x}")

    # e2e through the C ABI with host buffers: every step is one
    # vx_gemm_linear_host call (Bf16Gemm::Linear with host activations and
    # output), which stages x in from pinned memory, runs the product on the
    # same plan as the value above and stages y out to pinned memory, the
    # transfers by SM loads and stores over PCIe. Steps rotate over
    # E2E_STREAMS streams, each with its own gemm, x and pinned y, so one
    # step's copies overlap other steps' products; each stream replays a CUDA
    # graph of its E2E_GRAPH_STEPS steps (the copies and the product of every
    # step are in the graph), so the host's per-call cost stays out of the
    # timed region as in the value above.
    lanes = [torch.cuda.Stream(device) for _ in range(E2E_STREAMS)]
    lane_gemms = [lib.vx_gemm_create(lane.cuda_stream) for lane in lanes]
    if not all(lane_gemms):
        raise RuntimeError(lib.vx_last_error().decode())
    x_lanes = [torch.empty_like(x) for _ in range(E2E_STREAMS)]
    x_pinned = x_host.pin_memory()
    y_pinned = [torch.empty(ROWS, OUT, dtype=torch.bfloat16).pin_memory() for _ in range(E2E_STREAMS)]

    def e2e_step(i, k):
        st = lib.vx_gemm_linear_host(lane_gemms[k], x_pinned.data_ptr(), x_lanes[k].data_ptr(),
                                     _lib.WEIGHTS_Q8_TILES, tile_ptrs[i % COPIES], y_ptrs[i % COPIES],
                                     y_pinned[k].data_ptr(), _lib.OUT_BF16, ROWS, IN, OUT, 0)
        if st != 0:
            raise RuntimeError(lib.vx_last_error().decode())

    e2e_graphs = []
    for k in range(E2E_STREAMS):
        with torch.cuda.stream(lanes[k]):
            e2e_step(k, k)
            lanes[k].synchronize()
            g = torch.cuda.CUDAGraph()
            with torch.cuda.graph(g, stream=lanes[k]):
                for j in range(E2E_GRAPH_STEPS):
                    e2e_step(k + E2E_STREAMS * j, k)
            e2e_graphs.append(g)
    e2e_reps = max(2, min(args.steps // (100 * E2E_GRAPH_STEPS), 20))
    e2e_steps = e2e_reps * E2E_STREAMS * E2E_GRAPH_STEPS
    main_stream = torch.cuda.current_stream()

    def e2e_run(reps):
        for lane in lanes:
            lane.wait_event(e_start)
        for _ in range(reps):
            for k in range(E2E_STREAMS):
                with torch.cuda.stream(lanes[k]):
                    e2e_graphs[k].replay()
        for lane in lanes:
            ev = torch.cuda.Event()
            ev.record(lane)
            main_stream.wait_event(ev)

    e_start = torch.cuda.Event(enable_timing=True)
    e_stop = torch.cuda.Event(enable_timing=True)
    e_start.record(main_stream)
    e2e_run(1)  # warm-up
    torch.cuda.synchronize()
    barrier(world)
    e_start.record(main_stream)
    e2e_run(e2e_reps)
    e_stop.record(main_stream)
    torch.cuda.synchronize()
    e_ms = max_over_ranks(world, e_start.elapsed_time(e_stop))
    e2e_value = sum_over_ranks(world, STEP_BYTES * e2e_steps) / (e_ms / 1e3) / 1e9
    for k in range(E2E_STREAMS):  # the last step of stream k wrote ys[k]
        if not torch.equal(y_pinned[k], ys[(k + E2E_STREAMS * (E2E_GRAPH_STEPS - 1)) % COPIES].cpu()):
            raise RuntimeError("end-to-end output copy differs from the device output")
    del e2e_graphs
    torch.cuda.synchronize()
    for g in lane_gemms:
        lib.vx_gemm_destroy(g)

    clocks = sampler.summary()
    generator = measure_generator(rank, world)
    if rank != 0:
        return
    peak, peak_kind = measured_peak()
    sweep = measure_sweep(peak)
    cpu_value, cpu_desc = cpu_sample(os.cpu_count() or 1, 10.0)
    host_baselines = cpu_host_baselines() if (world or 1) == 1 else None
    plan = K.PlanWmma(ROWS, IN, OUT, 0)
    line = {
        "metric": METRIC, "value": value, "unit": "GB/s", "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": ms_max / max(args.steps, 1),
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "bf16",
        "data": "synthetic (seeded Q8_0 weights: q uniform [-127,127], fp16 scales |N(0,0.02)|/127; "
                "x ~ N(0,1) bf16)",
        "config": {"workload": "q8_product_m22_k2048_n6144_bf16out", "rows": ROWS, "in": IN,
                   "out": OUT, "accumulate": "fp32", "weight_copies": COPIES,
                   "l2": f"inputs larger than L2: {COPIES} rotating weight copies "
                         f"({COPIES * WEIGHT_BYTES / 1e6:.0f} MB)",
                   "api": "Bf16Gemm::Linear (vx_gemm_linear_ex, bf16 output) on one stream: the "
                          "library plans each product itself",
                   "launch": f"a dependent chain (each product waits for the previous one; programmatic "
                             f"dependent launch lets its weight stream start early), replayed from CUDA "
                             f"graphs of up to {GRAPH_LAUNCHES} launches; each product its own weight "
                             f"copy and output",
                   "plan": {"variant": plan.variant, "splits": plan.splits,
                            "blocks_per_split": plan.blocks_per_split,
                            "kernel": "ProductKernel, whole-reduction CTAs of 48 weight rows (12 warps: "
                                      "3 groups x 4 ways), mma.sync tile math, no cluster, no scratch"},
                   "timed_region": "a device-side sleep before the start event keeps host graph "
                                   "submission out of it",
                   "parallelism": f"replicas x{world}"},
        "stream": {"value": extra["stream"][1], "unit": "GB/s",
                   "ms_per_step": extra["stream"][0] / stream_steps,
                   "launches": stream_steps,
                   "frac": extra["stream"][1] / world / peak,
                   "launch": "independent products (no programmatic wait: each overlaps the one "
                             "before), measured stream plan",
                   "plan": {"splits": stream_plan.splits, "blocks_per_split": stream_plan.blocks_per_split,
                            "variant": stream_plan.variant}},
        "roofline": {"bound": "hbm", "achieved": achieved, "peak": peak, "unit": "GB/s",
                     "frac": achieved / peak, "traffic": profiled_traffic(),
                     "peak_source": f"{peak_kind} hbm_gbs (copy rate)",
                     "frac_of_8TBps": achieved / 8000.0,
                     "algorithmic_bytes_per_launch": STEP_BYTES},
        "cpu_baseline": {"value": cpu_value, "unit": "GB/s", "cores": os.cpu_count() or 1,
                         "kind": "port", "sample": cpu_desc},
        "cpu_baselines": host_baselines,
        "e2e": {"value": e2e_value, "unit": "GB/s", "h2d_bytes_per_step": X_BYTES,
                "d2h_bytes_per_step": Y_BYTES, "steps": e2e_steps, "streams": E2E_STREAMS,
                "api": "vx_gemm_linear_host (Bf16Gemm::Linear with host buffers, the value's plan): "
                       "pinned host x staged in and y staged out by SM loads and stores over PCIe "
                       "every step",
                "launch": f"one CUDA graph of {E2E_GRAPH_STEPS} steps per stream (the three "
                          f"launches of every step inside), replayed {e2e_reps} times"},
        "sweep": {"rows": sweep, "metric": "GB/s of algorithmic bytes (weights + x + fp32 y) per "
                  "Bf16Gemm::Linear call; err = max |y - exact| / sum |x w| (limit 1e-5)",
                  "launch": "dependent chain over rotating weight copies (more than L2), CUDA graph",
                  "config": "BASELINE config 1"},
        "gpu_launches": args.steps,
        "clocks": clocks,
        **generator,
    }
    print(json.dumps(line), flush=True)


# ---------------------------------------------------------------- DiT patch and step

DIT_LAYER_BYTES = (2560 * 1024 + 1024 * 2048 + 8192 * 1024 + 1024 * 4096) * 34 // 32  # 18,382,848
DIT_EVAL_BYTES = 12 * DIT_LAYER_BYTES + 2 * 1024 * 64 * 34 // 32  # 220,733,440
DIT_PATCH_BYTES = 9 * DIT_EVAL_BYTES  # 1,986,600,960: 10 Euler steps, 9 evaluations
PATCH_AUDIO_S = 0.16  # 4 latent frames x 640 samples at 16 kHz
# Config 3 algorithmic bytes per patch: the Q8_0 weights read once
# (4,034,512,896 B) plus the bf16 KV cache at context 512 (18.9 MB).
STEP_BYTES_CONFIG3 = 4_034_512_896 + 18_874_368


def measure_vae(gen, c, tokens, audio, feats, noises, warm: int, rank: int, decodes: int = 20) -> dict:
    """The AudioVAE decode on its own stream (vae.cpp:382-516): one patch of
    latents (4 frames -> 7680 samples at 48 kHz) per decoding on the
    released decoder with seeded weights; then the config-3 step loop with
    each patch's latent decoded behind the next step, as synthesizer.cpp:
    283-307 drives it (Step, Collect the previous patch, Enqueue this one on
    the latent event)."""
    import numpy as np
    import torch

    from voxcpm_b200.vae import AudioVae, default_vae_config

    vae = AudioVae(default_vae_config(), seed=200 + rank)
    vae_stream = torch.cuda.ExternalStream(vae.stream())
    frames = c.patch_size
    x = torch.randn(frames, c.feat_dim, device="cuda")
    torch.cuda.synchronize()
    a = torch.cuda.Event(enable_timing=True)
    b = torch.cuda.Event(enable_timing=True)
    times = []
    for i in range(decodes + 3):
        a.record(vae_stream)
        vae.Enqueue(x.data_ptr(), frames)
        b.record(vae_stream)
        samples = vae.Collect()
        if i >= 3:
            times.append(a.elapsed_time(b) * 1e3)
    decode_us = float(np.median(times))
    # Steps with the decode behind them.
    vae.Reset()
    gen.Prefill(tokens, 1 - audio, audio, feats)
    wall_ms, decoded = [], 0
    for n in noises:
        t0 = time.perf_counter()
        gen.Step(n, 10, 2.0)
        decoded += vae.Collect().size
        vae.Enqueue(gen.latent(), frames, gen.latent_event())
        wall_ms.append((time.perf_counter() - t0) * 1e3)
    decoded += vae.Collect().size
    if decoded != len(noises) * frames * vae.decode_hop or samples.size != frames * vae.decode_hop:
        raise RuntimeError("AudioVAE returned the wrong number of samples")
    with_vae_ms = float(np.median(wall_ms[warm:]))
    patch_audio_s = frames * vae.decode_hop / 48000
    vae.close()
    return {"decode_us_per_patch": decode_us, "audio_s_per_s_decode_only": patch_audio_s / (decode_us / 1e6),
            "step_wall_ms_with_vae": with_vae_ms,
            "audio_s_per_s_with_vae": patch_audio_s / (with_vae_ms / 1e3),
            "hbm_floor_us": VAE_WEIGHT_BYTES / (measured_peak()[0] * 1e9) * 1e6,
            "fp32_floor_us": VAE_FLOPS_PER_FRAME * frames / 74.4e12 * 1e6,
            "fp32_peak_note": "74.4 TFLOP/s: 148 SMs x 128 fp32 lanes x 2 x 1.965 GHz (nominal)",
            "config": "AudioVAE V2 decoder: latent 64, decoder 2048, rates 8 6 5 2 2 2, 48 kHz, float32, "
                      "seeded weights; its own stream, fed by the generator's latent event",
            "timing": f"device events around Enqueue on the AudioVAE stream, median of {decodes}; with "
                      "steps: wall time per config-3 step including Collect + Enqueue"}


# The released decoder's product weights in float32 (read once per
# decoding: input pointwise, per block the transposed convolution and three
# unit pointwise matrices) and its product flops per latent frame (2 x the
# multiply-adds; a block's input has `hop` frames per latent frame).
VAE_RATES = (8, 6, 5, 2, 2, 2)
VAE_WEIGHT_BYTES = 4 * (2048 * 64 + sum(
    (2048 >> b) * (1024 >> b) * 2 * r + 3 * (1024 >> b) ** 2 for b, r in enumerate(VAE_RATES)))
VAE_FLOPS_PER_FRAME = 2 * (64 * 2048 + sum(
    hop * 2 * (2048 >> b) * r * (1024 >> b) + 3 * hop * r * (1024 >> b) ** 2
    for b, (r, hop) in enumerate(zip(VAE_RATES, (1, 8, 48, 240, 480, 960)))))


STREAM_MIN_LAUNCHES = 2000  # the stream line's launches at least (a few ms)


BOX_REQUESTS = 64        # independent requests over the box
BOX_PATCHES = 63         # patches per request (about 10 s of audio)
BOX_SLOTS = 32           # requests generated together per GPU (GeneratorBatch slots, at most)


SWEEP_ROWS = (1, 2, 8, 22, 64, 128)
SWEEP_SHAPES = ((1024, 3072), (1024, 1024), (2048, 6144), (6144, 2048), (2048, 2560))
SWEEP_L2_BYTES = 160 << 20  # rotating weight copies per shape: more than the 126 MB L2


def measure_sweep(peak_gbs: float) -> list:
    """every M x (K, N) with Q8_0 tiles and bf16 rows
    (q uniform in [-127, 127] with fp16 scales |N(0, 0.02)|/127; bf16
    weights ~N(0, 0.02); x ~ N(0, 1) bf16), through Bf16Gemm::Linear (the
    reference's dispatch: 32-row products, larger row counts in 32-row
    chunks), fp32 output. Time: a dependent chain of launches over rotating
    weight copies, replayed from a CUDA graph. Error: max |y - exact| /
    sum |x w| per output against a float64 product of the same operands."""
    import numpy as np
    import torch

    from voxcpm_b200 import _lib
    from voxcpm_b200 import kernels as K
    from voxcpm_b200.gemm import Bf16Gemm, Matrix

    stream = torch.cuda.Stream()
    gemm = Bf16Gemm(stream)
    out_rows = []
    for (k, n) in SWEEP_SHAPES:
        blocks = K.RandomQ8_0(77, n, n, k)
        raw = blocks.reshape(-1, 34)
        scales = torch.from_numpy(raw[:, :2].copy().view(np.float16).astype(np.float64)).cuda()
        q = torch.from_numpy(raw[:, 2:].copy().view(np.int8).astype(np.float64)).cuda()
        w_q8_exact = (q * scales).reshape(n, k)
        tiles = torch.empty(K.Q8TilesBytes(n, k), dtype=torch.uint8, device="cuda")
        K.Q8_0ToTiles(torch.from_numpy(blocks).cuda(), n, k, tiles)
        w_bf16 = (torch.randn(n, k, device="cuda") * 0.02).to(torch.bfloat16)
        for fmt, w_one, exact_w, w_bytes in (
                (_lib.WEIGHTS_Q8_TILES, tiles, w_q8_exact, n * k * 34 // 32),
                (_lib.WEIGHTS_BF16, w_bf16.view(torch.int16), w_bf16.double(), n * k * 2)):
            copies = max(2, min(160, -(-SWEEP_L2_BYTES // w_bytes)))
            ws = [w_one.clone() for _ in range(copies)]
            for m in SWEEP_ROWS:
                x = torch.randn(m, k, device="cuda").to(torch.bfloat16)
                ys = [torch.empty(m, n, dtype=torch.float32, device="cuda") for _ in range(2)]
                torch.cuda.synchronize()
                with torch.cuda.stream(stream):
                    gemm.Linear(x.view(torch.int16), Matrix(fmt, ws[0]), ys[0], m, k, n, False)
                    stream.synchronize()
                    exact = x.double() @ exact_w.t()
                    mag = x.double().abs() @ exact_w.abs().t()
                    err = float(((ys[0].double() - exact).abs() / mag.clamp_min(1e-300)).max())
                    launches = max(copies, 20)
                    g = torch.cuda.CUDAGraph()
                    with torch.cuda.graph(g, stream=stream):
                        for i in range(launches):
                            gemm.Linear(x.view(torch.int16), Matrix(fmt, ws[i % copies]), ys[i % 2],
                                        m, k, n, False)
                    g.replay()
                    a = torch.cuda.Event(enable_timing=True)
                    b = torch.cuda.Event(enable_timing=True)
                    a.record(stream)
                    for _ in range(3):
                        g.replay()
                    b.record(stream)
                    b.synchronize()
                us = a.elapsed_time(b) * 1e3 / (3 * launches)
                step_bytes = w_bytes + m * k * 2 + m * n * 4
                gbs = step_bytes / us / 1e3
                out_rows.append({"m": m, "k": k, "n": n,
                                 "weights": "q8_0" if fmt == _lib.WEIGHTS_Q8_TILES else "bf16",
                                 "us": round(us, 3), "gbs": round(gbs, 1),
                                 "frac": round(gbs / peak_gbs, 4), "err": err})
                del g
            del ws
    gemm.close()
    return out_rows


def measure_generator(rank: int, world=None, context: int = 512, patch_replays: int = 50,
                      steps: int = 32) -> dict:
    """BASELINE configs 2 and 3 on the released shapes with seeded Q8_0
    weights: the DiT patch (replays of its CUDA graph, inputs on the device)
    and the full per-patch step at `context` positions with a bf16 KV cache
    (host noise in, latent and stop logits out, one graph per step)."""
    import numpy as np
    import torch

    from voxcpm_b200 import _lib
    from voxcpm_b200.generator import Generator, released_config

    c = released_config()
    c.max_length = context + steps + 16
    c.vocab = 1024
    t0 = time.perf_counter()
    gen = Generator(c, seed=100 + rank, checkpoint=_lib.CHECKPOINT_Q8, cache_type=_lib.CACHE_BF16)
    create_s = time.perf_counter() - t0
    stream = torch.cuda.ExternalStream(gen.stream())
    rng = np.random.default_rng(rank)
    mu = rng.normal(0, 1, 2 * c.dit.hidden).astype(np.float32)
    cond = rng.normal(0, 1, (c.patch_size, c.feat_dim)).astype(np.float32)
    noise = rng.normal(0, 1, (c.patch_size, c.feat_dim)).astype(np.float32)
    a = torch.cuda.Event(enable_timing=True)
    b = torch.cuda.Event(enable_timing=True)

    def time_patch(replays):
        gen.DitPatch(mu, cond, noise, 10, 2.0)  # captures the patch graph
        for _ in range(3):
            gen.ReplayDitPatch()
        torch.cuda.synchronize()
        a.record(stream)
        for _ in range(replays):
            gen.ReplayDitPatch()
        b.record(stream)
        b.synchronize()
        return a.elapsed_time(b) * 1e3 / replays

    persistent = gen.persistent()
    patch_us = time_patch(patch_replays)
    # The per-kernel sequence of the same patch, for comparison.
    gen.SetPersistent(False)
    per_kernel_us = time_patch(max(patch_replays // 5, 5))
    gen.SetPersistent(persistent)

    # Full step at `context`: a prompt of `context` rows (one audio row last),
    # then patches; each step's device time is bracketed by events on the
    # generator's stream, its wall time includes the host copies.
    tokens = rng.integers(0, c.vocab, context).astype(np.int32)
    audio = np.zeros(context, np.int32)
    audio[-1] = 1
    feats = np.zeros((context, c.patch_size, c.feat_dim), np.float32)
    feats[-1] = rng.normal(0, 1, (c.patch_size, c.feat_dim))
    noises = [rng.normal(0, 1, (c.patch_size, c.feat_dim)).astype(np.float32) for _ in range(steps)]
    warm = 2  # the first steps capture the step graph

    def time_steps():
        t0 = time.perf_counter()
        gen.Prefill(tokens, 1 - audio, audio, feats)
        prefill = time.perf_counter() - t0
        device_ms, wall_ms = [], []
        for n in noises:
            a.record(stream)
            t0 = time.perf_counter()
            gen.Step(n, 10, 2.0)
            wall_ms.append((time.perf_counter() - t0) * 1e3)
            b.record(stream)
            b.synchronize()
            device_ms.append(a.elapsed_time(b))
        return float(np.median(device_ms[warm:])), float(np.median(wall_ms[warm:])), prefill

    step_ms, step_wall_ms, prefill_s = time_steps()
    vae = measure_vae(gen, c, tokens, audio, feats, noises, warm, rank)
    # The same steps from the same prompt on the per-kernel path.
    gen.SetPersistent(False)
    per_kernel_step_ms, _, _ = time_steps()
    gen.SetPersistent(persistent)

    # Config 4: this rank's requests (rank, rank + world, ... of 64), each a
    # seeded prompt of 16..128 text tokens plus the audio-start row, then
    # BOX_PATCHES patches; device time on the generator's stream from the
    # first prefill to the last latent.
    n_ranks = world if world else 1
    mine = box_share(rank, n_ranks)
    visible = os.environ.get("CUDA_VISIBLE_DEVICES")
    gpu_index = int(visible.split(",")[torch.cuda.current_device()]) if visible else torch.cuda.current_device()
    box_clocks = ClockSampler(gpu_index)
    box_clocks.__enter__()
    torch.cuda.synchronize()
    a.record(stream)
    for req in mine:
        rq = np.random.default_rng(10_000 + req)
        rows = int(rq.integers(16, 129)) + 1
        r_tokens = rq.integers(0, c.vocab, rows).astype(np.int32)
        r_audio = np.zeros(rows, np.int32)
        r_audio[-1] = 1
        r_feats = np.zeros((rows, c.patch_size, c.feat_dim), np.float32)
        r_feats[-1] = rq.normal(0, 1, (c.patch_size, c.feat_dim))
        gen.Prefill(r_tokens, 1 - r_audio, r_audio, r_feats)
        for _ in range(BOX_PATCHES):
            gen.Step(rq.normal(0, 1, (c.patch_size, c.feat_dim)).astype(np.float32), 10, 2.0)
    b.record(stream)
    b.synchronize()
    box_s = a.elapsed_time(b) / 1e3
    box_audio = len(mine) * BOX_PATCHES * PATCH_AUDIO_S
    weight_bytes = gen.weight_bytes()
    gen.close()
    box_clocks.__exit__(None, None, None)
    batched_clocks = ClockSampler(gpu_index)
    with batched_clocks:
        batched_s = max_over_ranks(world, measure_box_batched(c, mine))
    box_s_max = max_over_ranks(world, box_s)
    box_audio_all = sum_over_ranks(world, box_audio)
    box_patches_all = sum_over_ranks(world, len(mine) * BOX_PATCHES)
    peak_gbs = measured_peak()[0]
    box_gbs_per_gpu = STEP_BYTES_CONFIG3 * box_patches_all / n_ranks / box_s_max / 1e9
    floor_us = DIT_PATCH_BYTES / (measured_peak()[0] * 1e9) * 1e6
    return {
        "dit_patch": {"us": patch_us, "bytes": DIT_PATCH_BYTES, "hbm_floor_us": floor_us,
                      "frac_of_floor": floor_us / patch_us, "replays": patch_replays,
                      "path": "persistent cooperative kernel" if persistent else "per-kernel sequence",
                      "per_kernel_us": per_kernel_us,
                      "config": "12-layer DiT 1024 (16 q / 2 kv heads x 128), 22 rows, 10 Euler steps "
                                "(9 evaluations), CFG 2.0, Q8_0 weights, one CUDA graph"},
        "step": {"ms_per_patch": step_ms, "wall_ms_per_patch": step_wall_ms,
                 "per_kernel_ms_per_patch": per_kernel_step_ms,
                 "audio_s_per_s": PATCH_AUDIO_S / (step_wall_ms / 1e3), "rtf": step_wall_ms / 1e3 / PATCH_AUDIO_S,
                 "context": context, "steps": steps - warm, "kv_cache": "bf16",
                 "weight_bytes": weight_bytes, "prefill_s": prefill_s, "create_s": create_s,
                 "path": "persistent DiT patch and one-row LM stacks" if persistent
                         else "per-kernel sequence",
                 "config": "LM 28x2048 + residual LM 8x2048 + encoder 12x1024 + DiT 12x1024, Q8_0, "
                           "one CUDA graph per patch"},
        "vae": vae,
        "box_batched": {"audio_s_per_s": box_audio_all / batched_s, "n_gpus": n_ranks,
                        "slots_per_gpu": min(BOX_SLOTS, len(mine)), "device_s": batched_s,
                        "requests": sum_over_ranks(world, len(mine)),
                        "hbm_gbs_per_gpu": STEP_BYTES_CONFIG3 * box_patches_all / n_ranks / batched_s / 1e9,
                        "sample": f"each rank's share of the {BOX_REQUESTS} requests in min({BOX_SLOTS}, share) "
                                  "slots of one GeneratorBatch (shared weights; one DiT pass for all active "
                                  "slots per Euler evaluation); a slot takes the next request when its "
                                  "request ends",
                        "clocks": batched_clocks.summary(),
                        "config": "BASELINE config 4 (box throughput), batched request slots, no collectives"},
        "box": {"audio_s_per_s": box_audio_all / box_s_max, "n_gpus": n_ranks,
                "requests": sum_over_ranks(world, len(mine)), "patches_per_request": BOX_PATCHES,
                "device_s": box_s_max, "audio_s": box_audio_all,
                "hbm_gbs_per_gpu": box_gbs_per_gpu, "hbm_frac_per_gpu": box_gbs_per_gpu / peak_gbs,
                "sample": f"all {BOX_REQUESTS} requests split over the ranks "
                          f"(prompts of 16..128 text tokens, per-request seeds), {BOX_PATCHES} patches each, "
                          "prefill included; requests run one after another on each GPU",
                "clocks": box_clocks.summary(),
                "config": "BASELINE config 4 (box throughput), one request stream per GPU, no collectives"},
    }


def box_share(rank: int, world: int) -> list:
    """The config-4 requests rank `rank` of `world` runs: requests rank,
    rank + world, ... of BOX_REQUESTS (every request on exactly one rank; no
    collective)."""
    return list(range(rank, BOX_REQUESTS, max(world, 1)))


def drive_box(batch, c, requests, slots: int, patches: int) -> int:
    """Runs `requests` through the slots of `batch` (GeneratorBatch-like:
    Prefill(slot, ...), Step(noise, active, timesteps, cfg)): requests fill
    free slots in order; every step advances all active slots by one patch;
    a slot that has produced `patches` patches takes the next request.
    Returns the number of steps."""
    import numpy as np

    values = (c.patch_size, c.feat_dim)
    queue = list(requests)
    left = [0] * slots
    rngs = [None] * slots
    steps = 0
    while True:
        for s in range(slots):
            if left[s] == 0 and queue:
                prompt, rngs[s] = box_request(c, queue.pop(0))
                batch.Prefill(s, *prompt)
                left[s] = patches
        active = np.array([1 if n > 0 else 0 for n in left], np.int32)
        if not active.any():
            return steps
        noise = np.zeros((slots,) + values, np.float32)
        for s in range(slots):
            if active[s]:
                noise[s] = rngs[s].normal(0, 1, values)
        batch.Step(noise, active, 10, 2.0)
        steps += 1
        left = [n - 1 if n > 0 else 0 for n in left]


def box_request(c, req: int):
    """Request `req` of config 4: a seeded prompt of 16..128 text tokens plus
    the audio-start row, and its generator for the patches' noise."""
    import numpy as np

    rq = np.random.default_rng(10_000 + req)
    rows = int(rq.integers(16, 129)) + 1
    tokens = rq.integers(0, c.vocab, rows).astype(np.int32)
    audio = np.zeros(rows, np.int32)
    audio[-1] = 1
    feats = np.zeros((rows, c.patch_size, c.feat_dim), np.float32)
    feats[-1] = rq.normal(0, 1, (c.patch_size, c.feat_dim))
    return (tokens, 1 - audio, audio, feats), rq


def measure_box_batched(c, requests) -> float:
    """Config 4 through a GeneratorBatch of BOX_SLOTS slots: the requests fill
    the slots; every step advances all active slots by one patch; a slot that
    has produced BOX_PATCHES patches takes the next request (prefill) while
    the others continue. Device seconds on the batch's stream from the first
    prefill to the last patch (a short warm-up first captures the graph).
    With every request BOX_PATCHES long, slots finish together and refill
    together."""
    import numpy as np
    import torch

    from voxcpm_b200 import _lib
    from voxcpm_b200.generator import GeneratorBatch

    slots = min(BOX_SLOTS, len(requests))
    batch = GeneratorBatch(c, slots, seed=100, checkpoint=_lib.CHECKPOINT_Q8, cache_type=_lib.CACHE_BF16)
    stream = torch.cuda.ExternalStream(batch.stream())
    drive_box(batch, c, requests[:slots], slots, 3)  # captures the graph of all slots active
    a = torch.cuda.Event(enable_timing=True)
    b = torch.cuda.Event(enable_timing=True)
    torch.cuda.synchronize()
    a.record(stream)
    drive_box(batch, c, requests, slots, BOX_PATCHES)
    b.record(stream)
    b.synchronize()
    batch.close()
    return a.elapsed_time(b) / 1e3


def profile_case(case: str, max_ctas: int = 0, cooperative: bool = True, slots: int = 8) -> None:
    """A few launches of one kernel on a small case, for ncu captures:
    `product`: 8 config-0 products with the stream plan (independent), then 8
    with the planner's plan (dependent); `dit`: two eager DiT patches (the
    persistent kernel) on the released DiT with one-layer LMs; `step`: two
    eager steps at context 512 (bf16 cache) with a 4-layer LM and a 2-layer
    residual LM (the persistent stack kernel at the released widths); `wide`: three
    products of 88 rows of 1024 -> 8192 (the gate/up product of four batched
    slots' DiT rows) on the planner's row-split plan, then three on the wide
    tcgen05 kernel;
    `batch`: two steps of a GeneratorBatch of 8 slots on the released shapes
    (the first captures the step's graph); `matmul`: three Bf16Gemm::Matmul
    calls of 4096 x 4096 x 4096 in the reduction-contiguous layout, timed
    with CUDA events (96 MB of operands and C); `vae`: six AudioVAE decodings
    of one patch (4 latent frames) on the released decoder, timed with CUDA
    events on its stream (183 MB of float32 weights)."""
    import numpy as np
    import torch

    from voxcpm_b200 import _lib
    from voxcpm_b200 import kernels as K

    lib = _lib.load()
    torch.cuda.set_device(0)
    lib.vx_set_persistent_max_ctas(max_ctas)
    lib.vx_set_persistent_cooperative(int(cooperative))
    if case == "step":
        from voxcpm_b200.generator import Generator, released_config

        c = released_config()
        c.lm.layers, c.residual_lm.layers = 4, 2
        c.max_length = 600
        c.vocab = 1024
        gen = Generator(c, seed=7, cache_type=_lib.CACHE_BF16)
        gen.SetGraphs(False)
        rng = np.random.default_rng(0)
        rows = 512
        audio = np.zeros(rows, np.int32)
        audio[-1] = 1
        feats = np.zeros((rows, c.patch_size, c.feat_dim), np.float32)
        feats[-1] = rng.normal(0, 1, (c.patch_size, c.feat_dim))
        gen.Prefill(rng.integers(0, c.vocab, rows).astype(np.int32), 1 - audio, audio, feats)
        for _ in range(2):
            gen.Step(rng.normal(0, 1, (c.patch_size, c.feat_dim)).astype(np.float32), 10, 2.0)
        gen.close()
        if K.DeviceError():
            raise RuntimeError("a bounded device wait expired")
        print(f"case {case}: ok", flush=True)
        return
    if case == "vae":
        from voxcpm_b200.vae import AudioVae, default_vae_config

        vae = AudioVae(default_vae_config(), seed=200)
        stream = torch.cuda.ExternalStream(vae.stream())
        x = torch.randn(4, 64, device="cuda")
        torch.cuda.synchronize()
        start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        for _ in range(6):
            start.record(stream)
            vae.Enqueue(x.data_ptr(), 4)
            end.record(stream)
            samples = vae.Collect()
            print(f"vae decode of 4 frames: {start.elapsed_time(end) * 1e3:.1f} us, {samples.size} samples")
        vae.close()
        return
    if case == "matmul":
        from voxcpm_b200.gemm import Bf16Gemm, MatmulShape

        n = 4096
        gen = torch.Generator(device="cuda").manual_seed(0)
        a = torch.randn(n * n, device="cuda", generator=gen).to(torch.bfloat16).view(torch.int16)
        b = torch.randn(n * n, device="cuda", generator=gen).to(torch.bfloat16).view(torch.int16)
        c = torch.empty(n * n, device="cuda")
        gemm = Bf16Gemm()
        shape = MatmulShape(1, 0, n, n, n, n, n, n, 0, 0, 0, 1, 0)
        start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        for _ in range(3):
            start.record()
            gemm.Matmul(shape, None, a, b, c)
            end.record()
            end.synchronize()
            print(f"matmul {n}^3: {start.elapsed_time(end) * 1e3:.1f} us, "
                  f"{2 * n ** 3 / (start.elapsed_time(end) * 1e-3) / 1e12:.1f} TFLOP/s")
        gemm.close()
        return
    if case == "product":
        tiles, ys = [], []
        for c in range(COPIES):
            blocks = torch.from_numpy(K.RandomQ8_0(1000, c, OUT, IN)).cuda()
            t = torch.empty(K.Q8TilesBytes(OUT, IN), dtype=torch.uint8, device="cuda")
            K.Q8_0ToTiles(blocks, OUT, IN, t)
            tiles.append(t)
            ys.append(torch.empty(ROWS, OUT, dtype=torch.bfloat16, device="cuda"))
        x = torch.randn(ROWS, IN, device="cuda").to(torch.bfloat16)
        plan = _lib.WmmaPlan(STREAM_SPLITS, -(-(IN // 32) // STREAM_SPLITS), 0, 0, STREAM_VARIANT)
        for i in range(8):
            _lib.check(lib.vx_product_ex(_lib.WEIGHTS_Q8_TILES, x.data_ptr(), tiles[i].data_ptr(),
                                         ys[i].data_ptr(), _lib.OUT_BF16, ROWS, IN, OUT,
                                         _lib.PRODUCT_INDEPENDENT, ctypes.byref(plan), None))
        for i in range(8):
            _lib.check(lib.vx_product(_lib.WEIGHTS_Q8_TILES, x.data_ptr(), tiles[8 + i].data_ptr(),
                                      ys[8 + i].data_ptr(), _lib.OUT_BF16, ROWS, IN, OUT, 0, None, None))
        torch.cuda.synchronize()
    elif case == "wide":
        rows, columns, out = 88, 1024, 8192
        blocks = torch.from_numpy(K.RandomQ8_0(1000, 0, out, columns)).cuda()
        t = torch.empty(K.Q8TilesBytes(out, columns), dtype=torch.uint8, device="cuda")
        K.Q8_0ToTiles(blocks, out, columns, t)
        x = torch.randn(rows, columns, device="cuda").to(torch.bfloat16)
        y = torch.empty(rows, out, dtype=torch.float32, device="cuda")
        # The planner's plan (row-split variant 30), then the wide tcgen05
        # kernel on the plan its planner makes for this shape (2 splits of
        # 16 blocks).
        wide = _lib.WmmaPlan(2, 16, 0, 0, K.TENSOR_CORE_WIDE_VARIANT)
        for plan in (None, ctypes.byref(wide)):
            for _ in range(3):
                _lib.check(lib.vx_product(_lib.WEIGHTS_Q8_TILES, x.data_ptr(), t.data_ptr(), y.data_ptr(),
                                          _lib.OUT_F32, rows, columns, out, 0, plan, None))
        torch.cuda.synchronize()
    elif case == "batch":
        from voxcpm_b200.generator import GeneratorBatch, released_config

        c = released_config()
        c.max_length = 256
        rows = 16
        rng = np.random.default_rng(0)
        feats = rng.normal(0, 1, (rows, c.patch_size, c.feat_dim)).astype(np.float32)
        audio = np.ones(rows, np.int32)
        batch = GeneratorBatch(c, slots, seed=1)
        for s in range(slots):
            batch.Prefill(s, np.zeros(rows, np.int32), 1 - audio, audio, feats)
        noise = rng.normal(0, 1, (slots, c.patch_size, c.feat_dim)).astype(np.float32)
        for _ in range(2):
            batch.Step(noise, None, 10, 2.0)
        torch.cuda.synchronize()
        batch.close()
    else:
        from voxcpm_b200.generator import Generator, released_config

        c = released_config()
        c.lm.layers = 1
        c.residual_lm.layers = 1
        c.max_length = 64
        gen = Generator(c, seed=7)
        gen.SetGraphs(False)
        rng = np.random.default_rng(0)
        mu = rng.normal(0, 1, 2 * c.dit.hidden).astype(np.float32)
        cond = rng.normal(0, 1, (c.patch_size, c.feat_dim)).astype(np.float32)
        noise = rng.normal(0, 1, (c.patch_size, c.feat_dim)).astype(np.float32)
        for _ in range(2):
            gen.DitPatch(mu, cond, noise, 10, 2.0)
        gen.close()
    if K.DeviceError():
        raise RuntimeError("a bounded device wait expired")
    print(f"case {case}: ok", flush=True)


def main():
    args = parse()
    if args.case is not None:
        profile_case(args.case, args.max_ctas, not args.non_cooperative, args.slots)
        return
    world, rank, local = init_dist(args.gpus)
    try:
        if args.impl == "reference":
            run_reference(args, world, rank)
        else:
            run_ours(args, world, rank, local)
    finally:
        if world > 1:
            import torch.distributed as dist

            dist.destroy_process_group()


if __name__ == "__main__":
    main()
