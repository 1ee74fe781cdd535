#!/usr/bin/env python
"""Benchmark of the k200 matmul hot path on B200.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
    torchrun --nproc-per-node N bench.py --gpus N ...   (N > 1)

Workload (the metric's configuration): the Q4_0 GEMVs of a
7B MLP at batch 1, chained as up then down:
    y1[1,11008] = x[1,4096]   . W_up^T   (K=4096,  N=11008)
    y2[1,4096]  = y1[1,11008] . W_down^T (K=11008, N=4096)
One step = both GEMVs over one activation vector.  Weights are Q4_0 blocks of
N(0, 0.02) values (GGML quantiser on the device), X is U[-1, 1] (synthetic,
seeded).  With N GPUs each weight is row-sharded N ways and each output is
all-gathered over NCCL, so the down projection sees the full y1.

Metric: Q4_0 weight GB/s (weight bytes of both matrices per step / step time,
whole job), the HBM-bound figure of merit the reference reports for its Q4
GEMV.  Between timed steps the weights rotate through enough distinct sets
that the whole rotation exceeds twice the L2 size, so every step streams its
weights from HBM.

--workload q4-gemm | f16-gemm | f32-gemm | i8-gemm [--batch B] measures BASELINE
configs 2-4 instead (the batched matmul in TFLOP/s of the logical 2*N*K*batch
work, with the HBM and tensor rooflines); the default, gemv, is config 1.

--impl reference times the reference's CPU implementation of the same path
(bench/native-q4-reference.h reference(), compiled from the reference sources
into oracle/_ref; the C restatement in oracle/ when that is absent) on the
host cores, one bounded sample of the workload per step.
"""
from __future__ import annotations

import argparse
import json
import math
import os
import statistics
import subprocess
import sys
import tempfile
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

UP = (4096, 11008)    # (K, N)
DOWN = (11008, 4096)
FALLBACK_HBM_GBS = 6650.0
FALLBACK_BF16_TFLOPS = 1590.0


def q4_bytes(k: int, n: int) -> int:
    return n * (k // 32) * 18


def read_peaks() -> dict:
    path = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(path):
        with open(path) as f:
            p = json.load(f)
        return {"hbm_gbs": float(p["hbm_gbs"]), "bf16_tflops": float(p.get("bf16_tflops", FALLBACK_BF16_TFLOPS)),
                "source": "measured"}
    return {"hbm_gbs": FALLBACK_HBM_GBS, "bf16_tflops": FALLBACK_BF16_TFLOPS, "source": "fallback"}


def profile_traffic(name: str):
    """Per-launch DRAM bytes of the dominant kernel from the committed ncu summary."""
    path = os.path.join(ROOT, "profiles", name)
    if not os.path.exists(path):
        return None
    for line in open(path):
        if line.startswith("traffic_bytes_per_launch:"):
            try:
                return int(float(line.split(":", 1)[1].strip()))
            except ValueError:
                return None
    return None


class ClockSampler:
    """nvidia-smi clocks/throttle reasons sampled every 200 ms during a window."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, device: int):
        self.device = device
        self.proc = None
        self.file = None
        self.t0 = self.t1 = None

    def start(self):
        self.file = tempfile.NamedTemporaryFile("w+", suffix=".csv", delete=False)
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits", "-lms", "200",
                 "-i", str(self.device)], stdout=self.file, stderr=subprocess.DEVNULL)
        except OSError:
            self.proc = None
        time.sleep(0.3)

    def mark(self, begin: bool):
        if begin:
            self.t0 = time.time()
        else:
            self.t1 = time.time()

    def stop(self) -> dict:
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        time.sleep(0.25)
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
        self.file.flush()
        rows = []
        with open(self.file.name) as f:
            for line in f:
                parts = [p.strip() for p in line.split(",")]
                if len(parts) < 9:
                    continue
                try:
                    rows.append((float(parts[1]), float(parts[2]), parts[5:9]))
                except ValueError:
                    continue
        os.unlink(self.file.name)
        if not rows:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["no samples"], "samples": 0}
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({names[i] for _, _, r in rows for i, v in enumerate(r) if v.lower() == "active"})
        return {"sm_mhz": statistics.median(r[0] for r in rows), "sm_max_mhz": max(r[1] for r in rows),
                "reasons": reasons, "samples": len(rows)}


# ---------------------------------------------------------------------------
# CPU arm (reference implementation on the host cores)
# ---------------------------------------------------------------------------
def cpu_weights(seed: int, k: int, n: int):
    import oracle as O

    w = O.normal(seed, n * k, 0.0, 0.02)
    q4 = O.q4_0_quantize(w, n, k)
    return q4, O.q4_0_dequantize(q4, n, k)


def cpu_step_fn(threads: int):
    """One (possibly row-sampled) up+down step of the reference CPU GEMV."""
    import oracle as O

    R = O.ref()
    kind = "reference" if R is not None else "port"
    dec_up = cpu_weights(11, *UP)[1]
    dec_down = cpu_weights(12, *DOWN)[1]
    x = O.uniform(0x09200ABC, UP[0], -1.0, 1.0)
    handles = {}

    def prepared(idx, dec, k, rows):
        key = (idx, rows)
        if key not in handles:
            handles[key] = R.ref_gemv_create(np.ascontiguousarray(dec[: rows * k]), k, rows, threads)
        return handles[key]

    def step(frac: float) -> int:
        """Runs both GEMVs over the first `frac` of their rows; returns Q4 bytes covered."""
        covered = 0
        inp = x
        for idx, ((k, n), dec) in enumerate(((UP, dec_up), (DOWN, dec_down))):
            rows = max(1, int(round(n * frac)))
            y = np.empty(rows, np.float64)
            xin = np.ascontiguousarray(inp[:k], np.float32)
            if R is not None:
                R.ref_gemv_run(prepared(idx, dec, k, rows), xin, 1, y)
            else:
                O.lib().ko_reference_fp64(dec[: rows * k], xin, k, rows, 1, y, threads)
            covered += q4_bytes(k, rows)
            nxt = np.zeros(n, np.float32)
            nxt[:rows] = y
            inp = nxt
        return covered

    return step, kind


def cpu_baseline(seconds: float = 10.0) -> dict:
    threads = os.cpu_count() or 1
    step, kind = cpu_step_fn(threads)
    step(0.05)  # warm caches and threads
    t0 = time.perf_counter()
    done = nbytes = 0
    while True:
        nbytes += step(1.0)
        done += 1
        if time.perf_counter() - t0 >= seconds and done >= 2:
            break
    dt = time.perf_counter() - t0
    return {"value": nbytes / dt / 1e9, "unit": "GB/s", "cores": threads, "kind": kind,
            "sample": f"{done} full up+down Q4_0 GEMV steps (K4096xN11008, K11008xN4096, batch 1), "
                      f"FP64 reference() over pre-decoded weights, {dt:.1f} s"}


def extra_cpu_baselines(seconds: float = 3.0) -> dict:
    """The other two CPU paths of the reference on this path, timed on the host:
    (a) library-bench's single-thread FP64 gold loop over the decoded Q4_0
    weights (bench/library-bench.cpp:121-123), on the up projection; (c) the
    per-call host quantiser of the rowwise-int8 path (src/k200.cpp:209-229,
    two-pass per-tensor A8), on config 4's batch-32 activations."""
    import oracle as O

    k, n = UP
    rows = 256
    dec = O.q4_0_dequantize(O.q4_0_quantize(O.normal(11, rows * k, 0.0, 0.02), rows, k), rows, k)
    x = O.uniform(0x09200ABC, k, -1.0, 1.0)
    t0, done = time.perf_counter(), 0
    while time.perf_counter() - t0 < seconds or done < 2:
        O.reference_fp64(dec, x, k, rows, 1, threads=1)
        done += 1
    dt = time.perf_counter() - t0
    gold = {"value": q4_bytes(k, rows) * done / dt / 1e9, "unit": "GB/s", "cores": 1, "kind": "port",
            "sample": f"{done} calls of the serial FP64 gold loop over {rows} rows of K{k} ({dt:.1f} s)"}
    xi = O.normal(0x09200ABC, 32 * 8192, 0.0, 1.0)
    t0, done = time.perf_counter(), 0
    while time.perf_counter() - t0 < seconds or done < 2:
        O.a8_tensor(xi)
        done += 1
    dt = time.perf_counter() - t0
    quant = {"value": dt / done * 1e3, "unit": "ms per call", "cores": 1, "kind": "port",
             "sample": f"{done} two-pass per-tensor A8 quantisations of 32x8192 f32 activations ({dt:.1f} s)"}
    return {"library_bench_gold_loop": gold, "i8_host_activation_quantiser": quant}


def run_reference(args) -> None:
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    threads = os.cpu_count() or 1
    step, kind = cpu_step_fn(threads)
    # size one step so that warmup + steps finish in about two minutes
    t = time.perf_counter()
    full = step(1.0)
    t_full = time.perf_counter() - t
    budget = 120.0 / max(1, args.steps + args.warmup)
    frac = min(1.0, budget / max(t_full, 1e-6))
    for _ in range(args.warmup):
        step(frac)
    t0 = time.perf_counter()
    nbytes = 0
    for _ in range(args.steps):
        nbytes += step(frac)
    dt = time.perf_counter() - t0
    value = nbytes / dt / 1e9
    sample = (f"each step: the first {frac:.4f} of the rows of both GEMVs "
              f"({full * frac / 1e6:.2f} MB of Q4_0 weights), FP64 reference() over pre-decoded weights")
    line = {
        "impl": "reference", "metric": "q4_0_gemv_weight_gbps", "value": value, "unit": "GB/s",
        "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": dt / max(1, args.steps) * 1e3, "higher_is_better": True, "scaling": "strong",
        "vs_baseline": None, "dtype": "f64", "data": "synthetic",
        "config": {"workload": "q4_0 GEMV 7B MLP up+down, batch 1 (config 1)", "up": "K4096xN11008",
                   "down": "K11008xN4096"},
        "cpu_baseline": {"value": value, "unit": "GB/s", "cores": threads, "kind": kind, "sample": sample},
        "e2e": {"value": value, "unit": "GB/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


# ---------------------------------------------------------------------------
# GPU arm
# ---------------------------------------------------------------------------
def run_ours(args) -> None:
    import torch
    import torch.distributed as dist

    import kunlunk200_lib_b200 as K

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world != args.gpus:
        raise SystemExit(f"--gpus {args.gpus} but WORLD_SIZE={world}: launch N>1 with torchrun")
    torch.cuda.set_device(local)
    if world > 1:
        import datetime

        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120), device_id=torch.device("cuda", local))
    dev = local
    K.select(dev)
    stream = torch.cuda.Stream()
    K.set_stream(dev, stream.cuda_stream)
    # resident inference weights: no kernel writes them, so each GEMV may start
    # streaming its first weight boxes while the previous kernel finishes
    K.set_static_weights(dev, True)
    l2 = torch.cuda.get_device_properties(dev).L2_cache_size

    from kunlunk200_lib_b200.shard import row_shard

    for k, n in (UP, DOWN):
        if n % world:  # equal slices: the all-gather writes Y without padding
            raise SystemExit(f"N={n} does not split evenly over {world} GPUs")
    n_up, n_down = row_shard(UP[1], world, rank)[1], row_shard(DOWN[1], world, rank)[1]
    shard_bytes = q4_bytes(UP[0], n_up) + q4_bytes(DOWN[0], n_down)
    total_bytes = q4_bytes(*UP) + q4_bytes(*DOWN)
    sets = max(2, math.ceil(2 * l2 / shard_bytes) + 1)

    gen = torch.Generator(device="cuda")
    weights = []
    with torch.cuda.stream(stream):
        for s in range(sets):
            pair = []
            for m, (k, n) in enumerate(((UP[0], n_up), (DOWN[0], n_down))):
                gen.manual_seed(1000003 * s + 7919 * m + 104729 * rank + 1)
                w = torch.randn((n, k), generator=gen, device="cuda", dtype=torch.float32) * 0.02
                q = torch.empty(q4_bytes(k, n), dtype=torch.uint8, device="cuda")
                K.quantize_q4_0(dev, q, w, k, n)
                pair.append(q)
                del w
            weights.append(pair)
        gen.manual_seed(0x09200ABC)
        x = torch.rand(UP[0], generator=gen, device="cuda") * 2 - 1
        y1_full = torch.empty(UP[1], device="cuda")
        y2_full = torch.empty(DOWN[1], device="cuda")
    stream.synchronize()
    kern = K.Kernel()

    # N > 1: each GEMV stores its rows into every rank's output over NVLink
    # (k200_matmul_q4_gather); the down GEMV waits on the device for every
    # rank's up rows.  Outputs alternate between two buffers by step parity.
    if world > 1:
        from kunlunk200_lib_b200.shard import PeerExchange

        def all_gather_obj(obj):
            got = [None] * world
            dist.all_gather_object(got, obj)
            return got

        ex_up = PeerExchange.over_group(K, dev, UP[1], world, rank, all_gather_obj)
        ex_down = PeerExchange.over_group(K, dev, DOWN[1], world, rank, all_gather_obj)
        up_begin, down_begin = row_shard(UP[1], world, rank)[0], row_shard(DOWN[1], world, rank)[0]
        scratch_bytes = max(K.matmul_q4_gather_scratch(dev, UP[0], n_up),
                            K.matmul_q4_gather_scratch(dev, DOWN[0], n_down))
        if not scratch_bytes:
            raise SystemExit("shard shape not handled by the batch-1 tensor-core GEMV")
        with torch.cuda.stream(stream):  # zeroed before the first GEMV on the library stream reads it
            scratch = torch.zeros(scratch_bytes, dtype=torch.uint8, device="cuda")
        stream.synchronize()
        dist.barrier()  # every rank's regions are mapped and zeroed before any rank stores into them
        torch.cuda.synchronize()

    def gemv_up(s: int):
        wu = weights[s % sets][0]
        if world == 1:
            K.matmul(kern, dev, y1_full, wu, x, UP[0], n_up, 1, K.Q4_0)
            return
        K.check(K.matmul_q4_gather(dev, ex_up.view(s), up_begin, wu, x, UP[0], n_up, scratch, scratch_bytes))

    def gemv_down(s: int):
        wd = weights[s % sets][1]
        if world == 1:
            K.matmul(kern, dev, y2_full, wd, y1_full, DOWN[0], n_down, 1, K.Q4_0)
            return
        K.check(K.matmul_q4_gather(dev, ex_down.view(s), down_begin, wd, ex_up.output(s), DOWN[0], n_down, scratch,
                                   scratch_bytes, wait_for=ex_up.view(s)))

    def step(s: int):
        gemv_up(s)
        gemv_down(s)

    def output(s: int) -> int:
        """Address of step s's full Y on this rank (complete after finish(s))."""
        return y2_full.data_ptr() if world == 1 else ex_down.output(s)

    def finish(s: int):
        """N > 1: wait on the device until every rank's rows of step s's Y are here."""
        if world > 1:
            K.check(K.gather_wait(dev, ex_down.view(s)))

    nwarm = max(3, args.warmup)
    with torch.cuda.stream(stream):
        for i in range(nwarm):
            step(i)
        finish(nwarm - 1)
    stream.synchronize()
    K.check(K.wait())
    if world > 1:
        dist.barrier()  # the next sequence starts again at buffer 0
        torch.cuda.synchronize()

    # one CUDA graph holds a whole number of rotations; the timed region
    # replays it until exactly `steps` steps ran (a remainder graph if needed)
    per_graph = sets * max(1, 48 // sets)
    per_graph *= 1 + per_graph % 2  # even: the output buffers alternate across replays
    reps, rem = divmod(args.steps, per_graph)

    def capture(nsteps: int):
        if nsteps == 0:
            return None
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g, stream=stream):
            for i in range(nsteps):
                step(i)
            finish(nsteps - 1)
        return g

    g_main = capture(per_graph) if reps else None
    g_rem = capture(rem)
    with torch.cuda.stream(stream):
        if g_main is not None:
            g_main.replay()
        if g_rem is not None:
            g_rem.replay()
    stream.synchronize()
    K.check(K.wait())

    visible = os.environ.get("CUDA_VISIBLE_DEVICES")
    phys = int(visible.split(",")[dev]) if visible and visible.split(",")[dev].strip().isdigit() else dev
    clocks = ClockSampler(phys)
    if rank == 0:
        clocks.start()
    start = torch.cuda.Event(enable_timing=True)
    end = torch.cuda.Event(enable_timing=True)
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    if rank == 0:
        clocks.mark(True)
    with torch.cuda.stream(stream):
        start.record(stream)
        for _ in range(reps):
            g_main.replay()
        if g_rem is not None:
            g_rem.replay()
        end.record(stream)
    stream.synchronize()
    torch.cuda.synchronize()
    if rank == 0:
        clocks.mark(False)
    if world > 1:
        dist.barrier()
    ms = start.elapsed_time(end)
    t = torch.tensor([ms], device="cuda")
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    ms = float(t.item())
    clock_info = clocks.stop() if rank == 0 else None
    if world > 1:  # rank 0's host was busy with the clock record: start the next phase together
        dist.barrier()
        torch.cuda.synchronize()
    value = total_bytes * args.steps / (ms * 1e-3) / 1e9
    launches = args.steps * 2 + (reps + (1 if rem else 0)) * (world > 1)

    # ---- per-launch durations of the dominant kernel (events around each launch,
    #      queued behind a sleep so the GPU runs them back to back)
    nprobe = 24 * sets
    evs = [torch.cuda.Event(enable_timing=True) for _ in range(2 * nprobe + 1)]
    with torch.cuda.stream(stream):
        torch.cuda._sleep(20_000_000)
        evs[0].record(stream)
        for i in range(nprobe):
            gemv_up(i)
            evs[2 * i + 1].record(stream)
            gemv_down(i)
            evs[2 * i + 2].record(stream)
        finish(nprobe - 1)
    stream.synchronize()
    K.check(K.wait())
    d_up = [evs[2 * i].elapsed_time(evs[2 * i + 1]) for i in range(nprobe)]
    d_down = [evs[2 * i + 1].elapsed_time(evs[2 * i + 2]) for i in range(nprobe)]
    alg_up = q4_bytes(UP[0], n_up) + 4 * UP[0] + 4 * n_up
    alg_down = q4_bytes(DOWN[0], n_down) + 4 * DOWN[0] + 4 * n_down
    mean_up, mean_down = statistics.mean(d_up), statistics.mean(d_down)

    def spread(d):
        return {"median": statistics.median(d) * 1e3, "min": min(d) * 1e3, "max": max(d) * 1e3, "launches": len(d)}
    # the timed region runs nothing but the two GEMV launches per step (and,
    # on N > 1, one wait launch per graph), so its average GEMV duration is
    # the region's device time over its GEMV launches
    launch_ms = ms / (args.steps * 2)
    achieved = (alg_up + alg_down) / 2 / (launch_ms * 1e-3) / 1e9
    peaks = read_peaks()

    # ---- end to end through the C ABI: pinned host X in, pinned host Y out
    e2e_steps = min(args.steps, 2000)
    xh = torch.empty(UP[0], dtype=torch.float32).pin_memory()
    xh.copy_(x.cpu())
    yh = torch.empty(DOWN[1], dtype=torch.float32).pin_memory()

    def host_step(i: int, kernel_copies: bool = True):
        """One decode step as a user issues it: input in, both GEMVs, output out.
        The copies are kernels (k200_copy_kernel, pinned host memory read and
        written over the bus), so the GEMVs keep their programmatic-launch
        overlap; kernel_copies=False uses copy-engine transfers instead."""
        if kernel_copies:
            K.check(K.copy_kernel(x, xh, xh.numel() * 4))
        else:
            K.check(K.copy_async(x, xh, xh.numel() * 4, K.HOST_TO_DEVICE))
        step(i)
        finish(i)
        if kernel_copies:
            K.check(K.copy_kernel(yh, output(i), yh.numel() * 4))
        else:
            K.check(K.copy_async(yh, output(i), yh.numel() * 4, K.DEVICE_TO_HOST))

    def timed_e2e(run_step) -> tuple[float, float]:
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        wall = time.perf_counter()
        with torch.cuda.stream(stream):
            e0.record(stream)
            for i in range(e2e_steps):
                run_step(i)
                K.check(K.wait())
            e1.record(stream)
        stream.synchronize()
        wall = time.perf_counter() - wall
        te = torch.tensor([e0.elapsed_time(e1)], device="cuda")
        if world > 1:
            dist.all_reduce(te, op=dist.ReduceOp.MAX)
        return total_bytes * e2e_steps / (float(te.item()) * 1e-3) / 1e9, wall

    # (1) each step recorded once with k200_graph_* and replayed: one launch
    #     per step (a graph per weight set; per output-buffer parity on N > 1)
    ngraphs = sets if world == 1 else sets * 2 // math.gcd(sets, 2)
    graphs = []
    with torch.cuda.stream(stream):
        for i in range(ngraphs):
            host_step(i)  # a direct run first: nothing grows during the recording
            K.check(K.wait())
            g = K.Graph(dev)
            with g:
                host_step(i)
            graphs.append(g)
    e2e_value, t_wall = timed_e2e(lambda i: graphs[i % ngraphs].launch())
    # (2) the calls issued one by one, with copy-engine transfers
    e2e_eager, t_wall_eager = timed_e2e(lambda i: host_step(i, kernel_copies=False))
    for g in graphs:
        g.close()

    cpu = cpu_baseline() if (rank == 0 and world == 1 and not args.no_cpu_baseline) else None
    if cpu is not None:
        cpu["also"] = extra_cpu_baselines()

    # the batched half of the metric (configs 2-4), same process, same GPUs
    batched = None
    if not args.no_batched:
        batched = []
        for wname, bk, bn, bb, blabel in BATCHED_SET:
            r = measure_gemm(K, torch, dist, dev, stream, world, rank, wname, bk, bn, bb, 0, 3, blabel,
                             target_s=0.4)
            if r is not None:
                batched.append({key: r[key] for key in ("metric", "value", "unit", "ms_per_step", "steps", "dtype",
                                                        "config", "roofline", "e2e", "gpu_launches", "clocks")})

    # the committed capture is of full-size launches; a shard's launch streams
    # its rows' share of the weights (traffic tracks the algorithmic bytes)
    shard_traffic = profile_traffic("q4_mma_gemv_k4096_n11008.md")
    if shard_traffic is not None and world > 1:
        full_alg = q4_bytes(*UP) + 4 * UP[0] + 4 * UP[1]
        shard_traffic = int(shard_traffic * ((alg_up + alg_down) / 2) / full_alg)
    if rank == 0:
        line = {
            "metric": "q4_0_gemv_weight_gbps", "value": value, "unit": "GB/s", "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms / args.steps,
            "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "f32",
            "data": "synthetic",
            "config": {"workload": "q4_0 GEMV 7B MLP up+down, batch 1 (config 1)",
                       "up": "K4096xN11008", "down": "K11008xN4096", "batch": 1,
                       "parallelism": f"row-shard{world}+fused-p2p-allgather" if world > 1 else "single",
                       "weights": "resident, declared static (k200_set_static_weights)",
                       "weight_bytes_per_step": total_bytes,
                       "l2": f"{sets} rotating weight sets ({sets * shard_bytes / 1e6:.0f} MB per GPU > 2x L2 "
                             f"{l2 / 1e6:.0f} MB)",
                       "timing": "CUDA graph replays, CUDA events on the launching stream, max over ranks"},
            "roofline": {"bound": "hbm", "achieved": achieved, "peak": peaks["hbm_gbs"], "unit": "GB/s",
                         "frac": achieved / peaks["hbm_gbs"],
                         "peak_source": peaks["source"],
                         "traffic": shard_traffic,
                         "kernel": "q4_mma_gemv_kernel",
                         "launch_us": launch_ms * 1e3,
                         "isolated_launch_us": {"up": mean_up * 1e3, "down": mean_down * 1e3,
                                                "up_spread": spread(d_up), "down_spread": spread(d_down)},
                         "algorithmic_bytes_per_launch": {"up": alg_up, "down": alg_down}},
            "cpu_baseline": cpu,
            "e2e": {"value": e2e_value, "unit": "GB/s", "h2d_bytes_per_step": xh.numel() * 4,
                    "d2h_bytes_per_step": yh.numel() * 4, "steps": e2e_steps,
                    "path": ("k200_graph_launch of the recorded step (k200_copy_kernel H2D from pinned host, "
                             "2x k200_matmul, k200_copy_kernel D2H to pinned host) + k200_wait per step"
                             if world == 1 else
                             "k200_graph_launch of the recorded step (k200_copy_kernel H2D, 2x "
                             "k200_matmul_q4_gather, k200_gather_wait, k200_copy_kernel D2H) + k200_wait per step"),
                    "wall_s": t_wall,
                    "eager": {"value": e2e_eager, "wall_s": t_wall_eager,
                              "path": "k200_copy_async H2D + the GEMVs + k200_copy_async D2H issued one by one "
                                      "through the C ABI, k200_wait per step"}},
            "gpu_launches": launches,
            "clocks": clock_info,
        }
        if world > 1:
            line["config"]["nvlink_bytes_per_step"] = 4 * (UP[1] + DOWN[1]) * (world - 1)
        if batched is not None:
            line["batched"] = batched
        print(json.dumps(line), flush=True)
    K.set_stream(dev, None)
    del g_main, g_rem
    if world > 1:
        dist.barrier()  # no rank still uses another rank's exchange regions
        ex_up.close()
        ex_down.close()
        dist.barrier()
        dist.destroy_process_group()


# ---------------------------------------------------------------------------
# Batched workloads, selected with --workload
# ---------------------------------------------------------------------------
GEMM_CONFIGS = {
    # workload: (weight type name, K, N, default batch, config label)
    "q4-gemm": ("q4_0", 4096, 14336, 128, "config 2: q4_0 batched GEMM (prefill), batch in {16, 128, 512}"),
    "f16-gemm": ("f16", 8192, 8192, 64, "config 3: f16 GEMV/GEMM, batch in {1, 64}"),
    "f32-gemm": ("f32", 8192, 8192, 64, "config 3: f32 GEMV/GEMM, batch in {1, 64}"),
    "i8-gemm": ("rowwise_i8", 8192, 28672, 256, "config 4: rowwise-int8 GEMM, batch in {1, 32, 256}"),
}


def gemm_shape(args):
    wname, k, n, batch, label = GEMM_CONFIGS[args.workload]
    return wname, args.k or k, args.n or n, args.batch or batch, label


def gemm_weight_bytes(K, wname: str, k: int, n: int) -> int:
    return {"q4_0": n * (k // 32) * 18, "f16": 2 * n * k, "f32": 4 * n * k}.get(wname) or K.packed_i8_size(k, n)


def gemm_cpu_rate(wname: str, k: int, n: int, batch: int, seconds: float, sample_rows: int = 0):
    """The reference's CPU arithmetic for the batched path on a row sample:
    FP64 dots over the exactly decoded weights (bench/native-q4-reference.h
    reference()) for f32/f16/q4_0 on all host cores, or the rowwise-int8
    two-component integer dots and combine (src/k200.cpp:209-239) on one core.
    Returns (TFLOP/s of the logical 2*n*k*batch work, cores, kind, sample)."""
    import oracle as O

    threads = os.cpu_count() or 1
    rows = sample_rows or max(1, min(n, 64))
    x = (O.normal(0x09200ABC, batch * k, 0.0, 1.0) if wname == "rowwise_i8"
         else O.uniform(0x09200ABC, batch * k, -1.0, 1.0))
    w = O.normal(0x7340D123, rows * k, 0.0, 0.02) if wname in ("q4_0", "rowwise_i8") else \
        O.uniform(0x7340D123, rows * k, -1.0, 1.0)
    if wname == "rowwise_i8":
        wq, scales = O.i8_pack_rows(w, k, rows)
        cores = 1

        def run():
            q0, q1, m0, m1 = O.a8_tensor(x)
            O.i8_matmul(wq, scales, q0, q1, m0, m1, k, rows, batch)
    else:
        if wname == "q4_0":
            dec = O.q4_0_dequantize(O.q4_0_quantize(w, rows, k), rows, k)
        elif wname == "f16":
            dec = O.f16(w).astype(np.float32)
        else:
            dec = w
        cores = threads

        def run():
            O.reference_fp64(dec, x, k, rows, batch, threads)
    run()
    t0 = time.perf_counter()
    done = 0
    while True:
        run()
        done += 1
        if time.perf_counter() - t0 >= seconds and done >= 2:
            break
    dt = time.perf_counter() - t0
    kind = "port"
    sample = (f"{done} calls of {rows} weight rows x K{k} x batch {batch} "
              f"({'int8 dots + combine' if wname == 'rowwise_i8' else 'FP64 reference() over decoded weights'}), "
              f"{dt:.1f} s")
    return 2.0 * rows * k * batch * done / dt / 1e12, cores, kind, sample


def gemm_dtype(wname: str) -> str:
    return {"q4_0": "f16 hi/lo x f16 hi/lo", "f16": "f16 x f16 hi/lo", "f32": "f32", "rowwise_i8": "int8"}[wname]


def measure_gemm(K, torch, dist, dev: int, stream, world: int, rank: int, wname: str, k: int, n: int,
                 batch: int, steps: int, warmup: int, label: str, cpu_seconds: float = 0.0,
                 target_s: float = 0.0) -> dict | None:
    """One batched matmul configuration: rotating
    resident weights (> 2x L2), CUDA-graph steps timed with CUDA events on the
    launching stream (max over ranks), clocks sampled during the timed
    region, and the same steps end to end through the C ABI.  With
    target_s > 0 the step count is chosen so the timed region lasts about
    that long.  Returns rank 0's JSON line (None on other ranks)."""
    from kunlunk200_lib_b200.shard import row_shard

    wtype = {"q4_0": K.Q4_0, "f16": K.F16, "f32": K.F32, "rowwise_i8": K.ROWWISE_I8}[wname]
    if n % world:
        raise SystemExit(f"N={n} does not split evenly over {world} GPUs")
    l2 = torch.cuda.get_device_properties(dev).L2_cache_size
    n_sh = row_shard(n, world, rank)[1]
    shard_bytes = gemm_weight_bytes(K, wname, k, n_sh)
    sets = max(2, math.ceil(2 * l2 / shard_bytes) + 1)
    gen = torch.Generator(device="cuda")
    weights = []
    with torch.cuda.stream(stream):
        for s_ in range(sets):
            gen.manual_seed(1000003 * s_ + 104729 * rank + 5)
            if wname in ("q4_0", "rowwise_i8"):
                w = torch.randn((n_sh, k), generator=gen, device="cuda", dtype=torch.float32) * 0.02
            else:
                w = torch.rand((n_sh, k), generator=gen, device="cuda", dtype=torch.float32) * 2 - 1
            if wname == "q4_0":
                W = torch.empty(shard_bytes, dtype=torch.uint8, device="cuda")
                K.quantize_q4_0(dev, W, w, k, n_sh)
            elif wname == "rowwise_i8":
                W = torch.empty(shard_bytes, dtype=torch.uint8, device="cuda")
                K.pack_i8_rows_device(dev, W, k, n_sh, 0, n_sh, w)
            elif wname == "f16":
                W = w.half()
            else:
                W = w
            del w
            weights.append(W)
        gen.manual_seed(0x09200ABC)
        if wname == "rowwise_i8":
            x = torch.randn((batch, k), generator=gen, device="cuda", dtype=torch.float32)
        else:
            x = torch.rand((batch, k), generator=gen, device="cuda", dtype=torch.float32) * 2 - 1
        y_sh = torch.empty((batch, n_sh), device="cuda")
    # N > 1: Y is gathered over NVLink.  Outputs up to 8 MB take the library's
    # row gather (k200_gather_rows: every rank's slice as tagged words into every
    # rank's exchange, no collective, then k200_gather_wait writes the full
    # [batch][n] Y on the device) -- a few microseconds where NCCL's all-gather
    # costs ~10-15; larger ones take NCCL's all-gather, whose plain 4-byte
    # values cross NVLink once instead of as 8-byte tagged words.
    peer = world > 1 and batch * n * 4 <= (8 << 20)
    y_full = y_sh if world == 1 or peer else torch.empty((world, batch, n_sh), device="cuda")
    stream.synchronize()
    kern = K.Kernel()
    i8 = wname == "rowwise_i8"
    ex = None
    if peer:
        from kunlunk200_lib_b200.shard import PeerExchange

        def all_gather_obj(obj):
            got = [None] * world
            dist.all_gather_object(got, obj)
            return got

        ex = PeerExchange.over_group(K, dev, n, world, rank, all_gather_obj, batch=batch)
        row_begin = row_shard(n, world, rank)[0]
        dist.barrier()  # every rank's regions are mapped before any rank stores into them
        torch.cuda.synchronize()

    def step(s_: int):
        W = weights[s_ % sets]
        sc = K.packed_i8_scales(W, k, n_sh) if i8 else None
        mx = K.packed_i8_maxima(W, k, n_sh) if i8 else None
        K.matmul(kern, dev, y_sh, W, x, k, n_sh, batch, wtype, sc, mx)
        if peer:
            # steps alternate between two exchange buffers (every sequence of
            # steps below has an even length, so the alternation never breaks)
            K.check(K.gather_rows(dev, ex.view(s_), row_begin, y_sh, n_sh, batch))
            K.check(K.gather_wait(dev, ex.view(s_)))
        elif world > 1:
            dist.all_gather_into_tensor(y_full, y_sh)

    def y_out(s_: int) -> int:
        """Address of step s_'s gathered Y on this rank."""
        return ex.output(s_) if peer else y_full.data_ptr()

    nwarm = max(3, warmup)
    if world > 1:
        nwarm += nwarm % 2
    w0, w1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with torch.cuda.stream(stream):
        step(0)  # first call: scratch growth, kernel set-up
        w0.record(stream)
        for i in range(1, nwarm):
            step(i)
        w1.record(stream)
    stream.synchronize()
    K.check(K.wait())
    if target_s > 0:
        est = w0.elapsed_time(w1) / max(1, nwarm - 1) * 1e-3
        t = torch.tensor([est], device="cuda")
        if world > 1:
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
        steps = int(min(4000, max(20, target_s / max(float(t.item()), 1e-6))))
    per_graph = sets * max(1, 24 // sets)
    if world > 1:  # even sequences of steps: the exchange buffers alternate by step parity
        steps += steps % 2
        per_graph *= 1 + per_graph % 2
    reps, rem = divmod(steps, per_graph)

    def capture(nsteps: int):
        if nsteps == 0:
            return None
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g, stream=stream):
            for i in range(nsteps):
                step(i)
        return g

    g_main, g_rem = (capture(per_graph) if reps else None), capture(rem)
    with torch.cuda.stream(stream):
        if g_main is not None:
            g_main.replay()
        if g_rem is not None:
            g_rem.replay()
    stream.synchronize()
    visible = os.environ.get("CUDA_VISIBLE_DEVICES")
    phys = int(visible.split(",")[dev]) if visible and visible.split(",")[dev].strip().isdigit() else dev
    clocks = ClockSampler(phys)
    if rank == 0:
        clocks.start()
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    if rank == 0:
        clocks.mark(True)
    with torch.cuda.stream(stream):
        start.record(stream)
        for _ in range(reps):
            g_main.replay()
        if g_rem is not None:
            g_rem.replay()
        end.record(stream)
    stream.synchronize()
    torch.cuda.synchronize()
    if rank == 0:
        clocks.mark(False)
    if world > 1:
        dist.barrier()
    t = torch.tensor([start.elapsed_time(end)], device="cuda")
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    ms = float(t.item())
    clock_info = clocks.stop() if rank == 0 else None
    if world > 1:  # rank 0's host was busy with the clock record: start the next phase together
        dist.barrier()
        torch.cuda.synchronize()
    flops_step = 2.0 * n * k * batch
    value = flops_step * steps / (ms * 1e-3) / 1e12
    ms_step = ms / steps
    # kernels of ours per matmul: the activation preparation (f16/q4_0 hi/lo
    # split; rowwise-int8 quantiser: one CTA up to 64K elements, else three
    # passes) and the matmul kernel itself
    tc = batch >= 4 and k % 16 == 0 and (wname != "q4_0" or k % 256 == 0) and wname != "f32"
    prep = (1 if (tc and wname in ("q4_0", "f16")) else 0) + ((1 if batch * k <= 65536 else 3) if i8 else 0)
    launches = steps * (1 + prep + (2 if peer else 0))
    peaks = read_peaks()
    hbm_gbs = shard_bytes / (ms_step * 1e-3) / 1e9
    tflops_gpu = flops_step / world / (ms_step * 1e-3) / 1e12
    tensor_peak = peaks["bf16_tflops"] * (2 if i8 else 1)
    hbm_frac, tensor_frac = hbm_gbs / peaks["hbm_gbs"], tflops_gpu / tensor_peak
    bound = "tensor" if tensor_frac > hbm_frac else "hbm"
    f32_gemm = wname == "f32" and batch >= 9 and k % 64 == 0
    kernel = ({"q4_0": "gemm_q4_kernel", "f16": "gemm_f16_kernel", "rowwise_i8": "gemm_i8_kernel"}[wname] if tc
              else "gemm_f32_kernel" if f32_gemm else "gemv_stream_kernel")
    roof = {"bound": bound,
            "achieved": tflops_gpu if bound == "tensor" else hbm_gbs,
            "peak": tensor_peak if bound == "tensor" else peaks["hbm_gbs"],
            "unit": "TFLOP/s" if bound == "tensor" else "GB/s",
            "frac": tensor_frac if bound == "tensor" else hbm_frac,
            "hbm": {"achieved": hbm_gbs, "frac": hbm_frac},
            "tensor": {"achieved": tflops_gpu, "frac": tensor_frac,
                       "peak_note": ("2x measured bf16 (dense int8 rate)" if i8 else "measured bf16")},
            "peak_source": peaks["source"], "traffic": None, "kernel": kernel, "launch_us": ms_step * 1e3}
    # end to end through the C ABI: pinned host X in, pinned host Y out, every step
    e2e_steps = max(10, min(steps, 500))
    xh = torch.empty((batch, k), dtype=torch.float32).pin_memory()
    xh.copy_(x.cpu())
    yh = torch.empty(batch * n, dtype=torch.float32).pin_memory()
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with torch.cuda.stream(stream):
        e0.record(stream)
        for i in range(e2e_steps):
            K.check(K.copy_async(x, xh, xh.numel() * 4, K.HOST_TO_DEVICE))
            step(i)
            K.check(K.copy_async(yh, y_out(i), yh.numel() * 4, K.DEVICE_TO_HOST))
            K.check(K.wait())
        e1.record(stream)
    stream.synchronize()
    te = torch.tensor([e0.elapsed_time(e1)], device="cuda")
    if world > 1:
        dist.all_reduce(te, op=dist.ReduceOp.MAX)
    e2e_value = flops_step * e2e_steps / (float(te.item()) * 1e-3) / 1e12
    cpu = None
    if rank == 0 and world == 1 and cpu_seconds > 0:
        v, cores, kind, sample = gemm_cpu_rate(wname, k, n, batch, cpu_seconds)
        cpu = {"value": v, "unit": "TFLOP/s", "cores": cores, "kind": kind, "sample": sample}
    del g_main, g_rem
    if ex is not None:
        dist.barrier()  # no rank still reads another's region
        ex.close()
    kern.close()
    del weights
    torch.cuda.synchronize()
    if rank != 0:
        return None
    unit = "TOP/s" if i8 else "TFLOP/s"
    return {
        "metric": f"{wname}_batched_matmul_tflops", "value": value, "unit": unit, "n_gpus": world,
        "steps": steps, "warmup": warmup, "ms_per_step": ms_step, "higher_is_better": True,
        "scaling": "strong", "vs_baseline": None, "dtype": gemm_dtype(wname), "data": "synthetic",
        "config": {"workload": f"{wname} matmul K{k} N{n} batch {batch} ({label})", "k": k, "n": n, "batch": batch,
                   "parallelism": (f"row-shard{world}+" + ("peer-gather" if peer else "nccl-allgather")) if world > 1
                                  else "single",
                   "work": "logical 2*N*K*batch per step",
                   "l2": f"{sets} rotating weight sets ({sets * shard_bytes / 1e6:.0f} MB per GPU)",
                   "timing": "CUDA graph replays, CUDA events on the launching stream, max over ranks"},
        "roofline": roof, "cpu_baseline": cpu,
        "e2e": {"value": e2e_value, "unit": unit, "h2d_bytes_per_step": xh.numel() * 4,
                "d2h_bytes_per_step": yh.numel() * 4, "steps": e2e_steps,
                "path": "k200_copy_async H2D + k200_matmul + k200_copy_async D2H + k200_wait per step"},
        "gpu_launches": launches, "clocks": clock_info,
    }


# The batched half of the metric, measured in the default run beside the
# batch-1 GEMV (BASELINE configs 2-4 at their prefill / decode-batch sizes).
BATCHED_SET = [("q4_0", 4096, 14336, 128, "config 2"), ("q4_0", 4096, 14336, 512, "config 2"),
               ("f16", 8192, 8192, 64, "config 3"), ("f32", 8192, 8192, 64, "config 3"),
               ("rowwise_i8", 8192, 28672, 256, "config 4")]


def run_gemm(args) -> None:
    import torch
    import torch.distributed as dist

    import kunlunk200_lib_b200 as K

    wname, k, n, batch, label = gemm_shape(args)
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world != args.gpus:
        raise SystemExit(f"--gpus {args.gpus} but WORLD_SIZE={world}: launch N>1 with torchrun")
    torch.cuda.set_device(local)
    if world > 1:
        import datetime

        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120), device_id=torch.device("cuda", local))
    dev = local
    K.select(dev)
    stream = torch.cuda.Stream()
    K.set_stream(dev, stream.cuda_stream)
    K.set_static_weights(dev, True)
    line = measure_gemm(K, torch, dist, dev, stream, world, rank, wname, k, n, batch, args.steps, args.warmup, label,
                        cpu_seconds=0.0 if args.no_cpu_baseline else 10.0)
    if line is not None:
        print(json.dumps(line), flush=True)
    K.set_stream(dev, None)
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()


def run_gemm_reference(args) -> None:
    if int(os.environ.get("RANK", "0")) != 0:
        return
    wname, k, n, batch, label = gemm_shape(args)
    import oracle as O  # noqa: F401  (the reference CPU arithmetic lives in the oracle)

    per_step = 120.0 / max(1, args.steps + args.warmup)
    value, cores, kind, sample = gemm_cpu_rate(wname, k, n, batch, max(0.05, per_step) * args.steps)
    unit = "TOP/s" if wname == "rowwise_i8" else "TFLOP/s"
    line = {"impl": "reference", "metric": f"{wname}_batched_matmul_tflops", "value": value, "unit": unit,
            "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup, "higher_is_better": True,
            "scaling": "strong", "vs_baseline": None, "dtype": "f64" if wname != "rowwise_i8" else "int8",
            "data": "synthetic", "config": {"workload": f"{wname} matmul K{k} N{n} batch {batch} ({label})"},
            "cpu_baseline": {"value": value, "unit": unit, "cores": cores, "kind": kind, "sample": sample},
            "e2e": {"value": value, "unit": unit, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=100000)
    ap.add_argument("--warmup", type=int, default=200)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-batched", action="store_true", help="default workload: skip the batched configs 2-4")
    ap.add_argument("--workload", choices=["gemv"] + sorted(GEMM_CONFIGS), default="gemv",
                    help="gemv: config 1 (the metric's workload, default); others: BASELINE configs 2-4")
    ap.add_argument("--batch", type=int, default=0, help="batched workloads: activation columns")
    ap.add_argument("--k", type=int, default=0, help="batched workloads: override K")
    ap.add_argument("--n", type=int, default=0, help="batched workloads: override N")
    args = ap.parse_args()
    if args.warmup < 3:
        args.warmup = 3
    if args.workload != "gemv":
        if args.steps == 100000:
            args.steps = 200
        run_gemm_reference(args) if args.impl == "reference" else run_gemm(args)
    elif args.impl == "reference":
        run_reference(args)
    else:
        run_ours(args)


if __name__ == "__main__":
    main()
