#!/usr/bin/env python3
"""Benchmark of the B200 quantized-linear path (driver contract: one JSON line).

Workload (BASELINE config 2 at M = 5184 tokens, the headline Q4_K profile):
one "step" is one ViT block's four quantized linears, each from F32
activations (K1 staging + K2 tcgen05 GEMM), with bias and F32 output:
  qkv  1024 -> 3072  Q4_K
  proj 1024 -> 1024  Q4_K
  fc1  1024 -> 4736  Q4_K  + erf-GELU
  fc2  4736 -> 1024  Q8_0  (K = 4736 is not a multiple of 256; the reference
                            stores fc2 as Q8_0 in every K-quant profile,
                            src/models/sam3/weights.hpp:148-164)
Weights are N(0, 0.02^2) with 1% of entries x8, seeds 0-3; activations
N(0, 1).  Synthetic data: no checkpoint exists on the box.

`value` is q-GEMM throughput (2*M*N*K summed over the 4 linears, all ranks)
with inputs resident in HBM; `e2e` is the same metric through the C ABI with
host buffers (pinned H2D of X and D2H of Y inside the timed region).
Multi-GPU: images shard across GPUs with no exchange (weak scaling, one
process per GPU, no collective on the data path).

`--impl reference` times the CPU restatement of the reference's GGML CPU path
(oracle/, GGML itself is not buildable here) on the box's host cores.
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import threading
import time
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))
sys.path.insert(0, str(ROOT / "sam.cpp_b200"))

M = 5184
LINEARS = [  # name, n, k, weight type, epilogue, seed
    ("qkv", 3072, 1024, 12, 0, 0),
    ("proj", 1024, 1024, 12, 0, 1),
    ("fc1", 4736, 1024, 12, 1, 2),
    ("fc2", 1024, 4736, 8, 0, 3),
]
WORKLOAD = "vit_block_linears_q4k_m5184"
METRIC = "SAM3 ViT-block quantized-linear throughput (q-GEMM TOPS, Q4_K + Q8_0 fc2, 5184 tokens)"


def step_ops(m=M):
    return sum(2.0 * m * n * k for _, n, k, *_ in LINEARS)


def make_weights(oracle_mod, n, k, qtype, seed):
    rng = np.random.default_rng(seed)
    w = rng.normal(0.0, 0.02, (n, k)).astype(np.float32)
    mask = rng.random(w.shape) < 0.01
    w[mask] *= 8
    bias = rng.normal(0.0, 0.02, n).astype(np.float32)
    return oracle_mod.quantize(qtype, w), bias


def peaks():
    """Roofline denominators.  The GEMMs run inside a long loop of steps, where
    the SMs settle at ~1.65 GHz (clock64 against %globaltimer in the kernels),
    so the sustained bf16 figure is the tensor peak; the fallback is the
    earlier measurement on this pool."""
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        return {"bf16_tflops": d.get("bf16_tflops_sustained") or d.get("bf16_tflops"),
                "bf16_tflops_burst": d.get("bf16_tflops"), "hbm_gbs": d.get("hbm_gbs"),
                "source": "measured sustained"}
    return {"bf16_tflops": 1400.0, "bf16_tflops_burst": 1590.0, "hbm_gbs": 6650.0, "source": "fallback"}


def profiled_traffic():
    """DRAM bytes per GEMM launch from the committed ncu summary, if any."""
    p = ROOT / "profiles" / "gemm_traffic.json"
    if p.exists():
        try:
            return json.loads(p.read_text())
        except ValueError:
            return None
    return None


class ClockSampler:
    """nvidia-smi clocks / throttle reasons sampled during the timed region."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index: int):
        self.gpu = gpu_index
        self.proc = None
        self.lines = []
        self.thread = None

    def start(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--id={self.gpu}", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                 "-lms", "50"], stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except OSError:
            self.proc = None
            return
        self.thread = threading.Thread(target=self._read, daemon=True)
        self.thread.start()
        time.sleep(0.15)

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    def stop(self):
        if not self.proc:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        time.sleep(0.1)
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
        if self.thread:
            self.thread.join(timeout=2)
        sm, smax, power, reasons = [], [], [], set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for line in self.lines:
            parts = [p.strip() for p in line.split(",")]
            if len(parts) < 9:
                continue
            try:
                sm.append(float(parts[1]))
                smax.append(float(parts[2]))
                power.append(float(parts[3]))
            except ValueError:
                continue
            for name, flag in zip(names, parts[5:9]):
                if flag.lower() == "active":
                    reasons.add(name)
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": max(smax) if smax else None,
                "power_w_max": max(power) if power else None, "samples": len(sm), "reasons": sorted(reasons)}


def dist_setup():
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    return world, rank, local


def cpu_sample_rate(oracle_mod, weights, threads, budget_s):
    """Oracle (restated GGML CPU path) throughput on a bounded sample of rows."""
    rng = np.random.default_rng(99)
    rows = 16
    xs = {name: rng.normal(0, 1, (rows, k)).astype(np.float32) for name, n, k, *_ in LINEARS}

    def run(r):
        t0 = time.perf_counter()
        for (name, n, k, qtype, epi, _), (packed, bias) in zip(LINEARS, weights):
            oracle_mod.cpu_linear(qtype, packed, k, n, xs[name][:r] if r <= rows else
                                  np.resize(xs[name], (r, k)), bias=bias, epilogue=epi, threads=threads)
        return time.perf_counter() - t0

    run(rows)  # warm-up (first-touch, thread pool)
    t = run(rows)
    per_row = t / rows
    sample_rows = int(max(rows, min(M, budget_s / max(per_row, 1e-9) / 2)))
    reps, total, start = 0, 0.0, time.perf_counter()
    while reps < 1 or (time.perf_counter() - start < budget_s and reps < 400):
        total += run(sample_rows)
        reps += 1
    ops = step_ops(sample_rows) * reps
    return ops / total / 1e12, sample_rows, reps, total


def run_reference(args, world, rank):
    """CPU reference arm: rank 0 times the restated GGML CPU path."""
    if rank != 0:
        return
    from oracle import oracle as o
    o.lib()
    threads = o.default_threads()
    weights = [make_weights(o, n, k, qtype, seed) for _, n, k, qtype, _, seed in LINEARS]
    rng = np.random.default_rng(7)
    # Size each step's row sample so the whole run stays within ~2 minutes.
    probe = {name: rng.normal(0, 1, (8, k)).astype(np.float32) for name, n, k, *_ in LINEARS}
    t0 = time.perf_counter()
    for (name, n, k, qtype, epi, _), (packed, bias) in zip(LINEARS, weights):
        o.cpu_linear(qtype, packed, k, n, probe[name], bias=bias, epilogue=epi, threads=threads)
    per_row = (time.perf_counter() - t0) / 8
    budget = 100.0 / max(args.steps + args.warmup, 1)
    rows = int(max(8, min(M, budget / max(per_row, 1e-9))))
    xs = {name: rng.normal(0, 1, (rows, k)).astype(np.float32) for name, n, k, *_ in LINEARS}
    ys = {name: np.empty((rows, n), np.float32) for name, n, *_ in LINEARS}

    def step():
        for (name, n, k, qtype, epi, _), (packed, bias) in zip(LINEARS, weights):
            o.cpu_linear(qtype, packed, k, n, xs[name], bias=bias, epilogue=epi, threads=threads, out=ys[name])

    for _ in range(args.warmup):
        step()
    t0 = time.perf_counter()
    for _ in range(args.steps):
        step()
    elapsed = time.perf_counter() - t0
    value = step_ops(rows) * args.steps / elapsed / 1e12
    line = {
        "impl": "reference", "metric": METRIC, "value": value, "unit": "TOPS", "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": elapsed / args.steps * 1e3,
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "int8xint8->f32",
        "data": "synthetic",
        "config": {"workload": WORKLOAD, "rows_per_step": rows, "tokens": M,
                   "linears": [l[0] for l in LINEARS], "formats": ["Q4_K", "Q4_K", "Q4_K", "Q8_0"]},
        "cpu_baseline": {"value": value, "unit": "TOPS", "cores": threads, "kind": "port",
                         "sample": f"{rows} of {M} token rows per step through the 4 linears; "
                                   "CPU restatement of GGML's CPU mul_mat (Q8_0xQ8_0, K-quant xQ8_K, "
                                   f"OpenMP, AVX-512 VNNI={'yes' if o.has_vnni() else 'no'}); GGML unavailable"},
        "e2e": {"value": value, "unit": "TOPS", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=2000)
    ap.add_argument("--warmup", type=int, default=20)
    ap.add_argument("--impl", default="samq", choices=["samq", "reference"])
    ap.add_argument("--e2e-steps", type=int, default=20)
    ap.add_argument("--cpu-budget", type=float, default=12.0, help="seconds of CPU baseline work")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--profile", choices=[l[0] for l in LINEARS],
                    help="only stage one linear's A operand and launch its GEMM --steps times "
                         "(small, single-kernel case for ncu captures)")
    args = ap.parse_args()
    args.warmup = max(args.warmup, 3)
    world, rank, local = dist_setup()

    if args.impl == "reference":
        run_reference(args, world, rank)
        return
    if args.profile:
        run_profile_case(args)
        return

    import torch
    import torch.distributed as dist
    import samq
    from oracle import oracle as o

    torch.cuda.set_device(local)
    if world > 1:
        from datetime import timedelta
        dist.init_process_group("nccl", timeout=timedelta(seconds=120), device_id=torch.device("cuda", local))
    samq.init(local)
    stream = torch.cuda.current_stream()

    weights, biases, xs, ys, host = [], [], [], [], []
    for name, n, k, qtype, epi, seed in LINEARS:
        packed, bias = make_weights(o, n, k, qtype, seed + 4 * rank)
        weights.append(samq.Weights(qtype, k, n, packed, device=local))
        biases.append(torch.from_numpy(bias).cuda())
        rng = np.random.default_rng(1000 + seed + 17 * rank)
        x = rng.normal(0, 1, (M, k)).astype(np.float32)
        xs.append(torch.from_numpy(x).cuda())
        ys.append(torch.empty((M, n), dtype=torch.float32, device="cuda"))
        host.append((torch.from_numpy(x).pin_memory(), torch.empty((M, n), dtype=torch.float32).pin_memory()))

    def launch(i):
        name, n, k, qtype, epi, _ = LINEARS[i]
        samq.linear(weights[i], xs[i], M, k, biases[i], epi, ys[i], n, stream)

    # Warm-up (also grows the per-stream scratch before timing).
    for _ in range(args.warmup):
        for i in range(len(LINEARS)):
            launch(i)
    torch.cuda.synchronize()
    samq.check(local, stream)

    # Timed region: K steps, barrier + synchronize on both sides, max over ranks.
    sample_every = max(1, args.steps // 200)
    events = []
    sampler = ClockSampler(int(os.environ.get("CUDA_VISIBLE_DEVICES", str(local)).split(",")[0])
                           if os.environ.get("CUDA_VISIBLE_DEVICES", "").split(",")[0].isdigit() else local)
    sampler.start()
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    start.record(stream)
    for s in range(args.steps):
        if s % sample_every == 0:
            evs = [torch.cuda.Event(enable_timing=True) for _ in range(2 * len(LINEARS))]
            for i in range(len(LINEARS)):
                evs[2 * i].record(stream)
                launch(i)
                evs[2 * i + 1].record(stream)
            events.append(evs)
        else:
            for i in range(len(LINEARS)):
                launch(i)
    end.record(stream)
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    clocks = sampler.stop()
    elapsed_ms = start.elapsed_time(end)
    samq.check(local, stream)
    t = torch.tensor([elapsed_ms], dtype=torch.float64, device="cuda")
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    elapsed_ms = float(t.item())
    value = step_ops() * args.steps * world / (elapsed_ms / 1e3) / 1e12

    # Per-launch durations of the sampled steps (linear = K1 + GEMM).
    per_linear = np.array([[evs[2 * i].elapsed_time(evs[2 * i + 1]) for i in range(len(LINEARS))] for evs in events])
    linear_ms = per_linear.mean(axis=0)

    # GEMM-only launch durations (dominant kernel) over a separate sampled pass
    # of the same launches: K1 staging is timed with its own events.
    gemm_ms = gemm_only_durations(samq, weights, xs, ys, biases, stream)

    # End to end through the C ABI with host buffers.
    e2e_steps = max(3, args.e2e_steps)
    h2d = sum(x.numel() * 4 for x, _ in host)
    d2h = sum(y.numel() * 4 for _, y in host)

    def e2e_step():
        for i, (name, n, k, qtype, epi, _) in enumerate(LINEARS):
            xs[i].copy_(host[i][0], non_blocking=True)
            samq.linear(weights[i], xs[i], M, k, biases[i], epi, ys[i], n, stream)
            host[i][1].copy_(ys[i], non_blocking=True)

    for _ in range(3):
        e2e_step()
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for _ in range(e2e_steps):
        e2e_step()
    e1.record(stream)
    torch.cuda.synchronize()
    e2e_ms = torch.tensor([e0.elapsed_time(e1)], dtype=torch.float64, device="cuda")
    if world > 1:
        dist.all_reduce(e2e_ms, op=dist.ReduceOp.MAX)
    e2e_value = step_ops() * e2e_steps * world / (float(e2e_ms.item()) / 1e3) / 1e12

    pk = peaks()
    gemm_flops = [2.0 * M * n * k for _, n, k, *_ in LINEARS]
    achieved = sum(gemm_flops) / (sum(gemm_ms) / 1e3) / 1e12
    traffic = profiled_traffic()
    roofline = {"bound": "tensor", "kernel": "gemm_f16_kernel (tcgen05 kind::f16, f32 accumulate)",
                "achieved": achieved, "peak": pk["bf16_tflops"], "unit": "TFLOP/s",
                "frac": achieved / pk["bf16_tflops"], "peak_source": f"{pk['source']} bf16",
                "frac_of_burst": achieved / pk["bf16_tflops_burst"],
                "traffic": traffic.get("bytes_per_launch") if traffic else None,
                "traffic_source": traffic.get("source") if traffic else None,
                "per_linear_gemm_us": {LINEARS[i][0]: gemm_ms[i] * 1e3 for i in range(len(LINEARS))},
                "per_linear_total_us": {LINEARS[i][0]: float(linear_ms[i]) * 1e3 for i in range(len(LINEARS))}}

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        threads = o.default_threads()
        packed = [make_weights(o, n, k, qtype, seed) for _, n, k, qtype, _, seed in LINEARS]
        rate, rows, reps, secs = cpu_sample_rate(o, packed, threads, args.cpu_budget)
        cpu = {"value": rate, "unit": "TOPS", "cores": threads, "kind": "port",
               "sample": f"{reps} x {rows} of {M} token rows through the 4 linears ({secs:.1f} s); CPU "
                         "restatement of GGML's CPU mul_mat (GGML itself unavailable), OpenMP"
                         f"{' + AVX-512 VNNI' if o.has_vnni() else ''}"}

    if rank == 0:
        line = {
            "metric": METRIC, "value": value, "unit": "TOPS", "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": elapsed_ms / args.steps, "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": "f16", "data": "synthetic",
            "config": {"workload": WORKLOAD, "tokens": M, "linears": [l[0] for l in LINEARS],
                       "shapes_nk": [[l[1], l[2]] for l in LINEARS], "formats": ["Q4_K", "Q4_K", "Q4_K", "Q8_0"],
                       "epilogues": ["bias", "bias", "bias+gelu_erf", "bias"], "input": "f32 activations",
                       "l2": "inputs exceed L2 (162 MB of X + 204 MB of Y per step)",
                       "parallelism": f"images sharded, {world} replica(s)"},
            "roofline": roofline,
            "cpu_baseline": cpu,
            "e2e": {"value": e2e_value, "unit": "TOPS", "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h,
                    "steps": e2e_steps},
            "gpu_launches": args.steps * 2 * len(LINEARS),
            "clocks": clocks,
        }
        print(json.dumps(line), flush=True)
    for w in weights:
        w.close()
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()


def run_profile_case(args):
    """One linear's GEMM launched alone, for ncu (-k regex:gemm)."""
    import torch
    import samq
    from oracle import oracle as o
    torch.cuda.set_device(0)
    samq.init(0)
    stream = torch.cuda.current_stream()
    name, n, k, qtype, epi, seed = next(l for l in LINEARS if l[0] == args.profile)
    packed, bias = make_weights(o, n, k, qtype, seed)
    w = samq.Weights(qtype, k, n, packed)
    x = torch.from_numpy(np.random.default_rng(seed).normal(0, 1, (M, k)).astype(np.float32)).cuda()
    a16 = torch.empty((M, k), dtype=torch.float16, device="cuda")
    y = torch.empty((M, n), dtype=torch.float32, device="cuda")
    b = torch.from_numpy(bias).cuda()
    samq.stage_f16(x, M, k, k, a16, stream)
    for _ in range(args.warmup + args.steps):
        samq.linear_f16(w, a16, M, k, b, epi, y, n, stream)
    torch.cuda.synchronize()
    samq.check(0, stream)
    w.close()
    print(json.dumps({"profile_case": name, "launches": args.warmup + args.steps}))


def gemm_only_durations(samq, weights, xs, ys, biases, stream, reps=50):
    """Average device time of each GEMM launch alone: the f16 A operand is
    staged once (samq_stage_f16_v1), then samq_linear_f16_v1 launches only the
    tcgen05 GEMM kernel, bracketed by events on the launching stream."""
    import torch
    out = []
    for i, (name, n, k, qtype, epi, _) in enumerate(LINEARS):
        m = xs[i].shape[0]
        a16 = torch.empty((m, k), dtype=torch.float16, device="cuda")
        samq.stage_f16(xs[i], m, k, k, a16, stream)
        for _ in range(3):
            samq.linear_f16(weights[i], a16, m, k, biases[i], epi, ys[i], n, stream)
        evs = []
        for _ in range(reps):
            a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            a.record(stream)
            samq.linear_f16(weights[i], a16, m, k, biases[i], epi, ys[i], n, stream)
            b.record(stream)
            evs.append((a, b))
        torch.cuda.synchronize()
        out.append(float(np.mean([a.elapsed_time(b) for a, b in evs])))
    return out


if __name__ == "__main__":
    main()
