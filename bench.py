#!/usr/bin/env python3
"""Benchmark of the B200 SAM 3 quantized path (driver contract: one JSON line).

Headline workload: the full SAM 3 vision backbone on one
1008 x 1008 image per GPU, batch 1: patch embedding + pos_embed + ln_pre, then
32 pre-LN ViT blocks (width 1024, 16 heads, MLP 4736, 2D RoPE; windowed 24x24
attention except global blocks 7, 15, 23, 31) with Q4_K qkv / proj / fc1 and
Q8_0 fc2 (src/models/sam3/weights.hpp:148-164), every linear fed Q8_1-staged
activations.  One "step" is one image through samq_vit_prefix_v1 and 32
samq_vit_block_forward_v1 calls.  `value` is images/s over all ranks with the
image resident in HBM; `e2e` adds, every step, the pinned host->device copy of
the normalized image and the device->host read of the 5184 x 1024 features.
Weights are random-init (N(0, 0.02^2), 1% x8), the image U[0,1] normalized:
synthetic, no checkpoint exists on the box.

`qgemm` reports BASELINE config 2 beside it: one ViT block's four quantized
linears at M = 5184 from f32 activations (K1 staging + K2 GEMM) in q-GEMM
TOPS, with the GEMM roofline.  Multi-GPU: images shard across GPUs with no
exchange (weak scaling, one process per GPU, no collective on the data path).

`--impl reference` times the CPU restatement of the reference's GGML CPU path
(oracle/; GGML itself is not buildable here) on the box's host cores over a
bounded sample of the backbone and reports the same images/s metric.
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
QGEMM_WORKLOAD = "vit_block_linears_q4k_m5184"
QGEMM_METRIC = "SAM3 ViT-block quantized-linear throughput (q-GEMM TOPS, Q4_K + Q8_0 fc2, 5184 tokens)"
WORKLOAD = "sam3_vit_backbone_q4k_1008px_batch1"
METRIC = "SAM3 vision backbone images/s (Q4_K, fc2 Q8_0, 1008x1008, batch 1 per GPU)"
E, MLP, HEADS, GRID, PATCH, IMAGE, POS_GRID, DEPTH, WINDOW = 1024, 4736, 16, 72, 14, 1008, 24, 32, 24
GLOBAL_BLOCKS = (7, 15, 23, 31)


def workload_config(world):
    """The `config` object of both arms' JSON lines (the same workload)."""
    lin_ops, attn_ops = backbone_ops()
    return {"workload": WORKLOAD, "image": f"{IMAGE}x{IMAGE}x3", "patch": PATCH, "tokens": M,
            "width": E, "heads": HEADS, "mlp": MLP, "blocks": DEPTH, "window": WINDOW,
            "global_blocks": list(GLOBAL_BLOCKS),
            "formats": {"qkv/proj/fc1": "Q4_K", "fc2": "Q8_0", "norms/biases/embeddings": "f32"},
            "batch_per_gpu": 1, "parallelism": f"images sharded, {world} replica(s)",
            "l2": "weights 1.1 GB per replica and 91 MB of block scratch exceed L2",
            "tflop_per_image": {"linears": lin_ops / 1e12, "attention": attn_ops / 1e12}}


def backbone_ops():
    """Algorithmic work of one image: 2 M N K over the 128 block linears and
    the patch GEMM, plus 4 N_q N_k hd per head of attention."""
    lin = DEPTH * step_ops() + 2.0 * M * E * 3 * PATCH * PATCH
    attn = (DEPTH - len(GLOBAL_BLOCKS)) * 4.0 * (GRID // WINDOW) ** 2 * (WINDOW * WINDOW) ** 2 * 64 * HEADS
    attn += len(GLOBAL_BLOCKS) * 4.0 * M * M * 64 * HEADS
    return lin, attn


def step_ops(m=M):
    return sum(2.0 * m * n * k for _, n, k, *_ in LINEARS)


def make_weights(quantize, n, k, qtype, seed):
    """Config-2 statistics: N(0, 0.02^2) with 1% of entries x8; `quantize`
    packs them (samq.quantize_rows on the GPU arm, the oracle's packer in the
    CPU baseline)."""
    rng = np.random.default_rng(seed)
    w = rng.normal(0.0, 0.02, (n, k)).astype(np.float32)
    mask = rng.random(w.shape) < 0.01
    w[mask] *= 8
    bias = rng.normal(0.0, 0.02, n).astype(np.float32)
    return quantize(qtype, w), bias


def peaks():
    """Roofline denominators from MEASURED_PEAKS.json: the GEMM roofline is
    measured on isolated launches (each timed alone between CUDA events after
    an L2 flush), so its denominator is the burst bf16 figure; the sustained
    one is reported beside it.  The fallback is the earlier measurement on this
    pool."""
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        return {"bf16_tflops": d.get("bf16_tflops") or d.get("bf16_tflops_sustained"),
                "bf16_tflops_sustained": d.get("bf16_tflops_sustained"), "hbm_gbs": d.get("hbm_gbs"),
                "source": "measured burst"}
    return {"bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0, "hbm_gbs": 6650.0, "source": "fallback burst"}


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


def cpu_linears_rate(oracle_mod, weights, threads, budget_s):
    """Oracle (restated GGML CPU path) q-GEMM throughput on a bounded row sample."""
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
    per_row = run(rows) / rows
    sample_rows = int(max(rows, min(M, budget_s / max(per_row, 1e-9) / 2)))
    reps, total, start = 0, 0.0, time.perf_counter()
    while reps < 1 or (time.perf_counter() - start < budget_s and reps < 400):
        total += run(sample_rows)
        reps += 1
    return step_ops(sample_rows) * reps / total / 1e12, sample_rows, reps, total


class CpuBackbone:
    """Bounded samples of the CPU backbone, extrapolated to seconds per image.

    The reference's CPU path is GGML's: quantized mul_mat (restated by
    oracle_cpu_linear: Q8_K / Q8_0 activation packing, integer block dots,
    OpenMP, AVX-512 VNNI when present), flash attention over F32 Q / K / V
    (restated by oracle_flash_attn_f32: per-row f32 online softmax, OpenMP),
    LayerNorm and the f32 patch convolution (numpy f32 / BLAS here).  One
    sample (`step`) is: `rows` token rows through one block's 4 linears (+2
    LayerNorms), one 24x24 window of 16-head attention, and `qrows` query rows
    of one head of global attention over all 5184 keys.  The patch convolution
    is timed once.
    """

    def __init__(self, oracle_mod, rows=1024, qrows=256):
        self.o = oracle_mod
        self.threads = oracle_mod.default_threads()
        self.rows, self.qrows = rows, qrows
        self.weights = [make_weights(oracle_mod.quantize, n, k, qtype, seed) for _, n, k, qtype, _, seed in LINEARS]
        rng = np.random.default_rng(11)
        self.x = {name: rng.normal(0, 1, (rows, k)).astype(np.float32) for name, n, k, *_ in LINEARS}
        self.y = {name: np.empty((rows, n), np.float32) for name, n, *_ in LINEARS}
        self.ln = rng.normal(0, 1, (rows, E)).astype(np.float32)
        self.qkv_w = rng.normal(0, 1, (WINDOW * WINDOW, 3 * E)).astype(np.float32)
        self.att_w = np.empty((WINDOW * WINDOW, E), np.float32)
        self.qg = rng.normal(0, 1, (qrows, 64)).astype(np.float32)
        self.kg = rng.normal(0, 1, (M, 64)).astype(np.float32)
        self.vg = rng.normal(0, 1, (M, 64)).astype(np.float32)
        self.att_g = np.empty((qrows, 64), np.float32)
        cols = rng.normal(0, 1, (M, 3 * PATCH * PATCH)).astype(np.float32)
        pw = rng.normal(0, 0.02, (3 * PATCH * PATCH, E)).astype(np.float32)
        t0 = time.perf_counter()
        for _ in range(3):
            cols @ pw
        self.prefix_s = (time.perf_counter() - t0) / 3

    def step(self):
        """One sample; returns the seconds per image it implies."""
        t0 = time.perf_counter()
        for (name, n, k, qtype, epi, _), (packed, bias) in zip(LINEARS, self.weights):
            self.o.cpu_linear(qtype, packed, k, n, self.x[name], bias=bias, epilogue=epi, threads=self.threads,
                              out=self.y[name])
        for _ in range(2):
            c = self.ln - self.ln.mean(axis=1, keepdims=True)
            c / np.sqrt((c * c).mean(axis=1, keepdims=True) + 1e-5)
        t1 = time.perf_counter()
        for h in range(HEADS):
            self.o.flash_attn_f32(self.qkv_w[:, 64 * h:64 * h + 64], self.qkv_w[:, E + 64 * h:E + 64 * h + 64],
                                  self.qkv_w[:, 2 * E + 64 * h:2 * E + 64 * h + 64], 0.125, threads=self.threads,
                                  out=self.att_w[:, 64 * h:64 * h + 64])
        t2 = time.perf_counter()
        self.o.flash_attn_f32(self.qg, self.kg, self.vg, 0.125, threads=self.threads, out=self.att_g)
        t3 = time.perf_counter()
        per_block_rows = (t1 - t0) * M / self.rows
        windowed = (t2 - t1) * (GRID // WINDOW) ** 2
        global_ = (t3 - t2) * (M / self.qrows) * HEADS
        return (DEPTH * per_block_rows + (DEPTH - len(GLOBAL_BLOCKS)) * windowed + len(GLOBAL_BLOCKS) * global_
                + self.prefix_s)

    def describe(self):
        return (f"per sample: {self.rows} of {M} token rows through one block's 4 linears + 2 LayerNorms "
                f"(restated GGML CPU mul_mat, OpenMP{', AVX-512 VNNI' if self.o.has_vnni() else ''}), one 24x24 "
                f"window of 16-head attention and {self.qrows} query rows of one global-attention head over "
                f"{M} keys (restated GGML CPU flash attention, f32 online softmax, OpenMP); patch conv timed once; "
                "extrapolated to 32 blocks (4 global) per image; GGML itself unavailable")


def run_reference(args, world, rank):
    """CPU reference arm: rank 0 times the restated CPU backbone (images/s).
    A step is one image, its time extrapolated from one bounded sample of
    every component; ms_per_step is that per-image time (1000 / value)."""
    if rank != 0:
        return
    from oracle import oracle as o
    o.lib()
    cpu = CpuBackbone(o)
    for _ in range(args.warmup):
        cpu.step()
    t0 = time.perf_counter()
    per_image = [cpu.step() for _ in range(args.steps)]
    wall = time.perf_counter() - t0
    mean_s = float(np.mean(per_image))
    value = 1.0 / mean_s
    line = {
        "impl": "reference", "metric": METRIC, "value": value, "unit": "images/s", "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": mean_s * 1e3,
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "int8xint8->f32 / f32",
        "data": "synthetic",
        "config": workload_config(world),
        "step": "one image, extrapolated from one bounded sample of each component",
        "wall_ms_per_sample": wall / args.steps * 1e3,
        "cpu_baseline": {"value": value, "unit": "images/s", "cores": cpu.threads, "kind": "port",
                         "sample": cpu.describe()},
        "e2e": {"value": value, "unit": "images/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


def make_backbone(samq, torch, device, rank, compute=None):
    """Random-init SAM 3 vision backbone on `device` (config 3 statistics),
    blocks in the headline compute mode (F16) unless `compute` is given."""
    from samq.synthetic import rope_freqs
    compute = samq.COMPUTE_F16 if compute is None else compute
    dev = torch.device("cuda", device)
    blocks, keep = [], []
    base = np.random.default_rng(2024 + rank)
    freqs_w = torch.from_numpy(rope_freqs(WINDOW * WINDOW, seed=1)).to(dev)
    freqs_g = torch.from_numpy(rope_freqs(M, seed=2)).to(dev)
    for i in range(DEPTH):
        rng = np.random.default_rng(base.integers(1 << 62))
        t = {}
        for name, n, k, qtype in (("qkv", 3 * E, E, 12), ("proj", E, E, 12), ("fc1", MLP, E, 12), ("fc2", E, MLP, 8)):
            w = rng.standard_normal((n, k), dtype=np.float32) * np.float32(0.02)
            w[rng.random((n, k), dtype=np.float32) < 0.01] *= 8
            t[name] = samq.Weights(qtype, k, n, samq.quantize_rows(qtype, w), device=device)
            t[name + "_b"] = torch.from_numpy(rng.normal(0, 0.02, n).astype(np.float32)).to(dev)
        for name in ("norm1", "norm2"):
            t[name + "_w"] = torch.from_numpy((1 + rng.normal(0, 0.02, E)).astype(np.float32)).to(dev)
            t[name + "_b"] = torch.from_numpy(rng.normal(0, 0.02, E).astype(np.float32)).to(dev)
        window = 0 if i in GLOBAL_BLOCKS else WINDOW
        blocks.append(samq.VitBlock(window, t["norm1_w"], t["norm1_b"], t["qkv"], t["qkv_b"], t["proj"],
                                    t["proj_b"], t["norm2_w"], t["norm2_b"], t["fc1"], t["fc1_b"], t["fc2"],
                                    t["fc2_b"], freqs_g if window == 0 else freqs_w, compute=compute))
        keep.append(t)
    rng = np.random.default_rng(77 + rank)
    prefix = {
        "patch_w": torch.from_numpy(rng.normal(0, 0.02, (E, 3, PATCH, PATCH)).astype(np.float32)).to(dev),
        "pos": torch.from_numpy(rng.normal(0, 0.02, (POS_GRID, POS_GRID, E)).astype(np.float32)).to(dev),
        "ln_w": torch.from_numpy((1 + rng.normal(0, 0.02, E)).astype(np.float32)).to(dev),
        "ln_b": torch.from_numpy(rng.normal(0, 0.02, E).astype(np.float32)).to(dev),
    }
    return blocks, prefix, keep


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=200)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", default="samq", choices=["samq", "reference"])
    ap.add_argument("--e2e-steps", type=int, default=20)
    ap.add_argument("--qgemm-steps", type=int, default=500)
    ap.add_argument("--cpu-budget", type=float, default=12.0, help="seconds of CPU baseline work")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--profile", choices=[l[0] for l in LINEARS] + list(PROFILE_EXTRA),
                    help="one kernel's case launched --warmup + --steps times, for ncu captures: a block "
                         "linear's GEMM (A operand staged once), attention_window / attention_global "
                         "(samq_vit_attention_v1 at 72x72, 16 heads), or text_fc2 (small-M Q8_0 "
                         "4096 -> 1024 at M = 32, the packet-streaming kernel)")
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

    torch.cuda.set_device(local)
    if world > 1:
        from datetime import timedelta
        dist.init_process_group("nccl", timeout=timedelta(seconds=120), device_id=torch.device("cuda", local))
    samq.init(local)
    stream = torch.cuda.current_stream()

    from samq.shard import max_over_ranks as shard_max

    def max_over_ranks(ms):
        return shard_max(ms, dist if world > 1 else None, torch.device("cuda", local))

    # ---- backbone (config 3): one image per step per GPU ------------------
    blocks, prefix, keep = make_backbone(samq, torch, local, rank)
    rng = np.random.default_rng(500 + rank)
    image_host = torch.from_numpy(((rng.random((3, IMAGE, IMAGE), dtype=np.float32) - 0.5) / 0.5)).pin_memory()
    image = image_host.cuda()
    feats = torch.empty((M, E), dtype=torch.float32, device="cuda")
    feats_host = torch.empty((M, E), dtype=torch.float32).pin_memory()

    def forward(img=image, out=feats, blks=blocks, compute=samq.COMPUTE_F16):
        samq.vit_prefix(img, IMAGE, IMAGE, PATCH, prefix["patch_w"], E, prefix["pos"], POS_GRID, prefix["ln_w"],
                        prefix["ln_b"], out, stream, compute=compute)
        for blk in blks:
            samq.vit_block_forward(blk, out, GRID, GRID, stream)

    for _ in range(args.warmup):
        forward()
    torch.cuda.synchronize()
    samq.check(local, stream)

    sampler = ClockSampler(int(os.environ.get("CUDA_VISIBLE_DEVICES", str(local)).split(",")[0])
                           if os.environ.get("CUDA_VISIBLE_DEVICES", "").split(",")[0].isdigit() else local)
    sampler.start()
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    start.record(stream)
    for _ in range(args.steps):
        forward()
    end.record(stream)
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    clocks = sampler.stop()
    samq.check(local, stream)
    elapsed_ms = max_over_ranks(start.elapsed_time(end))
    value = args.steps * world / (elapsed_ms / 1e3)
    feats_ok = bool(torch.isfinite(feats).all().item())

    # End to end through the C ABI with host buffers: every step copies its
    # image in from pinned host memory and its features out to pinned host
    # memory.  The copies run on a second stream against double-buffered
    # device buffers, so step s's upload and step s-1's download overlap the
    # backbone of step s-1 / s (the way a serving loop would issue them).
    e2e_steps = max(3, args.e2e_steps)
    copy_stream = torch.cuda.Stream()
    images = [torch.empty_like(image) for _ in range(2)]
    outs = [torch.empty_like(feats) for _ in range(2)]
    host_outs = [feats_host, torch.empty_like(feats_host).pin_memory()]
    ev = {name: [torch.cuda.Event() for _ in range(2)] for name in ("uploaded", "computed", "downloaded")}

    def e2e_run(steps):
        for s in range(steps):
            b = s % 2
            with torch.cuda.stream(copy_stream):
                if s >= 2:
                    copy_stream.wait_event(ev["computed"][b])  # images[b] read by step s-2's prefix
                images[b].copy_(image_host, non_blocking=True)
                ev["uploaded"][b].record(copy_stream)
            stream.wait_event(ev["uploaded"][b])
            if s >= 2:
                stream.wait_event(ev["downloaded"][b])  # outs[b] read back by step s-2's download
            forward(images[b], outs[b])
            ev["computed"][b].record(stream)
            with torch.cuda.stream(copy_stream):
                copy_stream.wait_event(ev["computed"][b])
                host_outs[b].copy_(outs[b], non_blocking=True)
                ev["downloaded"][b].record(copy_stream)

    e2e_run(3)
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(copy_stream)
    stream.wait_event(e0)
    e2e_run(e2e_steps)
    copy_stream.wait_stream(stream)
    e1.record(copy_stream)
    torch.cuda.synchronize()
    e2e_ms = max_over_ranks(e0.elapsed_time(e1))
    e2e_value = e2e_steps * world / (e2e_ms / 1e3)
    samq.check(local, stream)
    lin_ops, attn_ops = backbone_ops()

    # ---- q-GEMM (config 2): the four block linears from f32 ----------------
    weights, biases, xs, ys = [], [], [], []
    for name, n, k, qtype, epi, seed in LINEARS:
        packed, bias = make_weights(samq.quantize_rows, n, k, qtype, seed + 4 * rank)
        weights.append(samq.Weights(qtype, k, n, packed, device=local))
        biases.append(torch.from_numpy(bias).cuda())
        xs.append(torch.from_numpy(np.random.default_rng(1000 + seed + 17 * rank).normal(0, 1, (M, k))
                                   .astype(np.float32)).cuda())
        ys.append(torch.empty((M, n), dtype=torch.float32, device="cuda"))

    def qgemm_step():
        for i, (name, n, k, qtype, epi, _) in enumerate(LINEARS):
            samq.linear(weights[i], xs[i], M, k, biases[i], epi, ys[i], n, stream)

    for _ in range(args.warmup):
        qgemm_step()
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    q0, q1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    q0.record(stream)
    for _ in range(args.qgemm_steps):
        qgemm_step()
    q1.record(stream)
    torch.cuda.synchronize()
    qgemm_ms = max_over_ranks(q0.elapsed_time(q1))
    qgemm_tops = step_ops() * args.qgemm_steps * world / (qgemm_ms / 1e3) / 1e12
    samq.check(local, stream)

    # GEMM-only launch durations (the dominant kernel) on the same stream:
    # back to back over rotating operand sets larger than twice the L2 (every
    # launch reads its A and B from HBM), against the burst peak; the older
    # flush-then-time-one-launch figure beside it.
    gemm_cold = gemm_cold_durations(samq, torch, stream, rank)
    gemm_ms = [max_over_ranks(g) for g, _ in gemm_cold]
    gemm_host_ms = [max_over_ranks(h) for _, h in gemm_cold]
    gemm_isolated_ms = gemm_only_durations(samq, weights, xs, ys, biases, stream)
    pk = peaks()
    gemm_flops = [2.0 * M * n * k for _, n, k, *_ in LINEARS]
    achieved = sum(gemm_flops) / (sum(gemm_ms) / 1e3) / 1e12
    traffic = profiled_traffic()
    roofline = {"bound": "tensor", "kernel": "K2: gemm_f16_pair_kernel (cta_group::2, qkv / fc1) and gemm_f16_kernel "
                          "(proj / fc2); tcgen05 kind::f16, f32 accumulate",
                "achieved": achieved, "peak": pk["bf16_tflops"], "unit": "TFLOP/s",
                "frac": achieved / pk["bf16_tflops"], "peak_source": f"{pk['source']} bf16 (of measured)",
                "frac_of_sustained": achieved / pk["bf16_tflops_sustained"],
                "traffic": traffic.get("bytes_per_launch") if traffic else None,
                "traffic_source": traffic.get("source") if traffic else None,
                "per_linear": {LINEARS[i][0]: {"us": gemm_ms[i] * 1e3,
                                               "tflops": gemm_flops[i] / (gemm_ms[i] / 1e3) / 1e12,
                                               "frac": gemm_flops[i] / (gemm_ms[i] / 1e3) / 1e12 / pk["bf16_tflops"]}
                               for i in range(len(LINEARS))},
                "measured_on": "the 4 block-linear shapes at M=5184 (f32 epilogue, fused bias / GELU): per shape "
                               "enough distinct (weights, activations) sets that their operands exceed 2 x L2 "
                               "(256 MB), launched back to back in rotation (120+ launches, captured once as a "
                               "CUDA graph and replayed 3 times between two CUDA events on the replay stream), "
                               "so every launch reads A and B from HBM and none waits on the host; "
                               "achieved = sum 2MNK / sum of the average launch times",
                "host_issued": {LINEARS[i][0]: {"us": gemm_host_ms[i] * 1e3,
                                                "frac": gemm_flops[i] / (gemm_host_ms[i] / 1e3) / 1e12
                                                / pk["bf16_tflops"]} for i in range(len(LINEARS))},
                "isolated_launch": {LINEARS[i][0]: {"us": gemm_isolated_ms[i] * 1e3,
                                                    "frac": gemm_flops[i] / (gemm_isolated_ms[i] / 1e3) / 1e12
                                                    / pk["bf16_tflops"]} for i in range(len(LINEARS))},
                "isolated_method": "each launch alone between two CUDA events after a 256 MB L2-flushing read "
                                   "(includes the launch gap a lone kernel pays)"}

    # The exact-MMQ-arithmetic GEMM (gemm_mmq.cu) beside K2 on the same four
    # shapes with Q8_0 weights: integer codes on kind::f16 and on kind::i8.
    mmq = mmq_section(samq, torch, stream, max_over_ranks, xs, ys, biases, rank, args.warmup, world, pk)
    samq.check(local, stream)

    # The SimpleFPN neck (F32 semantics, dense.cu) on this image's 72 x 72 ViT
    # output: a secondary figure beside the quantized backbone.
    neck = neck_section(samq, torch, stream, args, max_over_ranks, pk)
    samq.check(local, stream)
    # Config 5's batching: the same backbone over 8 images per GPU per step.
    batch8 = batch_section(samq, torch, stream, args, max_over_ranks, blocks, prefix, world, rank)
    samq.check(local, stream)
    # The reference's default compute mode (F32 attention and patch columns)
    # on the same weights: a secondary figure beside the F16-mode headline.
    f32_blocks = [samq.VitBlock(b.window, *b._keep, compute=samq.COMPUTE_F32) for b in blocks]
    f32_mode = f32_section(samq, torch, stream, max_over_ranks, forward, f32_blocks, image, feats, world)
    samq.check(local, stream)
    # Config 5's sharding protocol: 64 images cut into contiguous per-rank ranges.
    sweep = sweep64_section(samq, torch, stream, max_over_ranks, blocks, prefix, world, rank,
                            dist if world > 1 else None)
    samq.check(local, stream)

    # Configs 4 and 5 through the whole image path (samq.sam3.Sam3Image).
    image_path = image_path_section(samq, torch, stream, max_over_ranks, world, rank, local,
                                    dist if world > 1 else None)
    samq.check(local, stream)

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        from oracle import oracle as o
        cb = CpuBackbone(o)
        cb.step()
        samples, t0 = [], time.perf_counter()
        while not samples or (time.perf_counter() - t0 < args.cpu_budget and len(samples) < 200):
            samples.append(cb.step())
        cpu = {"value": 1.0 / float(np.mean(samples)), "unit": "images/s", "cores": cb.threads, "kind": "port",
               "sample": f"{len(samples)} samples; " + cb.describe()}

    if rank == 0:
        line = {
            "metric": METRIC, "value": value, "unit": "images/s", "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": elapsed_ms / args.steps, "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": "f16", "data": "synthetic",
            "compute_mode": "F16: the reference's opt-in CudaComputeMode::F16 (f16 tensor-core attention operands, "
                            "f16 patch columns); quantized linears (Q8_1 staging, f16 operands on tcgen05) are the "
                            "same in both modes; the default F32 mode is timed in `f32_mode`",
            "config": workload_config(world),
            "roofline": roofline,
            "cpu_baseline": cpu,
            "e2e": {"value": e2e_value, "unit": "images/s", "h2d_bytes_per_step": image_host.numel() * 4,
                    "d2h_bytes_per_step": feats_host.numel() * 4, "steps": e2e_steps,
                    "copies": "pinned host buffers, second stream, double-buffered device buffers"},
            "gpu_launches": args.steps * (4 + DEPTH * 7),
            "clocks": clocks,
            "achieved_tflops": (lin_ops + attn_ops) * value / world / 1e12,
            "features_finite": feats_ok,
            "qgemm": {"metric": QGEMM_METRIC, "workload": QGEMM_WORKLOAD, "value": qgemm_tops, "unit": "TOPS",
                      "steps": args.qgemm_steps, "ms_per_step": qgemm_ms / args.qgemm_steps,
                      "gpu_launches": args.qgemm_steps * 2 * len(LINEARS)},
            "neck": neck,
            "batch8": batch8,
            "sweep64": sweep,
            "f32_mode": f32_mode,
            "image_path": image_path,
            "mmq": mmq,
        }
        print(json.dumps(line), flush=True)
    for w in weights:
        w.close()
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()


def batch_section(samq, torch, stream, args, max_over_ranks, blocks, prefix, world, rank, batch=8, steps=4):
    """BASELINE config 5's per-GPU batches: 8 seeded images per step, each
    through samq_vit_prefix_v1, then every block once for the whole batch
    (samq_vit_block_forward_batch_v1)."""
    rng = np.random.default_rng(900 + rank)
    imgs = torch.from_numpy(((rng.random((batch, 3, IMAGE, IMAGE), dtype=np.float32) - 0.5) / 0.5)).cuda()
    xb = torch.empty((batch, M, E), dtype=torch.float32, device="cuda")

    def fwd():
        for b in range(batch):
            samq.vit_prefix(imgs[b], IMAGE, IMAGE, PATCH, prefix["patch_w"], E, prefix["pos"], POS_GRID,
                            prefix["ln_w"], prefix["ln_b"], xb[b], stream, compute=samq.COMPUTE_F16)
        for blk in blocks:
            samq.vit_block_forward(blk, xb, GRID, GRID, stream, batch=batch)

    for _ in range(2):
        fwd()
    torch.cuda.synchronize()
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    a.record(stream)
    for _ in range(steps):
        fwd()
    b.record(stream)
    torch.cuda.synchronize()
    ms = max_over_ranks(a.elapsed_time(b))
    return {"metric": "SAM3 vision backbone images/s, per-GPU batch of 8 (config 5's batching)",
            "value": steps * batch * world / (ms / 1e3), "unit": "images/s", "batch_per_gpu": batch, "steps": steps,
            "ms_per_step": ms / steps, "features_finite": bool(torch.isfinite(xb).all().item()),
            "gpu_launches": steps * batch * 4 + steps * DEPTH * 7}


def f32_section(samq, torch, stream, max_over_ranks, forward, f32_blocks, image, feats, world, steps=10):
    """Images/s of the same backbone in the reference's default compute mode
    (SAMQ_COMPUTE_F32: F32 patch columns, f32 qkv and F32-precise attention)."""
    for _ in range(3):
        forward(image, feats, f32_blocks, samq.COMPUTE_F32)
    torch.cuda.synchronize()
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    a.record(stream)
    for _ in range(steps):
        forward(image, feats, f32_blocks, samq.COMPUTE_F32)
    b.record(stream)
    torch.cuda.synchronize()
    ms = max_over_ranks(a.elapsed_time(b))
    return {"metric": "SAM3 vision backbone images/s, compute mode F32 (the reference's default: F32 attention and "
                      "patch columns)", "value": steps * world / (ms / 1e3), "unit": "images/s", "steps": steps,
            "ms_per_step": ms / steps, "features_finite": bool(torch.isfinite(feats).all().item())}


def sweep64_section(samq, torch, stream, max_over_ranks, blocks, prefix, world, rank, dist, n_images=64, batch=8):
    """BASELINE config 5's sharding protocol on the vision backbone: 64
    distinct seeded images, rank g taking the contiguous range
    [g * 64 / G, (g + 1) * 64 / G) in per-GPU batches of 8 (prefix per image,
    then each block once per batch).  The time is the max over ranks of each
    rank's device time (CUDA events), after a barrier; images/s = 64 / time.
    The weights are the backbone's replica on every rank; no data crosses GPUs."""
    from samq.shard import batches, image_range
    start, end = image_range(n_images, world, rank)
    own = batches(start, end, batch)
    imgs = torch.empty((end - start, 3, IMAGE, IMAGE), dtype=torch.float32, device="cuda")
    for i in range(start, end):
        rng = np.random.default_rng(10_000 + i)  # image i has the same pixels whatever G is
        imgs[i - start].copy_(torch.from_numpy(((rng.random((3, IMAGE, IMAGE), dtype=np.float32) - 0.5) / 0.5)))
    xb = torch.empty((batch, M, E), dtype=torch.float32, device="cuda")

    def run():
        for b0, b1 in own:
            for j in range(b1 - b0):
                samq.vit_prefix(imgs[b0 - start + j], IMAGE, IMAGE, PATCH, prefix["patch_w"], E, prefix["pos"],
                                POS_GRID, prefix["ln_w"], prefix["ln_b"], xb[j], stream, compute=samq.COMPUTE_F16)
            for blk in blocks:
                samq.vit_block_forward(blk, xb, GRID, GRID, stream, batch=b1 - b0)

    run()  # warm-up
    torch.cuda.synchronize()
    if dist is not None:
        dist.barrier()
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    a.record(stream)
    run()
    b.record(stream)
    torch.cuda.synchronize()
    ms = max_over_ranks(a.elapsed_time(b))
    return {"metric": "SAM3 vision backbone images/s, 64 images sharded contiguously, per-GPU batches of 8 "
                      "(config 5 protocol)", "value": n_images / (ms / 1e3), "unit": "images/s",
            "scaling": "strong", "images": n_images, "images_this_rank": end - start, "batch_per_gpu": batch,
            "ms": ms, "features_finite": bool(torch.isfinite(xb).all().item()),
            "gpu_launches": (end - start) * 4 + len(own) * DEPTH * 7}


def mmq_section(samq, torch, stream, max_over_ranks, xs, ys, biases, rank, warmup, world, pk, reps=100):
    """samq_linear_mmq_v1 (GGML MMQ's exact arithmetic: MMQ-D4 staging + the
    per-block-rescaled integer GEMM) on the four ViT-block shapes at M = 5184
    with Q8_0 weights, both code variants, each call timed back to back (D4
    staging included, as `qgemm` includes K1).  The int8 variant is quoted
    against the nominal dense int8 peak (4.5 POPS; no measured int8 figure
    exists for this pool), both against the measured bf16 burst."""
    out = {}
    for variant, name in ((samq.MMQ_CODES_F16, "codes_f16_kind_f16"), (samq.MMQ_CODES_I8, "codes_i8_kind_i8")):
        per, total_ms = {}, 0.0
        for i, (lname, n, k, qtype, epi, seed) in enumerate(LINEARS):
            packed, _ = make_weights(samq.quantize_rows, n, k, 8, seed + 4 * rank)
            w = samq.MmqWeights(8, k, n, packed, variant=variant, device=torch.cuda.current_device())
            for _ in range(warmup):
                samq.linear_mmq(w, xs[i], M, k, biases[i], epi, ys[i], n, stream)
            torch.cuda.synchronize()
            a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            a.record(stream)
            for _ in range(reps):
                samq.linear_mmq(w, xs[i], M, k, biases[i], epi, ys[i], n, stream)
            b.record(stream)
            torch.cuda.synchronize()
            ms = max_over_ranks(a.elapsed_time(b) / reps)
            total_ms += ms
            tops = 2.0 * M * n * k / (ms / 1e3) / 1e12
            per[lname] = {"us": ms * 1e3, "tops": tops, "frac_bf16_burst": tops / pk["bf16_tflops"]}
            if variant == samq.MMQ_CODES_I8:
                per[lname]["frac_int8_nominal"] = tops / 4500.0
            w.close()
        ops = step_ops()
        out[name] = {"tops_four_linears": ops / (total_ms / 1e3) / 1e12 * world, "ms_four_linears": total_ms,
                     "per_linear": per}
    out["what"] = ("exact GGML MMQ arithmetic: integer codes on the tensor cores, one TMEM slot per 32-value block, "
                   "f32 per-block rescale in the epilogue (2 f32 operations per output per block); compare "
                   "`qgemm` (K2, f16 decoded operands, same shapes, K1 included)")
    return out


def image_path_section(samq, torch, stream, max_over_ranks, world, rank, local, dist, steps=4):
    """The whole SAM 3 image path through samq.sam3.Sam3Image, random-init
    models written by samq.synthetic, both in the headline F16 compute mode:

    config4: the full-linear Q8_0 model, one 1008 x 1008 image and its 32-token
      prompt per step: encode_image (ViT, neck, geometry token), encode_text,
      predict (fusion, decoder + scoring, segmentation head with 200 x 288 x
      288 mask logits); per-stage device times from CUDA events.
    config5: the mixed model (vision Q4_K, text Q8_0, fusion / decoder F32),
      64 distinct images sharded contiguously over the ranks, per-GPU batches
      of 8 (the 32 blocks batched, neck / geometry / predict per image), one
      fixed prompt encoded once; images/s = 64 / (max over ranks of the
      device time)."""
    from samq import synthetic
    from samq.sam3 import Sam3Image
    from samq.shard import batches, image_range
    hp = synthetic.Hparams()
    out = {}
    t0 = time.perf_counter()
    model = Sam3Image(synthetic.sam3_tensors(hp, "q8_0", seed=40 + rank), hp, compute=samq.COMPUTE_F16,
                      device=local)
    build_s = time.perf_counter() - t0
    pixels = torch.from_numpy(synthetic.image(hp, 400 + rank)).to("cuda")
    ids = synthetic.token_ids(hp, 401)
    ev = [torch.cuda.Event(enable_timing=True) for _ in range(4)]
    stage_ms = np.zeros(3)
    for step in range(2 + steps):
        ev[0].record(stream)
        feats = model.encode_image(pixels, stream)
        ev[1].record(stream)
        text = model.encode_text(ids, stream)
        ev[2].record(stream)
        pred = model.predict(feats, ids, text, stream)
        ev[3].record(stream)
        torch.cuda.synchronize()
        if step >= 2:
            stage_ms += [ev[i].elapsed_time(ev[i + 1]) for i in range(3)]
    stage_ms /= steps
    total = max_over_ranks(float(stage_ms.sum()))
    # The same image path replayed as one CUDA graph per prompt (ImagePathGraph):
    # the text features are computed once per prompt, the graph runs
    # encode_image + predict.
    from samq.sam3 import ImagePathGraph
    graph = ImagePathGraph(model, ids, text)
    graph.pixels.copy_(pixels)
    for _ in range(2):
        graph.replay()
    torch.cuda.synchronize()
    g0, g1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    g0.record(stream)
    for _ in range(steps):
        graph.replay()
    g1.record(stream)
    torch.cuda.synchronize()
    graph_ms = max_over_ranks(g0.elapsed_time(g1) / steps)
    graph_finite = bool(torch.isfinite(graph.prediction.mask_logits).all().item())
    out["config4"] = {"metric": "SAM3 full-component Q8_0 text-prompted segmentation images/s (1008x1008, "
                                "batch 1, text encoded per image)", "value": 1e3 / total * world,
                      "unit": "images/s", "ms_per_image": total, "steps": steps,
                      "stage_ms": {"encode_image": stage_ms[0], "encode_text": stage_ms[1],
                                   "predict": stage_ms[2]},
                      "graph": {"ms_per_image": graph_ms, "images_per_s": 1e3 / graph_ms * world,
                                "with_text_per_image_ms": graph_ms + stage_ms[1], "outputs_finite": graph_finite,
                                "what": "encode_image + predict captured once as a CUDA graph (ImagePathGraph), "
                                        "replayed per image; the prompt's text features computed once"},
                      "mask_logits": list(pred.mask_logits.shape),
                      "outputs_finite": bool(torch.isfinite(pred.mask_logits).all().item()
                                             and torch.isfinite(pred.boxes).all().item()),
                      "model_build_s": build_s}
    model.close()
    del model, feats, text, pred, graph
    torch.cuda.empty_cache()

    t0 = time.perf_counter()
    model = Sam3Image(synthetic.sam3_tensors(hp, "mixed", seed=50), hp, compute=samq.COMPUTE_F16, device=local)
    build_s = time.perf_counter() - t0
    ids = synthetic.token_ids(hp, 501)
    text = model.encode_text(ids, stream)
    n_images, batch = 64, 8
    start, end = image_range(n_images, world, rank)
    own = batches(start, end, batch)
    imgs = torch.empty((end - start, 3, hp.img_size, hp.img_size), device="cuda")
    for i in range(start, end):
        imgs[i - start].copy_(torch.from_numpy(synthetic.image(hp, 10_000 + i)))
    finite = [True]

    def run():
        for b0, b1 in own:
            for f in model.encode_images(imgs[b0 - start:b1 - start], stream):
                pred = model.predict(f, ids, text, stream)
            finite[0] = finite[0] and bool(torch.isfinite(pred.mask_logits[:, :64]).all().item())

    run()
    torch.cuda.synchronize()
    if dist is not None:
        dist.barrier()
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    a.record(stream)
    run()
    b.record(stream)
    torch.cuda.synchronize()
    ms = max_over_ranks(a.elapsed_time(b))
    out["config5"] = {"metric": "SAM3 mixed-allocation image path images/s (vision Q4_K, text Q8_0, fusion / "
                                "decoder F32), 64 images sharded contiguously, per-GPU batches of 8",
                      "value": n_images / (ms / 1e3), "unit": "images/s", "scaling": "strong", "ms": ms,
                      "images": n_images, "images_this_rank": end - start, "batch_per_gpu": batch,
                      "prompt": "one fixed 32-token prompt, encoded once outside the timed region",
                      "outputs_finite": finite[0], "model_build_s": build_s}
    model.close()
    del model, imgs
    torch.cuda.empty_cache()
    return out


NECK_MID, NECK_D = 512, 256


def neck_flops(gw=GRID, gh=GRID):
    """2 M N K of the neck's 11 dense products (vision.hpp:307-366)."""
    t = gw * gh
    e, mid, d = E, NECK_MID, NECK_D
    macs = (t * e * 4 * mid + 4 * t * mid * 4 * d + 16 * t * d * d + 16 * t * 9 * d * d  # scale 0
            + t * e * 4 * mid + 4 * t * mid * d + 4 * t * 9 * d * d                      # scale 1
            + t * e * d + t * 9 * d * d                                                  # scale 2
            + (gw // 2) * (gh // 2) * (e * d + 9 * d * d))                               # scale 3
    return 2.0 * macs


def make_neck(samq, torch, device, seed=0):
    """Random-init neck weights (fan-in scaled normal), SAM 3 shapes, on `device`."""
    rng = np.random.default_rng(seed)
    e, mid, d = E, NECK_MID, NECK_D
    shapes = {"s0_deconv1": (samq.DENSE_DECONV2X2, (e, mid, 2, 2)), "s0_deconv2": (samq.DENSE_DECONV2X2, (mid, d, 2, 2)),
              "s0_conv1x1": (samq.DENSE_CONV, (d, d, 1, 1)), "s0_conv3x3": (samq.DENSE_CONV, (d, d, 3, 3)),
              "s1_deconv1": (samq.DENSE_DECONV2X2, (e, mid, 2, 2)), "s1_conv1x1": (samq.DENSE_CONV, (d, mid, 1, 1)),
              "s1_conv3x3": (samq.DENSE_CONV, (d, d, 3, 3)), "s2_conv1x1": (samq.DENSE_CONV, (d, e, 1, 1)),
              "s2_conv3x3": (samq.DENSE_CONV, (d, d, 3, 3)), "s3_conv1x1": (samq.DENSE_CONV, (d, e, 1, 1)),
              "s3_conv3x3": (samq.DENSE_CONV, (d, d, 3, 3))}
    layers = {}
    for name, (kind, shape) in shapes.items():
        fan_in = shape[0] if kind == samq.DENSE_DECONV2X2 else shape[1] * shape[2] * shape[3]
        w = (rng.normal(size=shape) / np.sqrt(fan_in)).astype(np.float32)
        b = rng.normal(0, 0.02, shape[1] if kind == samq.DENSE_DECONV2X2 else shape[0]).astype(np.float32)
        layers[name] = (samq.Dense(kind, w, device=device), torch.from_numpy(b).cuda())
    return samq.Neck(layers)


def neck_section(samq, torch, stream, args, max_over_ranks, pk, steps=10):
    neck = make_neck(samq, torch, torch.cuda.current_device())
    x = torch.from_numpy(np.random.default_rng(7).normal(0, 1, (M, E)).astype(np.float32)).cuda()
    sizes = [4 * GRID, 2 * GRID, GRID, GRID // 2]
    outs = [torch.empty(s * s * NECK_D, device="cuda") for s in sizes]
    for _ in range(max(args.warmup, 3)):
        samq.neck_forward(neck, x, GRID, GRID, outs, stream)
    torch.cuda.synchronize()
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    a.record(stream)
    for _ in range(steps):
        samq.neck_forward(neck, x, GRID, GRID, outs, stream)
    b.record(stream)
    torch.cuda.synchronize()
    ms = max_over_ranks(a.elapsed_time(b)) / steps
    f32 = neck_flops() / (ms / 1e3) / 1e12
    # Three TF32 MMAs per F32 product; the TF32 dense rate is taken as half
    # the measured bf16 rate (the tensor cores' nominal TF32 : BF16 ratio).
    tf32_peak = pk["bf16_tflops"] / 2
    return {"metric": "SAM3 SimpleFPN neck, F32 semantics (ms per image, 72x72 grid)", "value": ms, "unit": "ms",
            "higher_is_better": False, "steps": steps, "gflop_f32": neck_flops() / 1e9, "tflops_f32_equivalent": f32,
            "tf32_mma_tflops": 3 * f32, "tf32_peak_estimate": tf32_peak, "frac_of_tf32_estimate": 3 * f32 / tf32_peak,
            "gpu_launches_per_call": 17, "method": "three-term TF32 split on tcgen05 kind::tf32, segment sums in f32"}


PROFILE_EXTRA = ("attention_window", "attention_global", "attention_window_f32", "attention_global_f32", "text_fc2",
                 "neck_conv3x3", "vit_block", "mmq_qkv", "fusion_self_attention")


def run_profile_case(args):
    """One kernel's case launched alone, for ncu (-k regex:<kernel>)."""
    import torch
    import samq
    from samq.synthetic import rope_freqs
    torch.cuda.set_device(0)
    samq.init(0)
    stream = torch.cuda.current_stream()
    launches = args.warmup + args.steps
    if args.profile == "vit_block":
        # One windowed ViT block (block 0 of the backbone) on a 72 x 72 grid,
        # every launch of it: the LayerNorm-staging, GEMM and attention
        # kernels in their in-block modes.
        blocks, _, keep = make_backbone(samq, torch, 0, 0)
        x = torch.from_numpy(np.random.default_rng(3).normal(0, 1, (M, E)).astype(np.float32)).cuda()
        for _ in range(launches):
            samq.vit_block_forward(blocks[0], x, GRID, GRID, stream)
        torch.cuda.synchronize()
        del keep
    elif args.profile == "neck_conv3x3":
        # The neck's largest product: conv3x3 256 -> 256 at 288 x 288
        # (scale 0), operand 2 x 85 MB (inputs larger than L2).
        rng = np.random.default_rng(3)
        w = samq.Dense(samq.DENSE_CONV, (rng.normal(size=(256, 256, 3, 3)) / 48).astype(np.float32))
        x = torch.from_numpy(rng.normal(size=(288 * 288 * 256,)).astype(np.float32)).cuda()
        y = torch.empty_like(x)
        for _ in range(launches):
            samq.conv2d(w, x, 288, 288, None, 0, y, stream)
        torch.cuda.synchronize()
        w.close()
    elif args.profile.startswith("attention"):
        window = WINDOW if args.profile.startswith("attention_window") else 0
        rng = np.random.default_rng(3)
        qkv = torch.from_numpy(rng.normal(0, 1, (M, 3 * E)).astype(np.float32)).cuda()
        freqs = torch.from_numpy(rope_freqs(WINDOW * WINDOW if window else M)).cuda()
        out = torch.empty((M, E), dtype=torch.float32, device="cuda")
        for _ in range(launches):
            samq.vit_attention(qkv, 3 * E, GRID, GRID, HEADS, window, freqs, out, E, stream,
                               compute=samq.COMPUTE_F32 if args.profile.endswith("_f32") else samq.COMPUTE_F16)
    elif args.profile == "fusion_self_attention":
        # The fusion encoder's self-attention: 5184 x 5184 tokens, 8 heads of
        # 32, no mask (samq_attention_v1 -> the tensor-core F32 kernel).
        T, H, hd = M, 8, 32
        D = H * hd
        rng = np.random.default_rng(3)
        qkv = torch.from_numpy(rng.normal(0, 1, (T, 3 * D)).astype(np.float32)).cuda()
        out = torch.empty((T, D), dtype=torch.float32, device="cuda")
        for _ in range(launches):
            samq.attention(qkv, 3 * D, qkv[:, D:], 3 * D, qkv[:, 2 * D:], 3 * D, T, T, H, hd, float(1 / np.sqrt(hd)),
                           out, D, stream=stream)
        torch.cuda.synchronize()
    elif args.profile == "mmq_qkv":
        # The exact-MMQ-arithmetic GEMM (samq_linear_mmq_v1, f16 codes) at the
        # qkv shape: D4 staging + gemm_mmq_kernel per launch.
        n, k = 3 * E, E
        packed, bias = make_weights(samq.quantize_rows, n, k, 8, 0)
        w = samq.MmqWeights(8, k, n, packed)
        x = torch.from_numpy(np.random.default_rng(0).normal(0, 1, (M, k)).astype(np.float32)).cuda()
        y = torch.empty((M, n), dtype=torch.float32, device="cuda")
        b = torch.from_numpy(bias).cuda()
        for _ in range(launches):
            samq.linear_mmq(w, x, M, k, b, 0, y, n, stream)
        torch.cuda.synchronize()
        w.close()
    elif args.profile == "text_fc2":
        n, k, m = 1024, 4096, 32
        packed, bias = make_weights(samq.quantize_rows, n, k, 8, 5)
        w = samq.Weights(8, k, n, packed)
        x = torch.from_numpy(np.random.default_rng(5).normal(0, 1, (m, k)).astype(np.float32)).cuda()
        a16 = torch.empty((m, k), dtype=torch.float16, device="cuda")
        y = torch.empty((m, n), dtype=torch.float32, device="cuda")
        b = torch.from_numpy(bias).cuda()
        samq.stage_f16(x, m, k, k, a16, stream)
        for _ in range(launches):
            samq.linear_f16(w, a16, m, k, b, 0, y, n, stream)
        torch.cuda.synchronize()
        w.close()
    if args.profile in PROFILE_EXTRA:
        torch.cuda.synchronize()
        samq.check(0, stream)
        print(json.dumps({"profile_case": args.profile, "launches": launches}))
        return
    name, n, k, qtype, epi, seed = next(l for l in LINEARS if l[0] == args.profile)
    packed, bias = make_weights(samq.quantize_rows, n, k, qtype, seed)
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


def gemm_cold_durations(samq, torch, stream, rank, reps=8, replays=3, l2_bytes=256 << 20):
    """Average device time of one K2 launch (samq_linear_f16_v1, A staged
    once per set) per ViT-block shape, launched back to back over rotating
    (weights, activations) sets whose A + B bytes exceed twice the L2, so that
    no launch finds its operands in L2.  Returns per shape (ms per launch
    replayed from a CUDA graph, ms per launch issued from the host loop)."""
    out = []
    for name, n, k, qtype, epi, seed in LINEARS:
        per_set = n * k * 2 + M * k * 2
        sets = max(2, min(24, -(-l2_bytes // per_set)))
        ws, As, bs = [], [], []
        for j in range(sets):
            packed, bias = make_weights(samq.quantize_rows, n, k, qtype, seed + 100 * j + 4 * rank)
            ws.append(samq.Weights(qtype, k, n, packed, device=torch.cuda.current_device()))
            x = torch.from_numpy(np.random.default_rng(2000 + j).normal(0, 1, (M, k)).astype(np.float32)).cuda()
            a16 = torch.empty((M, k), dtype=torch.float16, device="cuda")
            samq.stage_f16(x, M, k, k, a16, stream)
            As.append(a16)
            bs.append(torch.from_numpy(bias).cuda())
        y = torch.empty((M, n), dtype=torch.float32, device="cuda")
        cap = torch.cuda.Stream()
        cap.wait_stream(stream)
        for j in range(sets):
            samq.linear_f16(ws[j], As[j], M, k, bs[j], epi, y, n, cap)
        torch.cuda.synchronize()
        # One rotation captured as a CUDA graph: its replay issues the
        # launches from the device, so a kernel shorter than the host's
        # per-call cost (ctypes, tensor-map encodes, launch) is still timed
        # back to back rather than waiting on the host.
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph, stream=cap):
            for r in range(reps):
                for j in range(sets):
                    samq.linear_f16(ws[j], As[j], M, k, bs[j], epi, y, n, cap)
        with torch.cuda.stream(cap):
            graph.replay()
        torch.cuda.synchronize()
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        with torch.cuda.stream(cap):  # replay() launches on the current stream
            a.record(cap)
            for _ in range(replays):
                graph.replay()
            b.record(cap)
        torch.cuda.synchronize()
        graph_ms = a.elapsed_time(b) / (replays * reps * sets)
        a.record(stream)
        for r in range(reps):
            for j in range(sets):
                samq.linear_f16(ws[j], As[j], M, k, bs[j], epi, y, n, stream)
        b.record(stream)
        torch.cuda.synchronize()
        out.append((graph_ms, a.elapsed_time(b) / (reps * sets)))
        del graph
        for w in ws:
            w.close()
        del As, bs, y
    return out


def gemm_only_durations(samq, weights, xs, ys, biases, stream, reps=20):
    """Average device time of one GEMM launch per shape: the f16 A operand is
    staged once (samq_stage_f16_v1); then each of `reps` launches of
    samq_linear_f16_v1 (the tcgen05 GEMM kernel alone) is timed between two
    CUDA events on the launching stream, after a 256 MB read (twice the L2)
    so that it starts with its operands in HBM.  The flush reads rather than
    writes: a write leaves L2 full of dirty lines whose write-back to HBM
    would run during the timed launch and charge it for traffic that is not
    its own."""
    import torch
    flush = torch.ones(64 << 20, dtype=torch.float32, device="cuda")
    sink = torch.zeros((), dtype=torch.float32, device="cuda")
    out = []
    for i, (name, n, k, qtype, epi, _) in enumerate(LINEARS):
        m = xs[i].shape[0]
        a16 = torch.empty((m, k), dtype=torch.float16, device="cuda")
        samq.stage_f16(xs[i], m, k, k, a16, stream)
        for _ in range(3):
            samq.linear_f16(weights[i], a16, m, k, biases[i], epi, ys[i], n, stream)
        events = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(reps)]
        for a, b in events:
            torch.sum(flush, dim=0, out=sink)
            a.record(stream)
            samq.linear_f16(weights[i], a16, m, k, biases[i], epi, ys[i], n, stream)
            b.record(stream)
        torch.cuda.synchronize()
        out.append(sum(a.elapsed_time(b) for a, b in events) / reps)
    return out


if __name__ == "__main__":
    main()
