"""Whole-depth SAM 3 backbone parity: samq_vit_prefix_v1 + 32 x
samq_vit_block_forward_v1 (global attention at blocks 7, 15, 23 and 31,
windowed 24 x 24 elsewhere) against the CPU oracle run block by block on the
same random-init weights (src/models/sam3/vision.hpp:152-293).

The oracle computes every quantized linear with GGML MMQ's operand semantics
(Q8_1-staged activations times the f32-decoded weights, f64 dots), and the
LayerNorms, RoPE and attention in f64.  The device path differs by its f16
tensor-core operands (Q8_1 values and weights rounded once to f16, f16 Q / K /
V / P in attention) and f32 accumulation; these tests measure how that error
grows over the 32 blocks.

Bar on the backbone output (features of unit scale after ln_pre, growing
through the residual adds): mean absolute error <= 1e-2 (the bar the
end-to-end mask logits are held to, so no looser), cosine >= 0.9999, and on
the accumulated block contributions (out - prefix) cosine >= 0.9995.  The
per-depth cosine / max error is printed (pytest -s).
"""
import numpy as np
import pytest
import torch

import samq
from oracle import oracle as o
from test_gpu_vit import make_block

pytestmark = pytest.mark.gpu

E, MLP, PATCH, POS_GRID, DEPTH = 1024, 4736, 14, 24, 32
GLOBAL = (7, 15, 23, 31)
MEAN_ABS_MAX, COS_MIN, DELTA_COS_MIN = 1e-2, 0.9999, 0.9995


def _prefix_params(rng):
    return {"patch_w": rng.normal(0.0, 0.02, (E, 3, PATCH, PATCH)).astype(np.float32),
            "pos": rng.normal(0.0, 0.02, (POS_GRID, POS_GRID, E)).astype(np.float32),
            "ln_w": (1.0 + rng.normal(0.0, 0.02, E)).astype(np.float32),
            "ln_b": rng.normal(0.0, 0.02, E).astype(np.float32)}


def _stats(got, ref, base):
    g, r = got.astype(np.float64), ref.astype(np.float64)
    d = g - r
    cos = float((g.ravel() @ r.ravel()) / (np.linalg.norm(g) * np.linalg.norm(r)))
    dg, dr = (g - base).ravel(), (r - base).ravel()
    dcos = float(dg @ dr / (np.linalg.norm(dg) * np.linalg.norm(dr)))
    return {"cos": cos, "delta_cos": dcos, "mean_abs": float(np.abs(d).mean()), "max_abs": float(np.abs(d).max()),
            "max_rel": float(np.abs(d).max() / np.abs(r).max())}


def _run_backbone(grid, seed, sample_rows=None):
    """Builds 32 random-init blocks, runs the device backbone on one image and
    the oracle block by block (on the oracle's own previous output).  With
    sample_rows, the last block's oracle covers only those tokens."""
    rng = np.random.default_rng(seed)
    size = grid * PATCH
    image = ((rng.random((3, size, size)) - 0.5) / 0.5).astype(np.float32)
    pre = _prefix_params(rng)
    dev = torch.device("cuda")
    t = {k: torch.from_numpy(v).to(dev) for k, v in pre.items()}
    x = torch.empty((grid * grid, E), device=dev)
    samq.vit_prefix(torch.from_numpy(image).to(dev), size, size, PATCH, t["patch_w"], E, t["pos"], POS_GRID,
                    t["ln_w"], t["ln_b"], x)
    samq.check(0)
    ref = o.vit_prefix(image, PATCH, pre["patch_w"], pre["pos"], pre["ln_w"], pre["ln_b"])
    base = ref.copy()
    history = [("prefix", _stats(x.cpu().numpy(), ref, base))]
    for i in range(DEPTH):
        window = 0 if i in GLOBAL else 24
        host, block = make_block(rng, window, grid * grid if window == 0 else 576)
        samq.vit_block_forward(block, x, grid, grid)
        samq.check(0)
        last = i == DEPTH - 1
        rows = sample_rows if (last and sample_rows is not None) else None
        ref = o.vit_block(ref, host, grid, grid, rows=rows)
        got = x.cpu().numpy()
        if rows is not None:
            got, base = got[rows], base[rows]
        history.append((f"block {i:2d} ({'global' if window == 0 else 'window'})", _stats(got, ref, base)))
        for held in block._keep:
            if isinstance(held, samq.Weights):
                held.close()
    for name, s in history:
        print(f"{grid}x{grid} {name}: cos {s['cos']:.7f} delta_cos {s['delta_cos']:.7f} "
              f"mean_abs {s['mean_abs']:.3e} max_abs {s['max_abs']:.3e} max_rel {s['max_rel']:.3e}")
    return history[-1][1]


def test_backbone_32_blocks_48x48_all_rows():
    """A 672 x 672 image (48 x 48 tokens, 4 windows per windowed block), every
    token of the final features checked."""
    s = _run_backbone(48, seed=1234)
    assert s["mean_abs"] <= MEAN_ABS_MAX and s["cos"] >= COS_MIN and s["delta_cos"] >= DELTA_COS_MIN, s


def test_backbone_32_blocks_72x72_sampled_rows():
    """The full 1008 x 1008 image (72 x 72 tokens, 9 windows, 5184-token global
    attention): blocks 0..30 checked on all tokens, the last block on 256
    sampled tokens."""
    rng = np.random.default_rng(77)
    rows = np.sort(rng.choice(72 * 72, 256, replace=False))
    s = _run_backbone(72, seed=4321, sample_rows=rows)
    assert s["mean_abs"] <= MEAN_ABS_MAX and s["cos"] >= COS_MIN and s["delta_cos"] >= DELTA_COS_MIN, s
