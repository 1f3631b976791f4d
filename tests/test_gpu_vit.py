"""ViT block / backbone prefix parity: samq_vit_block_forward_v1 and
samq_vit_prefix_v1 against the f64 oracle (oracle.vit_block / vit_prefix).

The block oracle computes every quantized linear with GGML MMQ's operand
semantics: the input staged with the Q8_1 rule, times the f32-decoded weights
(no f16 rounding), f64 dots.  The device path differs by its f16 tensor-core
operands (the staged values and the weights rounded once to f16, f16 Q/K/V/P
inside attention), f32 accumulation, the f32 LayerNorm and the polynomial
erf-GELU.  Since a staged code can flip by one
when an upstream value moves by an ulp, the bar is on the block's
contribution (out - x): cosine >= 0.9999 and max error <= 1e-2 of its largest
magnitude.  The prefix runs the patch convolution on f16 operands (f32
accumulation) against an f64 convolution of the f32 inputs: cosine >= 0.99999
and max abs error <= 1e-2 on the unit-scale ln_pre output.
"""
import numpy as np
import pytest
import torch

import samq
from oracle import oracle as o

pytestmark = pytest.mark.gpu

E, MLP = 1024, 4736
COS_MIN, DELTA_REL_MAX = 0.9999, 1e-2


def _weights(rng, n, k):
    w = rng.normal(0.0, 0.02, (n, k)).astype(np.float32)
    w[rng.random(w.shape) < 0.01] *= 8.0
    return w


def make_block(rng, window, positions, qtype=o.Q4_K, fc2_type=o.Q8_0, E=E, MLP=MLP, compute=samq.COMPUTE_F16):
    """Random-init block with config-3 statistics: K-quant linears (fc2 Q8_0),
    N(0, 0.02^2) weights with 1% scaled x8, LN gamma 1 + N(0, 0.02^2)."""
    dev = torch.device("cuda")
    host, gpu = {"window": window}, {}
    for name, (n, k, t) in {"qkv": (3 * E, E, qtype), "proj": (E, E, qtype), "fc1": (MLP, E, qtype),
                            "fc2": (E, MLP, fc2_type)}.items():
        rows = o.quantize(t, _weights(rng, n, k))
        host[name + "_w"] = o.dequantize(t, rows, n * k).reshape(n, k)
        host[name + "_q"] = (t, rows)
        gpu[name] = samq.Weights(t, k, n, rows)
        bias = rng.normal(0.0, 0.02, n).astype(np.float32)
        host[name + "_b"] = bias
        gpu[name + "_b"] = torch.from_numpy(bias).to(dev)
    for name in ("norm1", "norm2"):
        w = (1.0 + rng.normal(0.0, 0.02, E)).astype(np.float32)
        b = rng.normal(0.0, 0.02, E).astype(np.float32)
        host[name + "_w"], host[name + "_b"] = w, b
        gpu[name + "_w"], gpu[name + "_b"] = torch.from_numpy(w).to(dev), torch.from_numpy(b).to(dev)
    host["freqs"] = o.rope_freqs(positions, seed=int(rng.integers(1 << 30)))
    gpu["freqs"] = torch.from_numpy(host["freqs"]).to(dev)
    block = samq.VitBlock(window, gpu["norm1_w"], gpu["norm1_b"], gpu["qkv"], gpu["qkv_b"], gpu["proj"],
                          gpu["proj_b"], gpu["norm2_w"], gpu["norm2_b"], gpu["fc1"], gpu["fc1_b"], gpu["fc2"],
                          gpu["fc2_b"], gpu["freqs"], compute=compute)
    return host, block


def run_block(block, x, grid):
    xd = torch.from_numpy(x).cuda()
    samq.vit_block_forward(block, xd, grid, grid)
    samq.check(0)
    return xd.cpu().numpy()


def compare(gpu, ref, x_in):
    dg = (gpu - x_in).astype(np.float64).ravel()
    dr = (ref - x_in).astype(np.float64).ravel()
    cos = float(dg @ dr / (np.linalg.norm(dg) * np.linalg.norm(dr)))
    rel = float(np.abs(dg - dr).max() / np.abs(dr).max())
    return cos, rel


@pytest.mark.parametrize("compute", [samq.COMPUTE_F16, samq.COMPUTE_F32])
@pytest.mark.parametrize("grid,window,seed", [(48, 24, 0), (24, 0, 1), (24, 24, 2)])
def test_vit_block_parity(grid, window, seed, compute):
    rng = np.random.default_rng(seed)
    positions = window * window if window else grid * grid
    host, block = make_block(rng, window, positions, compute=compute)
    x = rng.standard_normal((grid * grid, E)).astype(np.float32)
    out = run_block(block, x, grid)
    ref = o.vit_block(x, host, grid, grid)
    cos, rel = compare(out, ref, x)
    assert cos >= COS_MIN and rel <= DELTA_REL_MAX, (cos, rel)


def test_vit_block_full_grid_windowed():
    """72 x 72 windowed block; windows 0 and 8 checked against the oracle run
    on each window's tokens alone (windows are independent)."""
    rng = np.random.default_rng(5)
    host, block = make_block(rng, 24, 576)
    x = rng.standard_normal((72 * 72, E)).astype(np.float32)
    out = run_block(block, x, 72)
    for w in (0, 8):
        wy, wx = divmod(w, 3)
        ly, lx = np.divmod(np.arange(576), 24)
        toks = (wy * 24 + ly) * 72 + wx * 24 + lx
        ref = o.vit_block(x[toks], host, 24, 24)
        cos, rel = compare(out[toks], ref, x[toks])
        assert cos >= COS_MIN and rel <= DELTA_REL_MAX, (w, cos, rel)


def test_vit_block_full_grid_global():
    """72 x 72 global block; 96 sampled tokens against the oracle (K and V
    over all 5184 tokens)."""
    rng = np.random.default_rng(6)
    host, block = make_block(rng, 0, 72 * 72, qtype=o.Q6_K)
    x = rng.standard_normal((72 * 72, E)).astype(np.float32)
    out = run_block(block, x, 72)
    rows = np.sort(rng.choice(72 * 72, 96, replace=False))
    ref = o.vit_block(x, host, 72, 72, rows=rows)
    cos, rel = compare(out[rows], ref, x[rows])
    assert cos >= COS_MIN and rel <= DELTA_REL_MAX, (cos, rel)


@pytest.mark.parametrize("embed,mlp,grid,window", [(256, 1024, 24, 12), (512, 2048, 16, 0)])
def test_vit_block_other_widths(embed, mlp, grid, window):
    """E = 256 / 512 (the other widths the entry point takes): LayerNorm with 2 / 4
    float4 per lane, and 144-token windows, which are not a multiple of 32
    (the qkv split's direct-store path) and end in a 16-key attention block."""
    rng = np.random.default_rng(embed + grid)
    positions = window * window if window else grid * grid
    host, block = make_block(rng, window, positions, qtype=o.Q5_K, E=embed, MLP=mlp)
    x = rng.standard_normal((grid * grid, embed)).astype(np.float32)
    out = run_block(block, x, grid)
    ref = o.vit_block(x, host, grid, grid)
    cos, rel = compare(out, ref, x)
    assert cos >= COS_MIN and rel <= DELTA_REL_MAX, (cos, rel)


@pytest.mark.parametrize("compute", [samq.COMPUTE_F16, samq.COMPUTE_F32])
@pytest.mark.parametrize("size,patch,pos_grid", [(1008, 14, 24), (224, 14, 8)])
def test_vit_prefix_parity(size, patch, pos_grid, compute):
    rng = np.random.default_rng(size)
    image = ((rng.random((3, size, size)) - 0.5) / 0.5).astype(np.float32)  # U[0,1] normalized
    patch_w = rng.normal(0.0, 0.02, (E, 3, patch, patch)).astype(np.float32)
    pos = rng.normal(0.0, 0.02, (pos_grid, pos_grid, E)).astype(np.float32)
    ln_w = (1.0 + rng.normal(0.0, 0.02, E)).astype(np.float32)
    ln_b = rng.normal(0.0, 0.02, E).astype(np.float32)
    tokens = (size // patch) ** 2
    dev = torch.device("cuda")
    x = torch.empty((tokens, E), device=dev)
    t = [torch.from_numpy(a).to(dev) for a in (image, patch_w, pos, ln_w, ln_b)]
    samq.vit_prefix(t[0], size, size, patch, t[1], E, t[2], pos_grid, t[3], t[4], x, compute=compute)
    samq.check(0)
    out = x.cpu().numpy()
    ref = o.vit_prefix(image, patch, patch_w, pos, ln_w, ln_b)
    d = (out - ref).astype(np.float64).ravel()
    cos = float(out.ravel().astype(np.float64) @ ref.ravel() / (np.linalg.norm(out) * np.linalg.norm(ref)))
    # F16 columns: f16 operands, f32 accumulation; F32: F32 semantics.
    cos_min, abs_max = (0.99999, 1e-2) if compute == samq.COMPUTE_F16 else (1 - 1e-10, 5e-5)
    assert cos >= cos_min and np.abs(d).max() <= abs_max, (cos, np.abs(d).max())


def test_vit_block_rejects_bad_shapes():
    rng = np.random.default_rng(9)
    host, block = make_block(rng, 24, 576)
    x = torch.zeros((50 * 50, E), device="cuda")
    with pytest.raises(samq.SamqError):
        samq.vit_block_forward(block, x, 50, 50)  # 24 does not divide 50


@pytest.mark.parametrize("compute", [samq.COMPUTE_F16, samq.COMPUTE_F32])
@pytest.mark.parametrize("window,grid", [(24, 48), (0, 24)])
def test_vit_block_batch_matches_single_images(window, grid, compute):
    """samq_vit_block_forward_batch_v1 on 3 images (windowed: one grid of
    stacked images; global: one attention group per image) gives each image
    the bits of samq_vit_block_forward_v1 on that image alone."""
    rng = np.random.default_rng(40 + window)
    positions = window * window if window else grid * grid
    host, block = make_block(rng, window, positions, compute=compute)
    batch = 3
    xs = rng.standard_normal((batch, grid * grid, E)).astype(np.float32)
    xd = torch.from_numpy(xs).cuda()
    samq.vit_block_forward(block, xd, grid, grid, batch=batch)
    samq.check(0)
    got = xd.cpu().numpy()
    for b in range(batch):
        np.testing.assert_array_equal(got[b], run_block(block, xs[b], grid))
    cos, rel = compare(got[1], o.vit_block(xs[1], host, grid, grid), xs[1])
    assert cos >= COS_MIN and rel <= DELTA_REL_MAX, (cos, rel)
