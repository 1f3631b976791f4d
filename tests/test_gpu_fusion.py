"""Fusion-encoder layer on the device (samq_fusion_layer_forward_v1) against
oracle.fusion_layer (src/models/sam3/fusion_encoder.hpp:38-150), at the SAM 3
shapes (D = 256, 8 heads of 32, FFN 2048, 33 prompt tokens with the last
padding tokens masked) on a 72 x 72 and a 24 x 24 token grid, with Q8_0
linears (the full-linear Q8_0 profile) and with F32 linears (the mixed
profile's fusion=f32).

Bars on the layer's contribution (out - x): Q8_0, cosine >= 0.9999 and max
error <= 1e-2 of its largest magnitude (Q8_1 re-staging, as the ViT block);
F32, cosine >= 1 - 1e-9 and max error <= 1e-4 of its largest magnitude (F32
semantics end to end).
"""
import numpy as np
import pytest
import torch

import samq
from oracle import oracle as o

pytestmark = pytest.mark.gpu
D, HEADS, FFN, P = 256, 8, 2048, 33


def _dev(a):
    return torch.from_numpy(np.ascontiguousarray(a, dtype=np.float32)).cuda()


def make_layer(rng, quantized):
    host, linears = {}, {}
    shapes = {"sa_in_proj": (3 * D, D), "sa_out_proj": (D, D), "ca_in_proj": (3 * D, D), "ca_out_proj": (D, D),
              "linear1": (FFN, D), "linear2": (D, FFN)}
    for name, (n, k) in shapes.items():
        w = (rng.normal(0, 1, (n, k)) / np.sqrt(k)).astype(np.float32)
        b = rng.normal(0, 0.02, n).astype(np.float32)
        if quantized:
            rows = o.quantize(o.Q8_0, w)
            handle = samq.Weights(o.Q8_0, k, n, rows)
            w = o.dequantize(o.Q8_0, rows, n * k).reshape(n, k)
        else:
            handle = samq.Dense(samq.DENSE_LINEAR, w)
        host[name] = {"w": w, "b": b, "quantized": quantized}
        linears[name] = (handle, _dev(b))
    norms = {}
    for i in (1, 2, 3):
        host[f"norm{i}_w"] = (1 + rng.normal(0, 0.02, D)).astype(np.float32)
        host[f"norm{i}_b"] = rng.normal(0, 0.02, D).astype(np.float32)
        norms[f"norm{i}_w"], norms[f"norm{i}_b"] = _dev(host[f"norm{i}_w"]), _dev(host[f"norm{i}_b"])
    return host, samq.FusionLayer(HEADS, norms, linears)


@pytest.mark.parametrize("quantized", [True, False])
@pytest.mark.parametrize("grid", [24, 72])
def test_fusion_layer_parity(quantized, grid):
    rng = np.random.default_rng(grid + quantized)
    host, layer = make_layer(rng, quantized)
    n = grid * grid
    x = rng.standard_normal((n, D)).astype(np.float32)
    pos = rng.uniform(-1, 1, (n, D)).astype(np.float32)
    prompt = rng.standard_normal((P, D)).astype(np.float32)
    bias = np.zeros(P, np.float32)
    bias[25:32] = -1.0e9  # padding text tokens (the geometry token, last, stays valid)
    xd = _dev(x)
    samq.fusion_layer_forward(layer, xd, _dev(pos), n, _dev(prompt), _dev(bias), P)
    samq.check(0)
    got = xd.cpu().numpy().astype(np.float64)
    ref = o.fusion_layer(x, pos, prompt, bias, host, HEADS).astype(np.float64)
    dg, dr = (got - x).ravel(), (ref - x).ravel()
    cos = float(dg @ dr / (np.linalg.norm(dg) * np.linalg.norm(dr)))
    rel = float(np.abs(dg - dr).max() / np.abs(dr).max())
    cos_min, rel_max = (0.9999, 1e-2) if quantized else (1 - 1e-9, 1e-4)
    assert cos >= cos_min and rel <= rel_max, (cos, rel)
