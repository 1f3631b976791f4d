"""DETR decoder, dot-product scoring and presence head on the device
(samq_decoder_forward_v1) against oracle.decoder
(src/models/sam3/detector.hpp:67-713), at the SAM 3 shapes (D = 256, 8 heads
of 32, FFN 2048, 200 queries, 6 layers, 33 prompt tokens of which the last
padding tokens are masked) on a 24 x 24 and the 72 x 72 token grid.

F32 linears (the mixed profile's decoder=f32): F32 semantics end to end, so
the outputs agree to f32 level: queries max error <= 1e-3 of their largest
magnitude, boxes <= 1e-4 absolute, scores and presence <= 1e-3 absolute.

Q8_0 linears (the full-linear Q8_0 profile): every linear re-stages its input
to Q8_1, so a 1-ulp difference ahead of a staging step can move a quantized
value by a whole step, and six post-norm layers carry it on.  The yardstick is
the oracle's own response to an f32-level perturbation of its inputs (one ulp
of noise on the encoder features): the device's distance from the oracle may
be at most 2x that drift plus a small floor, per output.
"""
import numpy as np
import pytest
import torch

import samq
from oracle import oracle as o

pytestmark = pytest.mark.gpu
D, HEADS, FFN, P, NQ, LAYERS, SCORE_FFN = 256, 8, 2048, 33, 200, 6, 2048


def _dev(a):
    return torch.from_numpy(np.ascontiguousarray(a, dtype=np.float32)).cuda()


def _linear(rng, n, k, quantized, scale=1.0):
    w = (rng.normal(0, 1, (n, k)) * scale / np.sqrt(k)).astype(np.float32)
    b = rng.normal(0, 0.02, n).astype(np.float32)
    if quantized:
        rows = o.quantize(o.Q8_0, w)
        handle = samq.Weights(o.Q8_0, k, n, rows)
        w = o.dequantize(o.Q8_0, rows, n * k).reshape(n, k)
    else:
        handle = samq.Dense(samq.DENSE_LINEAR, w)
    return {"w": w, "b": b, "quantized": quantized}, (handle, _dev(b))


def _norm(rng):
    return (1 + rng.normal(0, 0.05, D)).astype(np.float32), rng.normal(0, 0.02, D).astype(np.float32)


def make_decoder(rng, quantized):
    host = {"layers": []}
    dev_layers = []
    shapes = {"sa_in_proj": (3 * D, D), "sa_out_proj": (D, D), "ca_text_in_proj": (3 * D, D),
              "ca_text_out_proj": (D, D), "ca_in_proj": (3 * D, D), "ca_out_proj": (D, D), "linear1": (FFN, D),
              "linear2": (D, FFN)}
    for _ in range(LAYERS):
        hl, dl = {}, {}
        for name, (n, k) in shapes.items():
            hl[name], dl[name] = _linear(rng, n, k, quantized)
        for nm in ("norm1", "norm2", "norm_ca_text", "norm3"):
            w, b = _norm(rng)
            hl[nm + "_w"], hl[nm + "_b"] = w, b
            dl[nm + "_w"], dl[nm + "_b"] = _dev(w), _dev(b)
        host["layers"].append(hl)
        dev_layers.append(dl)
    params = {}

    def param(name, value):
        host[name] = np.asarray(value, np.float32)
        params[name] = _dev(host[name])

    param("query_embed", rng.normal(0, 1, (NQ, D)))
    param("presence_token", rng.normal(0, 1, D))
    param("reference_points", rng.normal(0, 1.2, (NQ, 4)))
    for axis in ("x", "y"):
        param(f"rpb_{axis}0_w", rng.normal(0, 1.0, (256, 2)))
        param(f"rpb_{axis}0_b", rng.normal(0, 0.1, 256))
    for nm in ("norm", "presence_norm", "prompt_mlp_norm"):
        w, b = _norm(rng)
        param(nm + "_w", w)
        param(nm + "_b", b)
    lin = {}

    def chain(name, dims, last_scale=1.0):
        hs, ds = [], []
        for j in range(len(dims) - 1):
            h, d = _linear(rng, dims[j + 1], dims[j], quantized, last_scale if j == len(dims) - 2 else 1.0)
            hs.append(h)
            ds.append(d)
        host[name], lin[name] = hs, ds

    chain("ref_point_head", [512, D, D])
    chain("bbox_embed", [D, D, D, 4], last_scale=0.2)
    chain("presence_head", [D, D, D, 1])
    chain("prompt_mlp", [D, SCORE_FFN, D])
    for name, (n, k) in {"rpb_x1": (HEADS, 256), "rpb_y1": (HEADS, 256), "prompt_proj": (D, D),
                         "hs_proj": (D, D)}.items():
        host[name], lin[name] = _linear(rng, n, k, quantized)
    return host, samq.Decoder(HEADS, NQ, dev_layers, params, lin)


def inputs(rng, grid):
    n = grid * grid
    enc = rng.standard_normal((n, D)).astype(np.float32)
    pos = rng.uniform(-1, 1, (n, D)).astype(np.float32)
    prompt = rng.standard_normal((P, D)).astype(np.float32)
    bias = np.zeros(P, np.float32)
    bias[25:32] = -1.0e9  # padding text tokens (the geometry token, last, stays valid)
    valid = np.where(bias == 0, P / np.count_nonzero(bias == 0), 0).astype(np.float32)
    return enc, pos, prompt, bias, valid


def run_device(dec, grid, enc, pos, prompt, bias, valid):
    qo = torch.zeros((NQ + 1, D), device="cuda")
    boxes = torch.zeros((NQ, 4), device="cuda")
    scores = torch.zeros(NQ, device="cuda")
    presence = torch.zeros(1, device="cuda")
    samq.decoder_forward(dec, _dev(enc), _dev(pos), grid, _dev(prompt), _dev(bias), _dev(valid), P, qo, boxes, scores,
                         presence)
    samq.check(0)
    return qo.cpu().numpy(), boxes.cpu().numpy(), scores.cpu().numpy(), float(presence.cpu().numpy()[0])


def distances(a, b):
    qa, ba, sa, pa = a
    qb, bb, sb, pb = b
    return {"queries": float(np.abs(qa.astype(np.float64) - qb).max() / np.abs(qb).max()),
            "boxes": float(np.abs(ba.astype(np.float64) - bb).max()),
            "scores": float(np.abs(sa.astype(np.float64) - sb).max()),
            "presence": abs(pa - pb)}


@pytest.mark.parametrize("grid", [24, 72])
def test_decoder_f32_linears(grid):
    rng = np.random.default_rng(100 + grid)
    host, dec = make_decoder(rng, False)
    args = inputs(rng, grid)
    got = run_device(dec, grid, *args)
    ref = o.decoder(args[0], args[1], args[2], args[3], args[4], host, grid, HEADS)
    d = distances(got, ref)
    print(grid, d)
    assert d["queries"] <= 1e-3 and d["boxes"] <= 1e-4 and d["scores"] <= 1e-3 and d["presence"] <= 1e-3, d


@pytest.mark.parametrize("grid", [24, 72])
def test_decoder_q8_0_linears(grid):
    rng = np.random.default_rng(200 + grid)
    host, dec = make_decoder(rng, True)
    enc, pos, prompt, bias, valid = inputs(rng, grid)
    got = run_device(dec, grid, enc, pos, prompt, bias, valid)
    ref = o.decoder(enc, pos, prompt, bias, valid, host, grid, HEADS)
    noisy_enc = (enc + enc * np.float32(2.0 ** -23) * np.random.default_rng(7).choice([-1, 1], enc.shape)).astype(
        np.float32)
    noisy = o.decoder(noisy_enc, pos, prompt, bias, valid, host, grid, HEADS)
    d, drift = distances(got, ref), distances(noisy, ref)
    print(grid, d, drift)
    floors = {"queries": 2e-3, "boxes": 1e-3, "scores": 1e-2, "presence": 1e-2}
    for key, floor in floors.items():
        assert d[key] <= 2.0 * drift[key] + floor, (key, d, drift)
    # the drift itself stays small: the decoder is not amplifying f32 noise into wrong detections
    assert drift["boxes"] <= 0.05 and drift["queries"] <= 0.1, drift
