"""Geometry encoder (samq_geometry_encoder_forward_v1) and segmentation head
(samq_seg_head_forward_v1) on the device against oracle.geometry_encoder
(src/models/sam3/prompt_encoder.hpp:44-160) and oracle.seg_head
(src/models/sam3/mask_decoder.hpp:57-202), at the SAM 3 shapes (D = 256,
8 heads of 32, FFN 2048, 200 object queries, 33 prompt tokens) on a 24 x 24
and the 72 x 72 grid (mask logits at 288 x 288).

F32 linears: F32 semantics end to end, max error <= 1e-4 of the output's
largest magnitude.  Q8_0 linears: the quantized GEMM multiplies f16 operands
(the decoded weight and the decoded Q8_1 activation, each rounded to f16), so
it is held to the oracle evaluated over those exact operands
(oracle.exact_operands): at most 2x that oracle's drift under one ulp of noise
on the image input plus 1e-3 (relative to the largest magnitude).  Against
GGML MMQ's decoded-operand semantics its distance may exceed the exact-operand
oracle's own distance from them by at most 1e-3.
"""
import numpy as np
import pytest
import torch

import samq
from oracle import oracle as o

pytestmark = pytest.mark.gpu
D, HEADS, FFN, P, NQ = 256, 8, 2048, 33, 200


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


def _noisy(x, seed=7):
    return (x + x * np.float32(2.0 ** -23) * np.random.default_rng(seed).choice([-1, 1], x.shape)).astype(np.float32)


def _rel(a, b):
    b = np.asarray(b, np.float64)
    return float(np.abs(np.asarray(a, np.float64) - b).max() / np.abs(b).max())


def make_geometry(rng, quantized):
    host = {"layers": []}
    layers = []
    shapes = {"sa_in_proj": (3 * D, D), "sa_out_proj": (D, D), "ca_in_proj": (3 * D, D), "ca_out_proj": (D, D),
              "linear1": (FFN, D), "linear2": (D, FFN)}
    for _ in range(3):
        hl, dl = {}, {}
        for name, (n, k) in shapes.items():
            hl[name], dl[name] = _linear(rng, n, k, quantized)
        for nm in ("norm1", "norm2", "norm3"):
            w, b = _norm(rng)
            hl[nm + "_w"], hl[nm + "_b"] = w, b
            dl[nm + "_w"], dl[nm + "_b"] = _dev(w), _dev(b)
        host["layers"].append(hl)
        layers.append(dl)
    host["cls"] = rng.normal(0, 1, D).astype(np.float32)
    params = {"cls_token": _dev(host["cls"])}
    for nm in ("norm", "encode_norm"):
        w, b = _norm(rng)
        host[nm + "_w"], host[nm + "_b"] = w, b
        params[nm + "_w"], params[nm + "_b"] = _dev(w), _dev(b)
    host["final_proj"], fp = _linear(rng, D, D, quantized)
    return host, samq.GeometryEncoder(HEADS, layers, params, fp)


@pytest.mark.parametrize("quantized", [False, True])
def test_geometry_encoder(quantized):
    grid = 72
    rng = np.random.default_rng(300 + quantized)
    host, enc = make_geometry(rng, quantized)
    image = rng.standard_normal((grid * grid, D)).astype(np.float32)
    pos = samq.sine_pe_2d(grid, grid, D)
    out = torch.zeros(D, device="cuda")
    samq.geometry_encoder_forward(enc, _dev(image), _dev(pos), grid * grid, out)
    samq.check(0)
    got = out.cpu().numpy()
    ref = o.geometry_encoder(image, pos, host, HEADS)[0]
    err = _rel(got, ref)
    if not quantized:
        assert err <= 1e-4, err
        return
    with o.exact_operands():
        exact = o.geometry_encoder(image, pos, host, HEADS)[0]
        drift = _rel(o.geometry_encoder(_noisy(image), pos, host, HEADS)[0], exact)
    err_exact, operand = _rel(got, exact), _rel(exact, ref)
    print("geometry", err, err_exact, drift, operand)
    assert err_exact <= 2.0 * drift + 1e-3, (err_exact, drift)
    assert err <= operand + 1e-3, (err, operand)


def make_seg_head(rng, quantized):
    host = {}
    params = {}
    for nm in ("cross_attn_norm",):
        w, b = _norm(rng)
        host[nm + "_w"], host[nm + "_b"] = w, b
        params[nm + "_w"], params[nm + "_b"] = _dev(w), _dev(b)
    host["ca_in_proj"], ca_in = _linear(rng, 3 * D, D, quantized)
    host["ca_out_proj"], ca_out = _linear(rng, D, D, quantized)
    host["conv_w"], host["conv_b"], host["norm_w"], host["norm_b"] = [], [], [], []
    convs = []
    params["conv_b"], params["norm_w"], params["norm_b"] = [], [], []
    for _ in range(2):
        w = (rng.normal(0, 1, (D, D, 3, 3)) / np.sqrt(9 * D)).astype(np.float32)
        b = rng.normal(0, 0.02, D).astype(np.float32)
        gw, gb = _norm(rng)
        host["conv_w"].append(w)
        host["conv_b"].append(b)
        host["norm_w"].append(gw)
        host["norm_b"].append(gb)
        convs.append(samq.Dense(samq.DENSE_CONV, w))
        params["conv_b"].append(_dev(b))
        params["norm_w"].append(_dev(gw))
        params["norm_b"].append(_dev(gb))
    host["instance_w"] = (rng.normal(0, 1, (D, D, 1, 1)) / np.sqrt(D)).astype(np.float32)
    host["instance_b"] = rng.normal(0, 0.02, D).astype(np.float32)
    instance = samq.Dense(samq.DENSE_CONV, host["instance_w"])
    params["instance_b"] = _dev(host["instance_b"])
    host["mask_embed"], me = [], []
    for _ in range(3):
        h, d = _linear(rng, D, D, quantized)
        host["mask_embed"].append(h)
        me.append(d)
    return host, samq.SegHead(HEADS, params, convs, instance, ca_in, ca_out, me)


def seg_inputs(rng, grid):
    enc = rng.standard_normal((grid * grid, D)).astype(np.float32)
    fpn1 = rng.standard_normal((4 * grid * grid, D)).astype(np.float32)
    fpn0 = rng.standard_normal((16 * grid * grid, D)).astype(np.float32)
    queries = rng.standard_normal((NQ, D)).astype(np.float32)
    prompt = rng.standard_normal((P, D)).astype(np.float32)
    bias = np.zeros(P, np.float32)
    bias[25:32] = -1.0e9
    return enc, fpn0, fpn1, queries, prompt, bias


def run_seg(head, grid, enc, fpn0, fpn1, queries, prompt, bias):
    logits = torch.zeros((NQ, 16 * grid * grid), device="cuda")
    samq.seg_head_forward(head, _dev(enc), grid, _dev(fpn0), _dev(fpn1), _dev(queries), NQ, _dev(prompt), _dev(bias),
                          P, logits)
    samq.check(0)
    return logits.cpu().numpy()


@pytest.mark.parametrize("grid", [24, 72])
def test_seg_head_f32_linears(grid):
    rng = np.random.default_rng(400 + grid)
    host, head = make_seg_head(rng, False)
    args = seg_inputs(rng, grid)
    got = run_seg(head, grid, *args)
    ref = o.seg_head(*args[:5], args[5], host, grid, HEADS)
    err = _rel(got, ref)
    print("seg f32", grid, err)
    assert err <= 1e-4, err


@pytest.mark.parametrize("grid", [24, 72])
def test_seg_head_q8_0_linears(grid):
    rng = np.random.default_rng(500 + grid)
    host, head = make_seg_head(rng, True)
    enc, fpn0, fpn1, queries, prompt, bias = seg_inputs(rng, grid)
    got = run_seg(head, grid, enc, fpn0, fpn1, queries, prompt, bias)
    ref = o.seg_head(enc, fpn0, fpn1, queries, prompt, bias, host, grid, HEADS)
    with o.exact_operands():
        exact = o.seg_head(enc, fpn0, fpn1, queries, prompt, bias, host, grid, HEADS)
        drift = _rel(o.seg_head(_noisy(enc), fpn0, fpn1, queries, prompt, bias, host, grid, HEADS), exact)
    err, err_exact, operand = _rel(got, ref), _rel(got, exact), _rel(exact, ref)
    print("seg q8_0", grid, err, err_exact, drift, operand)
    assert err_exact <= 2.0 * drift + 1e-3, (err_exact, drift)
    assert err <= operand + 1e-3, (err, operand)
