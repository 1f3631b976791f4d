"""The oracle's f64 module restatements pinned on the CPU to independent
implementations of the same definitions (torch, float64): LayerNorm
(ggml_norm + affine), GroupNorm over NHWC maps, nearest 2x upscaling, erf-GELU,
the general attention (causal mask, additive bias, fully masked rows), the 3x3,
1x1 and stride-2 2x2 convolutions, the 2x2 transposed convolution and the 2x2
max pool of the neck and heads.
These restatements are what the GPU parity tests of the config-4 modules
compare against, so they are checked here against code this repository did
not write."""
import numpy as np
import pytest
import torch
import torch.nn.functional as F

from oracle import oracle as o

TOL = 1e-10


def t64(a):
    return torch.from_numpy(np.ascontiguousarray(np.asarray(a, np.float64)))


def test_layer_norm_matches_torch():
    rng = np.random.default_rng(1)
    x = rng.normal(0, 3, (37, 96)).astype(np.float32)
    w = rng.normal(1, 0.1, 96).astype(np.float32)
    b = rng.normal(0, 0.1, 96).astype(np.float32)
    ref = F.layer_norm(t64(x), (96,), t64(w), t64(b), eps=1e-5).numpy()
    got = o.layer_norm(x, w, b)  # rounded to f32 by the oracle
    np.testing.assert_allclose(got, ref.astype(np.float32), rtol=0, atol=1e-6)


def test_group_norm_nhwc_matches_torch():
    rng = np.random.default_rng(2)
    H, W, C, G = 9, 7, 32, 8
    x = rng.normal(0.5, 2, (H, W, C))
    w = rng.normal(1, 0.2, C)
    b = rng.normal(0, 0.2, C)
    ref = F.group_norm(t64(x).permute(2, 0, 1)[None], G, t64(w), t64(b), eps=1e-5)[0].permute(1, 2, 0).numpy()
    got = o.group_norm_nhwc(x, G, w, b)
    np.testing.assert_allclose(got, ref, rtol=0, atol=TOL)


def test_upsample2x_nhwc_matches_torch_nearest():
    rng = np.random.default_rng(3)
    x = rng.normal(size=(5, 6, 4))
    ref = F.interpolate(t64(x).permute(2, 0, 1)[None], scale_factor=2, mode="nearest")[0].permute(1, 2, 0).numpy()
    np.testing.assert_array_equal(o.upsample2x_nhwc(x), ref)


def test_gelu_erf64_matches_torch():
    v = np.linspace(-8, 8, 1001)
    np.testing.assert_allclose(o.gelu_erf64(v), F.gelu(t64(v), approximate="none").numpy(), rtol=0, atol=1e-14)


@pytest.mark.parametrize("causal,with_bias", [(False, False), (True, False), (False, True)])
def test_attention_gen_matches_torch(causal, with_bias):
    rng = np.random.default_rng(4 + 2 * causal + with_bias)
    heads, hd, lq, lk = 3, 32, 11, 11
    q = rng.normal(size=(lq, heads * hd))
    k = rng.normal(size=(lk, heads * hd))
    v = rng.normal(size=(lk, heads * hd))
    scale = 1.0 / np.sqrt(hd)
    bias = None
    mask = torch.zeros(heads, lq, lk, dtype=torch.float64)
    if with_bias:
        bias = rng.normal(size=(heads, lq, lk))
        bias[:, :, 3] = -np.inf  # a masked key for every query
        mask = t64(bias)
    if causal:
        mask = mask + torch.triu(torch.full((lq, lk), float("-inf"), dtype=torch.float64), diagonal=1)
    qh = t64(q).view(lq, heads, hd).transpose(0, 1)
    kh = t64(k).view(lk, heads, hd).transpose(0, 1)
    vh = t64(v).view(lk, heads, hd).transpose(0, 1)
    s = qh @ kh.transpose(1, 2) * scale + mask
    ref = (torch.softmax(s, dim=-1) @ vh).transpose(0, 1).reshape(lq, heads * hd).numpy()
    got = o.attention_gen(q, k, v, heads, hd, scale, causal=causal, bias=bias)
    np.testing.assert_allclose(np.asarray(got, np.float64), ref, rtol=0, atol=1e-6)


def test_attention_gen_fully_masked_row_is_zero():
    rng = np.random.default_rng(9)
    q = rng.normal(size=(2, 32))
    k = rng.normal(size=(4, 32))
    v = rng.normal(size=(4, 32))
    bias = np.zeros((1, 2, 4))
    bias[0, 1, :] = -np.inf
    got = np.asarray(o.attention_gen(q, k, v, 1, 32, 0.2, bias=bias), np.float64)
    assert np.all(got[1] == 0.0) and np.all(np.isfinite(got[0]))


@pytest.mark.parametrize("k,stride,pad", [(3, 1, None), (1, 1, None), (2, 2, 0)])
def test_conv2d_nhwc_matches_torch(k, stride, pad):
    rng = np.random.default_rng(10 + k)
    H, W, Ci, Co = 8, 10, 5, 7
    x = rng.normal(size=(H, W, Ci))
    w = rng.normal(size=(Co, Ci, k, k))
    b = rng.normal(size=Co)
    p = k // 2 if pad is None else pad
    ref = F.conv2d(t64(x).permute(2, 0, 1)[None], t64(w), t64(b), stride=stride, padding=p)[0].permute(1, 2, 0).numpy()
    np.testing.assert_allclose(o.conv2d_nhwc(x, w, b, stride=stride, pad=pad), ref, rtol=0, atol=TOL)


def test_deconv2x2_nhwc_matches_torch():
    rng = np.random.default_rng(20)
    H, W, Ci, Co = 4, 6, 5, 3
    x = rng.normal(size=(H, W, Ci))
    w = rng.normal(size=(Ci, Co, 2, 2))
    b = rng.normal(size=Co)
    ref = F.conv_transpose2d(t64(x).permute(2, 0, 1)[None], t64(w), t64(b), stride=2)[0].permute(1, 2, 0).numpy()
    np.testing.assert_allclose(o.deconv2x2_nhwc(x, w, b), ref, rtol=0, atol=TOL)


def test_maxpool2x2_nhwc_matches_torch():
    rng = np.random.default_rng(21)
    x = rng.normal(size=(6, 8, 3))
    ref = F.max_pool2d(t64(x).permute(2, 0, 1)[None], 2, 2)[0].permute(1, 2, 0).numpy()
    np.testing.assert_array_equal(np.asarray(o.maxpool2x2_nhwc(x), np.float64), ref)
