"""Seeded synthetic SAM 3 image models (random-init: no checkpoint is needed or
available), tensor by tensor under the reference's GGUF tensor names
(src/models/sam3/tensors.hpp:90-442), quantized by samq_quantize_rows_v1
under a weight profile (src/models/sam3/weights.hpp:81-312).

Statistics follow the benchmark configurations: linear weights N(0, 0.02^2)
with 1% of entries scaled by 8, biases N(0, 0.02^2), LayerNorm gamma
1 + N(0, 0.02^2), unit-modulus RoPE tables (the converter copies the
checkpoint's freqs_cis buffers, so any unit-modulus table is valid).  Module
heads whose random init must stay well conditioned (the box refinement and
scoring layers) are scaled like a trained model's: weights N(0, 1 / k).

Layouts (row-major numpy): linear weights [out][in]; convolutions
[cout][cin][kh][kw]; 2x2 deconvolutions [cin][cout][2][2]; the patch
embedding [E][3][p][p]; vit.pos_embed [24][24][E]; freqs_cis
[positions][32][2]; quantized linears as Quantized(qtype, k, n, rows).
"""
from __future__ import annotations

from dataclasses import dataclass, field

import numpy as np

from . import Q4_K, Q8_0, quantize_rows


@dataclass
class Quantized:
    """Packed GGUF rows of an [n][k] linear weight."""
    qtype: int
    k: int
    n: int
    rows: np.ndarray


@dataclass
class Hparams:
    """SAM 3 image-model hyperparameters (src/models/sam3/architecture.hpp)."""
    img_size: int = 1008
    patch: int = 14
    embed: int = 1024
    depth: int = 32
    mlp: int = 4736
    pos_grid: int = 24
    window: int = 24
    global_blocks: tuple = (7, 15, 23, 31)
    neck_dim: int = 256
    text_width: int = 1024
    text_layers: int = 24
    text_mlp: int = 4096
    vocab: int = 49408
    ctx: int = 32
    fenc_layers: int = 6
    fenc_heads: int = 8
    ffn: int = 2048
    ddec_layers: int = 6
    ddec_heads: int = 8
    queries: int = 200
    geom_layers: int = 3
    seg_heads: int = 8

    @property
    def grid(self) -> int:
        return self.img_size // self.patch

    def window_of(self, block: int) -> int:
        return 0 if block in self.global_blocks else self.window


# Weight profiles: the type of each module's quantizable linears, None = F32.
# "q8_0" is image-full-linear-q8_0-v1; "mixed" the schema-5 policy
# vision=q4_k,text=q8_0,fusion=f32,decoder=f32 (the decoder module covers the
# DETR decoder, scoring, geometry encoder and segmentation head).  K-quant
# vision profiles keep fc2 (4736 wide) in Q8_0 (weights.hpp:148-164).
PROFILES = {
    "q8_0": {"vision": Q8_0, "text": Q8_0, "fusion": Q8_0, "decoder": Q8_0},
    "mixed": {"vision": Q4_K, "text": Q8_0, "fusion": None, "decoder": None},
}


@dataclass
class _Builder:
    rng: np.random.Generator
    profile: dict
    tensors: dict = field(default_factory=dict)

    def f32(self, name, value):
        self.tensors[name] = np.ascontiguousarray(value, dtype=np.float32)

    def linear(self, name, n, k, module, scale=None, bias=True):
        w = self.rng.normal(0.0, 0.02 if scale is None else scale, (n, k)).astype(np.float32)
        if scale is None:
            w[self.rng.random(w.shape) < 0.01] *= 8.0
        qtype = self.profile[module]
        if qtype is not None and module == "vision" and qtype != Q8_0 and k % 256:
            qtype = Q8_0  # the K-quant fc2 fallback
        if qtype is not None and k % (32 if qtype == Q8_0 else 256) == 0:
            self.tensors[name + ".weight"] = Quantized(qtype, k, n, quantize_rows(qtype, w))
        else:
            self.tensors[name + ".weight"] = w
        if bias:
            self.f32(name + ".bias", self.rng.normal(0.0, 0.02, n))

    def fused(self, prefix, n, k, module, in_proj="in_proj", scale=None):
        """An nn.MultiheadAttention in_proj (GGUF names ...in_proj_weight / _bias)."""
        w = self.rng.normal(0.0, 0.02 if scale is None else scale, (n, k)).astype(np.float32)
        if scale is None:
            w[self.rng.random(w.shape) < 0.01] *= 8.0
        qtype = self.profile[module]
        self.tensors[f"{prefix}.{in_proj}_weight"] = (Quantized(qtype, k, n, quantize_rows(qtype, w))
                                                     if qtype is not None else w)
        self.f32(f"{prefix}.{in_proj}_bias", self.rng.normal(0.0, 0.02, n))

    def norm(self, name, width):
        self.f32(name + ".weight", 1.0 + self.rng.normal(0.0, 0.02, width))
        self.f32(name + ".bias", self.rng.normal(0.0, 0.02, width))


def rope_freqs(positions: int, head_dim: int = 64, seed: int = 0) -> np.ndarray:
    """A unit-modulus (cos, sin) table [positions][head_dim / 2][2]."""
    ang = np.random.default_rng(seed).uniform(-np.pi, np.pi, (positions, head_dim // 2))
    return np.stack([np.cos(ang), np.sin(ang)], axis=-1).astype(np.float32)


def linear_weight(rng: np.random.Generator, n: int, k: int) -> np.ndarray:
    """N(0, 0.02^2) with 1% of entries scaled by 8 (the benchmark weights)."""
    w = rng.normal(0.0, 0.02, (n, k)).astype(np.float32)
    w[rng.random(w.shape) < 0.01] *= 8.0
    return w


def sam3_tensors(hp: Hparams, profile: str = "q8_0", seed: int = 0, text: bool = True) -> dict:
    """All tensors of a SAM 3 image model (detector path; text=False leaves
    out the text encoder) keyed by GGUF name."""
    b = _Builder(np.random.default_rng(seed), PROFILES[profile])
    E, D = hp.embed, hp.neck_dim
    # ViT backbone (tensors.hpp:97-127)
    b.f32("vit.patch_embed.proj.weight", b.rng.normal(0.0, 0.02, (E, 3, hp.patch, hp.patch)))
    b.f32("vit.pos_embed", b.rng.normal(0.0, 0.02, (hp.pos_grid, hp.pos_grid, E)))
    b.norm("vit.ln_pre", E)
    for i in range(hp.depth):
        p = f"vit.blocks.{i}"
        b.norm(p + ".norm1", E)
        b.linear(p + ".attn.qkv", 3 * E, E, "vision")
        b.linear(p + ".attn.proj", E, E, "vision")
        b.norm(p + ".norm2", E)
        b.linear(p + ".mlp.lin1", hp.mlp, E, "vision")
        b.linear(p + ".mlp.lin2", E, hp.mlp, "vision")
        window = hp.window_of(i)
        positions = hp.grid * hp.grid if window == 0 else window * window
        b.f32(p + ".attn.freqs_cis", rope_freqs(positions, seed=seed * 1000 + i))
    # Neck (detector), F32 convolutions (tensors.hpp:129-170)
    conv = lambda cout, cin, ks: b.rng.normal(0.0, 1.0 / np.sqrt(cin * ks * ks), (cout, cin, ks, ks))
    deconv = lambda cin, cout: b.rng.normal(0.0, 1.0 / np.sqrt(cin), (cin, cout, 2, 2))
    bias = lambda n: b.rng.normal(0.0, 0.02, n)
    for name, w, n in (("0.dconv_2x2_0", deconv(E, 512), 512), ("0.dconv_2x2_1", deconv(512, D), D),
                       ("0.conv_1x1", conv(D, D, 1), D), ("0.conv_3x3", conv(D, D, 3), D),
                       ("1.dconv_2x2", deconv(E, 512), 512), ("1.conv_1x1", conv(D, 512, 1), D),
                       ("1.conv_3x3", conv(D, D, 3), D), ("2.conv_1x1", conv(D, E, 1), D),
                       ("2.conv_3x3", conv(D, D, 3), D), ("3.conv_1x1", conv(D, E, 1), D),
                       ("3.conv_3x3", conv(D, D, 3), D)):
        b.f32(f"neck.det.{name}.weight", w)
        b.f32(f"neck.det.{name}.bias", bias(n))
    # Text encoder (tensors.hpp:196-223)
    if text:
        T = hp.text_width
        b.f32("text.token_embed.weight", b.rng.normal(0.0, 0.02, (hp.vocab, T)))
        b.f32("text.pos_embed", b.rng.normal(0.0, 0.01, (hp.ctx, T)))
        for i in range(hp.text_layers):
            p = f"text.blocks.{i}"
            b.linear(p + ".attn.in_proj", 3 * T, T, "text")
            b.linear(p + ".attn.out_proj", T, T, "text")
            b.norm(p + ".ln_1", T)
            b.norm(p + ".ln_2", T)
            b.linear(p + ".mlp.fc1", hp.text_mlp, T, "text")
            b.linear(p + ".mlp.fc2", T, hp.text_mlp, "text")
        b.norm("text.ln_final", T)
        b.linear("text.resizer", D, T, "text")
    # Fusion encoder (tensors.hpp:226-253)
    for i in range(hp.fenc_layers):
        p = f"fenc.layers.{i}"
        b.fused(p + ".sa", 3 * D, D, "fusion")
        b.linear(p + ".sa.out_proj", D, D, "fusion")
        b.fused(p + ".ca", 3 * D, D, "fusion")
        b.linear(p + ".ca.out_proj", D, D, "fusion")
        b.linear(p + ".linear1", hp.ffn, D, "fusion")
        b.linear(p + ".linear2", D, hp.ffn, "fusion")
        for nm in ("norm1", "norm2", "norm3"):
            b.norm(f"{p}.{nm}", D)
    # DETR decoder, scoring (tensors.hpp:255-351)
    unit = lambda k: 1.0 / np.sqrt(k)
    b.f32("ddec.query_embed.weight", b.rng.normal(0.0, 1.0, (hp.queries, D)))
    b.f32("ddec.presence_token.weight", b.rng.normal(0.0, 1.0, D))
    b.f32("ddec.reference_points.weight", b.rng.normal(0.0, 1.2, (hp.queries, 4)))
    b.norm("ddec.norm", D)
    for j, out in enumerate((D, D, 4)):
        b.linear(f"ddec.bbox_embed.layers.{j}", out, D, "decoder", scale=unit(D) * (0.2 if j == 2 else 1.0))
    b.linear("ddec.ref_point_head.layers.0", D, 512, "decoder", scale=unit(512))
    b.linear("ddec.ref_point_head.layers.1", D, D, "decoder", scale=unit(D))
    for axis in ("x", "y"):
        b.f32(f"ddec.boxRPB_embed_{axis}.layers.0.weight", b.rng.normal(0.0, 1.0, (D, 2)))
        b.f32(f"ddec.boxRPB_embed_{axis}.layers.0.bias", b.rng.normal(0.0, 0.1, D))
        b.linear(f"ddec.boxRPB_embed_{axis}.layers.1", hp.ddec_heads, D, "decoder", scale=unit(D))
    for j, out in enumerate((D, D, 1)):
        b.linear(f"ddec.presence_token_head.layers.{j}", out, D, "decoder", scale=unit(D))
    b.norm("ddec.presence_token_out_norm", D)
    for i in range(hp.ddec_layers):
        p = f"ddec.layers.{i}"
        for att in ("sa", "ca", "ca_text"):
            b.fused(f"{p}.{att}", 3 * D, D, "decoder", scale=unit(D))
            b.linear(f"{p}.{att}.out_proj", D, D, "decoder", scale=unit(D))
        b.linear(p + ".linear1", hp.ffn, D, "decoder", scale=unit(D))
        b.linear(p + ".linear2", D, hp.ffn, "decoder", scale=unit(hp.ffn))
        for nm in ("norm1", "norm2", "norm_ca_text", "norm3"):
            b.norm(f"{p}.{nm}", D)
    b.linear("scoring.prompt_proj", D, D, "decoder", scale=unit(D))
    b.linear("scoring.hs_proj", D, D, "decoder", scale=unit(D))
    b.linear("scoring.prompt_mlp.layers.0", hp.ffn, D, "decoder", scale=unit(D))
    b.linear("scoring.prompt_mlp.layers.1", D, hp.ffn, "decoder", scale=unit(hp.ffn))
    b.norm("scoring.prompt_mlp.out_norm", D)
    # Geometry encoder, text-only prompt form (tensors.hpp:354-403)
    b.f32("geom.cls_embed.weight", b.rng.normal(0.0, 1.0, D))
    b.linear("geom.final_proj", D, D, "decoder", scale=unit(D))
    b.norm("geom.norm", D)
    b.norm("geom.encode_norm", D)
    for i in range(hp.geom_layers):
        p = f"geom.layers.{i}"
        for att in ("sa", "ca"):
            b.fused(f"{p}.{att}", 3 * D, D, "decoder", scale=unit(D))
            b.linear(f"{p}.{att}.out_proj", D, D, "decoder", scale=unit(D))
        b.linear(p + ".linear1", hp.ffn, D, "decoder", scale=unit(D))
        b.linear(p + ".linear2", D, hp.ffn, "decoder", scale=unit(hp.ffn))
        for nm in ("norm1", "norm2", "norm3"):
            b.norm(f"{p}.{nm}", D)
    # Segmentation head (tensors.hpp:405-442)
    for i in range(2):
        b.f32(f"seg.pixel_decoder.conv_layers.{i}.weight", conv(D, D, 3))
        b.f32(f"seg.pixel_decoder.conv_layers.{i}.bias", bias(D))
        b.norm(f"seg.pixel_decoder.norms.{i}", D)
    for j in range(3):
        b.linear(f"seg.mask_predictor.mask_embed.layers.{j}", D, D, "decoder", scale=unit(D))
    b.fused("seg.cross_attend_prompt", 3 * D, D, "decoder", scale=unit(D))
    b.linear("seg.cross_attend_prompt.out_proj", D, D, "decoder", scale=unit(D))
    b.norm("seg.cross_attn_norm", D)
    b.f32("seg.instance_seg_head.weight", conv(D, D, 1))
    b.f32("seg.instance_seg_head.bias", bias(D))
    return b.tensors


def image(hp: Hparams, seed: int) -> np.ndarray:
    """U[0,1] pixels normalised (x - 0.5) / 0.5 (image_ops.hpp:98-103), [3][S][S]."""
    rng = np.random.default_rng(seed)
    return ((rng.random((3, hp.img_size, hp.img_size)) - 0.5) / 0.5).astype(np.float32)


def token_ids(hp: Hparams, seed: int, length: int | None = None) -> np.ndarray:
    """The API-valid token form [49406, ids, 49407, 0 padding] (tokenizer.hpp:103-118)."""
    rng = np.random.default_rng(seed)
    n = hp.ctx - 2 if length is None else length
    ids = np.zeros(hp.ctx, np.int32)
    ids[0] = 49406
    ids[1:1 + n] = rng.integers(1, 49405, n)
    ids[1 + n] = 49407
    return ids
