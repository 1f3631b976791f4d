"""The SAM 3 image path on the device, stage by stage as the reference's
ModelDefinition runs it (src/models/sam3/execution.hpp:55-343):

  encode_image(pixels)      ViT prefix + 32 blocks, the detector neck, the
                            image positional encoding and the geometry token
  encode_text(ids)          token embedding, 24 causal blocks, final LayerNorm,
                            the 1024 -> 256 resizer
  prepare_prompt(...)       text tokens + geometry token, key bias and pooling
                            weights (execution.hpp:157-175)
  predict(features, ids, text)
                            fusion encoder, DETR decoder with scoring and
                            presence, segmentation head: boxes, class logits,
                            presence logit and mask logits [Q][(4 grid)^2]

Every stage is a C-ABI call of libsamq (no host arithmetic on activations);
weights are loaded from a tensor dict keyed by GGUF name (samq.synthetic
writes one): quantized linears become Weights handles (K4 repack), F32
linears and convolutions Dense handles, everything else device tensors.
"""
from __future__ import annotations

from dataclasses import dataclass

import numpy as np

from . import (COMPUTE_F32, DENSE_CONV, DENSE_DECONV2X2, DENSE_LINEAR, EPILOGUE_NONE, NECK_LAYERS, Decoder, Dense,
               FusionLayer, GeometryEncoder, Neck, SegHead, TextBlock, VitBlock, Weights, decoder_forward,
               fusion_layer_forward, geometry_encoder_forward, layer_norm, linear, neck_forward, seg_head_forward,
               sine_pe_2d, text_block_forward, token_embed, vit_block_forward, vit_prefix)
from .synthetic import Hparams, Quantized

NECK_NAMES = {"s0_deconv1": "0.dconv_2x2_0", "s0_deconv2": "0.dconv_2x2_1", "s0_conv1x1": "0.conv_1x1",
              "s0_conv3x3": "0.conv_3x3", "s1_deconv1": "1.dconv_2x2", "s1_conv1x1": "1.conv_1x1",
              "s1_conv3x3": "1.conv_3x3", "s2_conv1x1": "2.conv_1x1", "s2_conv3x3": "2.conv_3x3",
              "s3_conv1x1": "3.conv_1x1", "s3_conv3x3": "3.conv_3x3"}


@dataclass
class ImageFeatures:
    """encode_image's result: the neck maps at 4x, 2x, 1x ([pixels][D] NHWC),
    the image positional encoding and the geometry prompt token."""
    neck: list
    position: object
    geometry: object
    grid: int


@dataclass
class Prompt:
    tokens: object      # [T + 1][D] device: text tokens then the geometry token
    bias: object        # [T + 1] device additive key bias (0 / -1e9)
    validity: object    # [T + 1] device pooling weights


@dataclass
class Prediction:
    fusion: object
    queries: object     # [Q + 1][D]: presence query, normalized object queries
    boxes: object       # [Q][4] (cx, cy, w, h)
    class_logits: object
    presence_logit: object
    mask_logits: object  # [Q][(4 grid)^2]


class Sam3Image:
    """A SAM 3 image model resident on one device."""

    def __init__(self, tensors: dict, hp: Hparams, compute: int = COMPUTE_F32, device: int = 0):
        import torch
        self.torch = torch
        self.hp, self.compute, self.device = hp, compute, device
        self.dev = torch.device("cuda", device)
        self._t = tensors
        self._keep = []
        E, D = hp.embed, hp.neck_dim
        t = self.tensor
        # ViT
        self.patch_w, self.pos_embed = t("vit.patch_embed.proj.weight"), t("vit.pos_embed")
        self.ln_pre = (t("vit.ln_pre.weight"), t("vit.ln_pre.bias"))
        self.blocks = []
        for i in range(hp.depth):
            p = f"vit.blocks.{i}"
            self.blocks.append(VitBlock(hp.window_of(i), t(p + ".norm1.weight"), t(p + ".norm1.bias"),
                                        self.quantized(p + ".attn.qkv.weight"), t(p + ".attn.qkv.bias"),
                                        self.quantized(p + ".attn.proj.weight"), t(p + ".attn.proj.bias"),
                                        t(p + ".norm2.weight"), t(p + ".norm2.bias"),
                                        self.quantized(p + ".mlp.lin1.weight"), t(p + ".mlp.lin1.bias"),
                                        self.quantized(p + ".mlp.lin2.weight"), t(p + ".mlp.lin2.bias"),
                                        t(p + ".attn.freqs_cis"), compute=compute))
        neck = {}
        for ours, name in NECK_NAMES.items():
            w = tensors[f"neck.det.{name}.weight"]
            kind = DENSE_DECONV2X2 if "dconv" in name else DENSE_CONV
            neck[ours] = (self._dense(kind, w), t(f"neck.det.{name}.bias"))
        self.neck = Neck(neck)
        # Text encoder
        self.has_text = "text.token_embed.weight" in tensors
        if self.has_text:
            self.token_table, self.text_pos = t("text.token_embed.weight"), t("text.pos_embed")
            self.text_blocks = []
            for i in range(hp.text_layers):
                p = f"text.blocks.{i}"
                self.text_blocks.append(TextBlock(
                    t(p + ".ln_1.weight"), t(p + ".ln_1.bias"), self.quantized(p + ".attn.in_proj.weight"),
                    t(p + ".attn.in_proj.bias"), self.quantized(p + ".attn.out_proj.weight"),
                    t(p + ".attn.out_proj.bias"), t(p + ".ln_2.weight"), t(p + ".ln_2.bias"),
                    self.quantized(p + ".mlp.fc1.weight"), t(p + ".mlp.fc1.bias"),
                    self.quantized(p + ".mlp.fc2.weight"), t(p + ".mlp.fc2.bias")))
            self.ln_final = (t("text.ln_final.weight"), t("text.ln_final.bias"))
            self.resizer = (self.quantized("text.resizer.weight"), t("text.resizer.bias"))
        # Geometry encoder
        lin = self.linear_pair
        geo_layers = []
        for i in range(hp.geom_layers):
            p = f"geom.layers.{i}"
            geo_layers.append({"sa_in_proj": lin(p + ".sa.in_proj_weight", p + ".sa.in_proj_bias"),
                               "sa_out_proj": lin(p + ".sa.out_proj.weight", p + ".sa.out_proj.bias"),
                               "ca_in_proj": lin(p + ".ca.in_proj_weight", p + ".ca.in_proj_bias"),
                               "ca_out_proj": lin(p + ".ca.out_proj.weight", p + ".ca.out_proj.bias"),
                               "linear1": lin(p + ".linear1.weight", p + ".linear1.bias"),
                               "linear2": lin(p + ".linear2.weight", p + ".linear2.bias"),
                               **self.norms(p, ("norm1", "norm2", "norm3"))})
        self.geometry = GeometryEncoder(hp.fenc_heads, geo_layers,
                                        {"cls_token": t("geom.cls_embed.weight"), "norm_w": t("geom.norm.weight"),
                                         "norm_b": t("geom.norm.bias"), "encode_norm_w": t("geom.encode_norm.weight"),
                                         "encode_norm_b": t("geom.encode_norm.bias")},
                                        lin("geom.final_proj.weight", "geom.final_proj.bias"))
        # Fusion encoder
        self.fusion = []
        for i in range(hp.fenc_layers):
            p = f"fenc.layers.{i}"
            self.fusion.append(FusionLayer(
                hp.fenc_heads, self.norms(p, ("norm1", "norm2", "norm3")),
                {"sa_in_proj": lin(p + ".sa.in_proj_weight", p + ".sa.in_proj_bias"),
                 "sa_out_proj": lin(p + ".sa.out_proj.weight", p + ".sa.out_proj.bias"),
                 "ca_in_proj": lin(p + ".ca.in_proj_weight", p + ".ca.in_proj_bias"),
                 "ca_out_proj": lin(p + ".ca.out_proj.weight", p + ".ca.out_proj.bias"),
                 "linear1": lin(p + ".linear1.weight", p + ".linear1.bias"),
                 "linear2": lin(p + ".linear2.weight", p + ".linear2.bias")}))
        # DETR decoder + scoring
        layers = []
        for i in range(hp.ddec_layers):
            p = f"ddec.layers.{i}"
            ly = {}
            for att, ours in (("sa", "sa"), ("ca_text", "ca_text"), ("ca", "ca")):
                ly[f"{ours}_in_proj"] = lin(f"{p}.{att}.in_proj_weight", f"{p}.{att}.in_proj_bias")
                ly[f"{ours}_out_proj"] = lin(f"{p}.{att}.out_proj.weight", f"{p}.{att}.out_proj.bias")
            ly["linear1"] = lin(p + ".linear1.weight", p + ".linear1.bias")
            ly["linear2"] = lin(p + ".linear2.weight", p + ".linear2.bias")
            ly.update(self.norms(p, ("norm1", "norm2", "norm_ca_text", "norm3")))
            layers.append(ly)
        params = {"query_embed": t("ddec.query_embed.weight"), "presence_token": t("ddec.presence_token.weight"),
                  "reference_points": t("ddec.reference_points.weight"),
                  "rpb_x0_w": t("ddec.boxRPB_embed_x.layers.0.weight"),
                  "rpb_x0_b": t("ddec.boxRPB_embed_x.layers.0.bias"),
                  "rpb_y0_w": t("ddec.boxRPB_embed_y.layers.0.weight"),
                  "rpb_y0_b": t("ddec.boxRPB_embed_y.layers.0.bias"),
                  "norm_w": t("ddec.norm.weight"), "norm_b": t("ddec.norm.bias"),
                  "presence_norm_w": t("ddec.presence_token_out_norm.weight"),
                  "presence_norm_b": t("ddec.presence_token_out_norm.bias"),
                  "prompt_mlp_norm_w": t("scoring.prompt_mlp.out_norm.weight"),
                  "prompt_mlp_norm_b": t("scoring.prompt_mlp.out_norm.bias")}
        chain = lambda prefix, n: [lin(f"{prefix}.layers.{j}.weight", f"{prefix}.layers.{j}.bias") for j in range(n)]
        heads = {"ref_point_head": chain("ddec.ref_point_head", 2), "bbox_embed": chain("ddec.bbox_embed", 3),
                 "presence_head": chain("ddec.presence_token_head", 3),
                 "prompt_mlp": chain("scoring.prompt_mlp", 2),
                 "rpb_x1": lin("ddec.boxRPB_embed_x.layers.1.weight", "ddec.boxRPB_embed_x.layers.1.bias"),
                 "rpb_y1": lin("ddec.boxRPB_embed_y.layers.1.weight", "ddec.boxRPB_embed_y.layers.1.bias"),
                 "prompt_proj": lin("scoring.prompt_proj.weight", "scoring.prompt_proj.bias"),
                 "hs_proj": lin("scoring.hs_proj.weight", "scoring.hs_proj.bias")}
        self.decoder = Decoder(hp.ddec_heads, hp.queries, layers, params, heads)
        # Segmentation head
        seg_params = {"cross_attn_norm_w": t("seg.cross_attn_norm.weight"),
                      "cross_attn_norm_b": t("seg.cross_attn_norm.bias"),
                      "conv_b": [t(f"seg.pixel_decoder.conv_layers.{i}.bias") for i in range(2)],
                      "norm_w": [t(f"seg.pixel_decoder.norms.{i}.weight") for i in range(2)],
                      "norm_b": [t(f"seg.pixel_decoder.norms.{i}.bias") for i in range(2)],
                      "instance_b": t("seg.instance_seg_head.bias")}
        convs = [self._dense(DENSE_CONV, tensors[f"seg.pixel_decoder.conv_layers.{i}.weight"]) for i in range(2)]
        self.seg = SegHead(hp.seg_heads, seg_params, convs,
                           self._dense(DENSE_CONV, tensors["seg.instance_seg_head.weight"]),
                           lin("seg.cross_attend_prompt.in_proj_weight", "seg.cross_attend_prompt.in_proj_bias"),
                           lin("seg.cross_attend_prompt.out_proj.weight", "seg.cross_attend_prompt.out_proj.bias"),
                           chain("seg.mask_predictor.mask_embed", 3))
        self._positions = {}

    # ---- weight loading --------------------------------------------------------
    def tensor(self, name: str):
        return self.torch.from_numpy(np.ascontiguousarray(self._t[name], dtype=np.float32)).to(self.dev)

    def quantized(self, name: str) -> Weights:
        q = self._t[name]
        if not isinstance(q, Quantized):
            raise TypeError(f"{name} must be a quantized linear on this path")
        w = Weights(q.qtype, q.k, q.n, q.rows, device=self.device)
        self._keep.append(w)
        return w

    def _dense(self, kind: int, w) -> Dense:
        d = Dense(kind, np.ascontiguousarray(w, dtype=np.float32), device=self.device)
        self._keep.append(d)
        return d

    def linear_pair(self, weight: str, bias: str):
        """(Weights or Dense, bias device tensor) for a module linear."""
        w = self._t[weight]
        handle = self.quantized(weight) if isinstance(w, Quantized) else self._dense(DENSE_LINEAR, w)
        return handle, self.tensor(bias)

    def norms(self, prefix: str, names) -> dict:
        out = {}
        for nm in names:
            out[nm + "_w"], out[nm + "_b"] = self.tensor(f"{prefix}.{nm}.weight"), self.tensor(f"{prefix}.{nm}.bias")
        return out

    def close(self):
        for h in self._keep:
            h.close()
        self._keep = []

    # ---- stages -------------------------------------------------------------------
    def position(self, grid: int):
        if grid not in self._positions:
            pe = sine_pe_2d(grid, grid, self.hp.neck_dim)
            self._positions[grid] = self.torch.from_numpy(pe).to(self.dev)
        return self._positions[grid]

    def encode_image(self, pixels, stream=None) -> ImageFeatures:
        """execution.hpp:55-120: ViT, neck (4x, 2x, 1x kept), positional
        encoding, geometry token.  pixels: [3][S][S] normalised, host or device."""
        torch, hp = self.torch, self.hp
        size, grid, E, D = hp.img_size, hp.grid, hp.embed, hp.neck_dim
        image = pixels if isinstance(pixels, torch.Tensor) else torch.from_numpy(np.ascontiguousarray(pixels))
        image = image.to(self.dev, non_blocking=True)
        x = torch.empty((grid * grid, E), device=self.dev)
        vit_prefix(image, size, size, hp.patch, self.patch_w, E, self.pos_embed, hp.pos_grid, self.ln_pre[0],
                   self.ln_pre[1], x, stream=stream, compute=self.compute)
        for blk in self.blocks:
            vit_block_forward(blk, x, grid, grid, stream=stream)
        maps = [torch.empty(((grid * s) ** 2 // 4, D), device=self.dev) for s in (8, 4, 2)]
        maps.append(torch.empty(((grid // 2) ** 2, D), device=self.dev))
        neck_forward(self.neck, x, grid, grid, maps, stream=stream)
        position = self.position(grid)
        geometry = torch.empty(D, device=self.dev)
        geometry_encoder_forward(self.geometry, maps[2], position, grid * grid, geometry, stream=stream)
        return ImageFeatures(maps[:3], position, geometry, grid)

    def encode_images(self, pixels, stream=None) -> list:
        """encode_image over a batch [B][3][S][S] (device): the 32 blocks run
        batched (samq_vit_block_forward_batch_v1, weights read once per block
        for the whole batch), the neck and geometry token per image."""
        torch, hp = self.torch, self.hp
        size, grid, E, D = hp.img_size, hp.grid, hp.embed, hp.neck_dim
        batch = pixels.shape[0]
        x = torch.empty((batch, grid * grid, E), device=self.dev)
        for b in range(batch):
            vit_prefix(pixels[b], size, size, hp.patch, self.patch_w, E, self.pos_embed, hp.pos_grid, self.ln_pre[0],
                       self.ln_pre[1], x[b], stream=stream, compute=self.compute)
        for blk in self.blocks:
            vit_block_forward(blk, x, grid, grid, stream=stream, batch=batch)
        position = self.position(grid)
        out = []
        for b in range(batch):
            maps = [torch.empty(((grid * s) ** 2 // 4, D), device=self.dev) for s in (8, 4, 2)]
            maps.append(torch.empty(((grid // 2) ** 2, D), device=self.dev))
            neck_forward(self.neck, x[b], grid, grid, maps, stream=stream)
            geometry = torch.empty(D, device=self.dev)
            geometry_encoder_forward(self.geometry, maps[2], position, grid * grid, geometry, stream=stream)
            out.append(ImageFeatures(maps[:3], position, geometry, grid))
        return out

    def encode_text(self, ids, stream=None):
        """execution.hpp:126-153: [ctx][256] text features."""
        torch, hp = self.torch, self.hp
        L, T = hp.ctx, hp.text_width
        ids = np.ascontiguousarray(ids, dtype=np.int32)
        x = torch.empty((L, T), device=self.dev)
        token_embed(self.token_table, hp.vocab, T, ids, self.text_pos, x, stream=stream)
        for blk in self.text_blocks:
            text_block_forward(blk, x, L, stream=stream)
        normed = torch.empty_like(x)
        layer_norm(x, L, T, T, self.ln_final[0], self.ln_final[1], normed, T, stream=stream)
        out = torch.empty((L, hp.neck_dim), device=self.dev)
        linear(self.resizer[0], normed, L, T, self.resizer[1], EPILOGUE_NONE, out, hp.neck_dim, stream=stream)
        return out

    def prompt_masks(self, ids):
        """The host half of prepare_prompt (execution.hpp:157-175): key bias 0 /
        -1e9 at padding ids, pooling weights (T + 1) / n_valid at valid tokens,
        the geometry token (last) valid; uploaded as device tensors."""
        torch, L = self.torch, self.hp.ctx
        ids = np.asarray(ids)
        valid_count = 1 + int(np.count_nonzero(ids[:L]))
        scale = np.float32(L + 1) / np.float32(valid_count)
        bias = np.append(np.where(ids[:L] != 0, 0.0, -1.0e9), 0.0).astype(np.float32)
        validity = np.append(np.where(ids[:L] != 0, scale, 0.0), scale).astype(np.float32)
        return torch.from_numpy(bias).to(self.dev), torch.from_numpy(validity).to(self.dev)

    def prepare_prompt(self, features: ImageFeatures, ids, text, masks=None) -> Prompt:
        """execution.hpp:157-175: tokens = [text; geometry] with prompt_masks."""
        bias, validity = self.prompt_masks(ids) if masks is None else masks
        tokens = self.torch.cat([text, features.geometry.view(1, -1)], dim=0).contiguous()
        return Prompt(tokens, bias, validity)

    def predict(self, features: ImageFeatures, ids, text, stream=None, masks=None) -> Prediction:
        """execution.hpp:241-324 (predict_joint): fusion -> decoder + scoring ->
        segmentation head.  With `masks` (prompt_masks(ids), computed once per
        prompt) it issues device work only, so it can be captured in a graph."""
        torch, hp = self.torch, self.hp
        grid, D, Q = features.grid, hp.neck_dim, hp.queries
        prompt = self.prepare_prompt(features, ids, text, masks)
        P = prompt.tokens.shape[0]
        fused = features.neck[2].clone()
        for layer in self.fusion:
            fusion_layer_forward(layer, fused, features.position, grid * grid, prompt.tokens, prompt.bias, P,
                                 stream=stream)
        queries = torch.empty((Q + 1, D), device=self.dev)
        boxes = torch.empty((Q, 4), device=self.dev)
        scores = torch.empty(Q, device=self.dev)
        presence = torch.empty(1, device=self.dev)
        decoder_forward(self.decoder, fused, features.position, grid, prompt.tokens, prompt.bias, prompt.validity, P,
                        queries, boxes, scores, presence, stream=stream)
        masks = torch.empty((Q, 16 * grid * grid), device=self.dev)
        seg_head_forward(self.seg, fused, grid, features.neck[0], features.neck[1], queries[1:], Q, prompt.tokens,
                         prompt.bias, P, masks, stream=stream)
        return Prediction(fused, queries, boxes, scores, presence, masks)


class ImagePathGraph:
    """encode_image + predict for one prompt, captured once as a CUDA graph.

    The image path issues ~400 kernel launches per image, most of them small
    (the decoder and fusion layers run on 201 queries / 33 prompt tokens), so
    on the host it is launch-bound; a graph replays the whole sequence with
    one launch.  Usage: copy the normalised pixels into `pixels`, call
    `replay()`; the results are in `prediction` (device tensors reused by
    every replay).  The library's per-stream scratch is sized by a warm-up
    run on the capture stream before capture, so no allocation happens while
    capturing; the text features and the prompt masks are computed outside."""

    def __init__(self, model: Sam3Image, ids, text):
        torch, hp = model.torch, model.hp
        self.model, self.torch = model, torch
        self.stream = torch.cuda.Stream(device=model.dev)
        self.pixels = torch.zeros((3, hp.img_size, hp.img_size), device=model.dev)
        self.text = text
        self.masks = model.prompt_masks(ids)
        self.ids = np.asarray(ids)
        self.stream.wait_stream(torch.cuda.current_stream(model.dev))
        with torch.cuda.stream(self.stream):
            self._run()
        self.stream.synchronize()
        self.graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(self.graph, stream=self.stream):
            self.features, self.prediction = self._run()

    def _run(self):
        feats = self.model.encode_image(self.pixels)
        return feats, self.model.predict(feats, self.ids, self.text, masks=self.masks)

    def replay(self):
        self.graph.replay()
