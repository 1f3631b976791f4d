"""End-to-end SAM 3 image path (config 4: the full-linear Q8_0 profile) on the
device through samq.sam3.Sam3Image (encode_image, encode_text, predict:
src/models/sam3/execution.hpp:55-343) against the oracle composed from the
same stages, on one random-init model and image at a 24 x 24 token grid
(336 x 336 pixels; every other dimension is SAM 3's: 32 ViT blocks, 24 text
blocks, 6 fusion and 6 decoder layers, 200 queries, mask logits at 96 x 96).

Why the bars are relative: every quantized linear re-stages its input to
Q8_1, and through the 6 decoder layers (and the 32 + 24 backbone and text
blocks) a difference at the f32 rounding level flips staging codes until the
drift saturates.  Measured on the oracle itself: 2^-22 relative noise on each
linear of the heads moves the mask logits by ~2% normalized L2 and the masks
(logit > 0) to IoU ~0.988, the same as the f16-operand gap of the device's
GEMM (oracle.exact_operands vs decoded operands).  So, for the mask logits:
  - heads from identical inputs (random neck maps and text features through
    the device's geometry encoder, fusion, decoder and segmentation head):
    normalized L2 to the oracle <= 1.5 x max(the oracle's noise drift, its
    f16-operand gap) and <= 0.05, IoU >= min(0.97, the yardstick's IoU -
    0.02), boxes within 1.5 x that yardstick's box distance + 1e-3;
  - the whole path from pixels and token ids: the same against the oracle's
    drift under noise on every linear of all stages, with the normalized L2
    capped at 0.15 (measured: device 0.074, IoU 0.958; the oracle under noise
    0.096, IoU 0.947 -- through 62 re-staged layers the drift is larger).
Per-stage figures are printed (pytest -s).
"""
import numpy as np
import pytest
import torch

import samq
from oracle import oracle as o
from samq import synthetic
from samq.sam3 import Sam3Image
from samq.synthetic import Quantized

pytestmark = pytest.mark.gpu
HP = synthetic.Hparams(img_size=336)


def _w(t, name):
    v = t[name]
    if isinstance(v, Quantized):
        return o.dequantize(v.qtype, v.rows, v.n * v.k).reshape(v.n, v.k), True, v
    return np.asarray(v, np.float32), False, None


def _lin(t, weight, bias):
    w, q, _ = _w(t, weight)
    return {"w": w, "b": np.asarray(t[bias], np.float32), "quantized": q}


def _norms(t, prefix, names):
    out = {}
    for nm in names:
        out[nm + "_w"], out[nm + "_b"] = t[f"{prefix}.{nm}.weight"], t[f"{prefix}.{nm}.bias"]
    return out


def oracle_model(t, hp):
    """The oracle's structures for every stage, from the GGUF-named tensors."""
    m = {"vit": [], "text": []}
    for i in range(hp.depth):
        p = f"vit.blocks.{i}"
        blk = {"window": hp.window_of(i), "freqs": t[p + ".attn.freqs_cis"]}
        for ours, name in (("qkv", ".attn.qkv"), ("proj", ".attn.proj"), ("fc1", ".mlp.lin1"), ("fc2", ".mlp.lin2")):
            w, _, q = _w(t, p + name + ".weight")
            blk[ours + "_w"], blk[ours + "_q"], blk[ours + "_b"] = w, (q.qtype, q.rows), t[p + name + ".bias"]
        blk.update(_norms(t, p, ("norm1", "norm2")))
        m["vit"].append(blk)
    from samq.sam3 import NECK_NAMES
    m["neck"] = {ours: (t[f"neck.det.{name}.weight"], t[f"neck.det.{name}.bias"]) for ours, name in NECK_NAMES.items()}
    for i in range(hp.text_layers):
        p = f"text.blocks.{i}"
        blk = {}
        for ours, name in (("in_proj", ".attn.in_proj"), ("out_proj", ".attn.out_proj"), ("fc1", ".mlp.fc1"),
                           ("fc2", ".mlp.fc2")):
            w, _, q = _w(t, p + name + ".weight")
            blk[ours + "_w"], blk[ours + "_q"], blk[ours + "_b"] = w, (q.qtype, q.rows), t[p + name + ".bias"]
        blk["norm1_w"], blk["norm1_b"] = t[p + ".ln_1.weight"], t[p + ".ln_1.bias"]
        blk["norm2_w"], blk["norm2_b"] = t[p + ".ln_2.weight"], t[p + ".ln_2.bias"]
        m["text"].append(blk)
    m["resizer"] = _w(t, "text.resizer.weight")[0]
    ge = {"cls": t["geom.cls_embed.weight"], "final_proj": _lin(t, "geom.final_proj.weight", "geom.final_proj.bias"),
          "norm_w": t["geom.norm.weight"], "norm_b": t["geom.norm.bias"],
          "encode_norm_w": t["geom.encode_norm.weight"], "encode_norm_b": t["geom.encode_norm.bias"], "layers": []}
    for i in range(hp.geom_layers):
        p = f"geom.layers.{i}"
        ly = {f"{a}_in_proj": _lin(t, f"{p}.{a}.in_proj_weight", f"{p}.{a}.in_proj_bias") for a in ("sa", "ca")}
        ly.update({f"{a}_out_proj": _lin(t, f"{p}.{a}.out_proj.weight", f"{p}.{a}.out_proj.bias") for a in ("sa", "ca")})
        ly["linear1"] = _lin(t, p + ".linear1.weight", p + ".linear1.bias")
        ly["linear2"] = _lin(t, p + ".linear2.weight", p + ".linear2.bias")
        ly.update(_norms(t, p, ("norm1", "norm2", "norm3")))
        ge["layers"].append(ly)
    m["geom"] = ge
    m["fusion"] = []
    for i in range(hp.fenc_layers):
        p = f"fenc.layers.{i}"
        ly = {f"{a}_in_proj": _lin(t, f"{p}.{a}.in_proj_weight", f"{p}.{a}.in_proj_bias") for a in ("sa", "ca")}
        ly.update({f"{a}_out_proj": _lin(t, f"{p}.{a}.out_proj.weight", f"{p}.{a}.out_proj.bias") for a in ("sa", "ca")})
        ly["linear1"] = _lin(t, p + ".linear1.weight", p + ".linear1.bias")
        ly["linear2"] = _lin(t, p + ".linear2.weight", p + ".linear2.bias")
        ly.update(_norms(t, p, ("norm1", "norm2", "norm3")))
        m["fusion"].append(ly)
    chain = lambda prefix, n: [_lin(t, f"{prefix}.layers.{j}.weight", f"{prefix}.layers.{j}.bias") for j in range(n)]
    dec = {"query_embed": t["ddec.query_embed.weight"], "presence_token": t["ddec.presence_token.weight"],
           "reference_points": t["ddec.reference_points.weight"],
           "rpb_x0_w": t["ddec.boxRPB_embed_x.layers.0.weight"], "rpb_x0_b": t["ddec.boxRPB_embed_x.layers.0.bias"],
           "rpb_y0_w": t["ddec.boxRPB_embed_y.layers.0.weight"], "rpb_y0_b": t["ddec.boxRPB_embed_y.layers.0.bias"],
           "rpb_x1": _lin(t, "ddec.boxRPB_embed_x.layers.1.weight", "ddec.boxRPB_embed_x.layers.1.bias"),
           "rpb_y1": _lin(t, "ddec.boxRPB_embed_y.layers.1.weight", "ddec.boxRPB_embed_y.layers.1.bias"),
           "norm_w": t["ddec.norm.weight"], "norm_b": t["ddec.norm.bias"],
           "presence_norm_w": t["ddec.presence_token_out_norm.weight"],
           "presence_norm_b": t["ddec.presence_token_out_norm.bias"],
           "prompt_mlp_norm_w": t["scoring.prompt_mlp.out_norm.weight"],
           "prompt_mlp_norm_b": t["scoring.prompt_mlp.out_norm.bias"],
           "ref_point_head": chain("ddec.ref_point_head", 2), "bbox_embed": chain("ddec.bbox_embed", 3),
           "presence_head": chain("ddec.presence_token_head", 3), "prompt_mlp": chain("scoring.prompt_mlp", 2),
           "prompt_proj": _lin(t, "scoring.prompt_proj.weight", "scoring.prompt_proj.bias"),
           "hs_proj": _lin(t, "scoring.hs_proj.weight", "scoring.hs_proj.bias"), "layers": []}
    for i in range(hp.ddec_layers):
        p = f"ddec.layers.{i}"
        ly = {f"{a}_in_proj": _lin(t, f"{p}.{a}.in_proj_weight", f"{p}.{a}.in_proj_bias") for a in ("sa", "ca", "ca_text")}
        ly.update({f"{a}_out_proj": _lin(t, f"{p}.{a}.out_proj.weight", f"{p}.{a}.out_proj.bias")
                   for a in ("sa", "ca", "ca_text")})
        ly["linear1"] = _lin(t, p + ".linear1.weight", p + ".linear1.bias")
        ly["linear2"] = _lin(t, p + ".linear2.weight", p + ".linear2.bias")
        ly.update(_norms(t, p, ("norm1", "norm2", "norm_ca_text", "norm3")))
        dec["layers"].append(ly)
    m["dec"] = dec
    m["seg"] = {"cross_attn_norm_w": t["seg.cross_attn_norm.weight"], "cross_attn_norm_b": t["seg.cross_attn_norm.bias"],
                "ca_in_proj": _lin(t, "seg.cross_attend_prompt.in_proj_weight", "seg.cross_attend_prompt.in_proj_bias"),
                "ca_out_proj": _lin(t, "seg.cross_attend_prompt.out_proj.weight",
                                    "seg.cross_attend_prompt.out_proj.bias"),
                "conv_w": [t[f"seg.pixel_decoder.conv_layers.{i}.weight"] for i in range(2)],
                "conv_b": [t[f"seg.pixel_decoder.conv_layers.{i}.bias"] for i in range(2)],
                "norm_w": [t[f"seg.pixel_decoder.norms.{i}.weight"] for i in range(2)],
                "norm_b": [t[f"seg.pixel_decoder.norms.{i}.bias"] for i in range(2)],
                "instance_w": t["seg.instance_seg_head.weight"], "instance_b": t["seg.instance_seg_head.bias"],
                "mask_embed": chain("seg.mask_predictor.mask_embed", 3)}
    return m


def oracle_prompt(hp, ids):
    L = hp.ctx
    valid = 1 + int(np.count_nonzero(ids[:L]))
    scale = np.float32(L + 1) / np.float32(valid)
    bias = np.append(np.where(ids[:L] != 0, 0.0, -1.0e9), 0.0).astype(np.float32)
    validity = np.append(np.where(ids[:L] != 0, scale, 0.0), scale).astype(np.float32)
    return bias, validity


def oracle_heads(m, hp, neck, text, ids):
    """Geometry, fusion, decoder and segmentation head from given neck maps
    (f32 [pixels][D] at 4x, 2x, 1x) and text features."""
    grid, D = hp.grid, hp.neck_dim
    pos = o.sine_pe_2d(grid, grid, D)
    geo = o.geometry_encoder(neck[2], pos, m["geom"], hp.fenc_heads)
    prompt = np.concatenate([np.asarray(text, np.float32), geo], axis=0)
    bias, validity = oracle_prompt(hp, ids)
    x = np.asarray(neck[2], np.float32)
    for ly in m["fusion"]:
        x = o.fusion_layer(x, pos, prompt, bias, ly, hp.fenc_heads)
    queries, boxes, scores, presence = o.decoder(x, pos, prompt, bias, validity, m["dec"], grid, hp.ddec_heads)
    masks = o.seg_head(x, neck[0], neck[1], queries[1:], prompt, bias, m["seg"], grid, hp.seg_heads)
    return {"fusion": x, "boxes": boxes, "scores": scores, "presence": presence, "masks": masks}


def oracle_backbone(m, t, hp, pixels, ids):
    x = o.vit_prefix(pixels, hp.patch, t["vit.patch_embed.proj.weight"], t["vit.pos_embed"], t["vit.ln_pre.weight"],
                     t["vit.ln_pre.bias"])
    for blk in m["vit"]:
        x = o.vit_block(x, blk, hp.grid, hp.grid)
    g = hp.grid
    maps = o.neck(x.reshape(g, g, hp.embed), m["neck"])
    neck = [np.asarray(mp, np.float64).reshape(-1, hp.neck_dim).astype(np.float32) for mp in maps[:3]]
    text = o.text_encoder(ids, t["text.token_embed.weight"], t["text.pos_embed"], m["text"], t["text.ln_final.weight"],
                          t["text.ln_final.bias"], m["resizer"], t["text.resizer.bias"])
    return neck, text


def _nl2(a, b):
    a, b = np.asarray(a, np.float64), np.asarray(b, np.float64)
    return float(np.linalg.norm(a - b) / np.linalg.norm(b))


def _iou(a, b):
    ma, mb = np.asarray(a) > 0, np.asarray(b) > 0
    union = np.count_nonzero(ma | mb)
    return 1.0 if union == 0 else np.count_nonzero(ma & mb) / union


@pytest.fixture(scope="module")
def case():
    tensors = synthetic.sam3_tensors(HP, "q8_0", seed=11)
    model = Sam3Image(tensors, HP)
    pixels = synthetic.image(HP, 12)
    ids = synthetic.token_ids(HP, 13, length=20)
    m = oracle_model(tensors, HP)
    yield tensors, model, pixels, ids, m
    model.close()


def _device_heads(model, neck, text, ids):
    dev = model.dev
    grid = HP.grid
    maps = [torch.from_numpy(np.ascontiguousarray(mp, np.float32)).to(dev) for mp in neck]
    position = model.position(grid)
    geometry = torch.empty(HP.neck_dim, device=dev)
    samq.geometry_encoder_forward(model.geometry, maps[2], position, grid * grid, geometry)
    from samq.sam3 import ImageFeatures
    feats = ImageFeatures(maps, position, geometry, grid)
    pred = model.predict(feats, ids, torch.from_numpy(np.asarray(text, np.float32)).to(dev))
    samq.check(0)
    return {"fusion": pred.fusion.cpu().numpy(), "boxes": pred.boxes.cpu().numpy(),
            "scores": pred.class_logits.cpu().numpy(), "presence": float(pred.presence_logit.cpu().numpy()[0]),
            "masks": pred.mask_logits.cpu().numpy()}


def _report(tag, got, ref):
    r = {"fusion_nl2": _nl2(got["fusion"], ref["fusion"]),
         "boxes_max": float(np.abs(got["boxes"] - ref["boxes"]).max()),
         "scores_max": float(np.abs(got["scores"] - ref["scores"]).max()),
         "presence": abs(got["presence"] - ref["presence"]),
         "masks_rel_max": float(np.abs(got["masks"] - ref["masks"]).max() / np.abs(ref["masks"]).max()),
         "masks_mean_abs": float(np.abs(got["masks"] - ref["masks"]).mean() / np.abs(ref["masks"]).mean()),
         "masks_nl2": _nl2(got["masks"], ref["masks"]), "iou": _iou(got["masks"], ref["masks"])}
    print(tag, {k: round(v, 6) for k, v in r.items()})
    return r


def _noise_drift(fn, ref, seed):
    """The oracle's own distance from `ref` with 2^-22 relative noise on the
    output of every quantized linear (fn re-runs the oracle)."""
    keep = o.staged_linear
    noise_rng = np.random.default_rng(seed)

    def noisy(w, v, bias=None, epilogue=o.EPILOGUE_NONE):
        y = keep(w, v, bias, epilogue).astype(np.float64)
        return (y * (1 + 2.0 ** -22 * noise_rng.standard_normal(y.shape))).astype(np.float32)
    o.staged_linear = noisy
    try:
        return _report("oracle under f32-level noise vs oracle", fn(), ref)
    finally:
        o.staged_linear = keep


def _check(r, yard, nl2_cap):
    assert r["iou"] >= min(0.97, yard["iou"] - 0.02), (r, yard)
    assert r["masks_nl2"] <= nl2_cap and r["masks_nl2"] <= 1.5 * max(yard["masks_nl2"], 1e-3), (r, yard)
    assert r["boxes_max"] <= 1.5 * yard["boxes_max"] + 1e-3, (r, yard)


def test_heads_from_identical_inputs(case):
    tensors, model, pixels, ids, m = case
    rng = np.random.default_rng(5)
    g, D = HP.grid, HP.neck_dim
    neck = [rng.standard_normal((n, D)).astype(np.float32) for n in (16 * g * g, 4 * g * g, g * g)]
    text = rng.standard_normal((HP.ctx, D)).astype(np.float32)
    got = _device_heads(model, neck, text, ids)
    sem = oracle_heads(m, HP, neck, text, ids)
    with o.exact_operands():
        exact = oracle_heads(m, HP, neck, text, ids)
    _report("heads vs exact-operand oracle", got, exact)
    r = _report("heads vs decoded-operand oracle", got, sem)
    gap = _report("exact-operand vs decoded-operand oracle", exact, sem)
    drift = _noise_drift(lambda: oracle_heads(m, HP, neck, text, ids), sem, 6)
    yard = {k: max(gap[k], drift[k]) for k in ("masks_nl2", "boxes_max")}
    yard["iou"] = min(gap["iou"], drift["iou"])
    _check(r, yard, 0.05)


def test_end_to_end_from_pixels(case):
    tensors, model, pixels, ids, m = case
    feats = model.encode_image(pixels)
    text = model.encode_text(ids)
    pred = model.predict(feats, ids, text)
    samq.check(0)
    got = {"fusion": pred.fusion.cpu().numpy(), "boxes": pred.boxes.cpu().numpy(),
           "scores": pred.class_logits.cpu().numpy(), "presence": float(pred.presence_logit.cpu().numpy()[0]),
           "masks": pred.mask_logits.cpu().numpy()}
    neck, txt = oracle_backbone(m, tensors, HP, pixels, ids)
    print("neck 1x nl2", _nl2(feats.neck[2].cpu().numpy(), neck[2]), "text nl2", _nl2(text.cpu().numpy(), txt))
    ref = oracle_heads(m, HP, neck, txt, ids)
    r = _report("end to end vs oracle", got, ref)

    def rerun():
        nneck, ntxt = oracle_backbone(m, tensors, HP, pixels, ids)
        return oracle_heads(m, HP, nneck, ntxt, ids)
    drift = _noise_drift(rerun, ref, 21)
    _check(r, drift, 0.15)


def test_image_path_graph_matches_eager(case):
    """ImagePathGraph (encode_image + predict captured as one CUDA graph)
    replays the same kernels in the same order: identical bits to the eager
    calls, on two different images through the same graph."""
    from samq.sam3 import ImagePathGraph
    tensors, model, pixels, ids, m = case
    text = model.encode_text(ids)
    graph = ImagePathGraph(model, ids, text)
    for seed in (12, 14):
        img = torch.from_numpy(synthetic.image(HP, seed)).cuda()
        feats = model.encode_image(img)
        eager = model.predict(feats, ids, text)
        graph.pixels.copy_(img)
        graph.replay()
        torch.cuda.synchronize()
        samq.check(0)
        for name in ("mask_logits", "boxes", "class_logits", "presence_logit", "queries"):
            a, b = getattr(eager, name), getattr(graph.prediction, name)
            assert torch.equal(a, b), (seed, name, float((a - b).abs().max()))
