"""Python binding of libsamq (include/samq.h) for tests, benchmarks and scripts.

The binding is a thin ctypes layer over the C ABI: every call goes to the
sm_100a kernels in ``libsamq.so``.  There is no fallback of any kind: when the
library is missing this module raises at import of the first call, and a
non-sm_100 device is rejected by the library itself.

Device buffers and streams may be given as torch tensors / torch streams or
as raw integer addresses.
"""
from __future__ import annotations

import ctypes
import os
from pathlib import Path

import numpy as np

PACKAGE_DIR = Path(__file__).resolve().parent.parent
LIB_PATH = Path(os.environ.get("SAMQ_LIBRARY", PACKAGE_DIR / "libsamq.so"))

Q8_0, Q8_1, Q4_K, Q5_K, Q6_K = 8, 9, 12, 13, 14
TYPE_NAMES = {Q8_0: "Q8_0", Q4_K: "Q4_K", Q5_K: "Q5_K", Q6_K: "Q6_K"}
NAME_TYPES = {v: k for k, v in TYPE_NAMES.items()}
EPILOGUE_NONE, EPILOGUE_GELU_ERF = 0, 1
F32, F16 = 0, 1
DENSE_LINEAR, DENSE_CONV, DENSE_DECONV2X2 = 0, 1, 2
COMPUTE_F32, COMPUTE_F16 = 0, 1  # sam::CudaComputeMode (default F32)
BLOCK = {Q8_0: (32, 34), Q4_K: (256, 144), Q5_K: (256, 176), Q6_K: (256, 210)}

STATUS_NAMES = {
    0: "SAMQ_OK", 1: "SAMQ_ERR_INVALID_ARGUMENT", 2: "SAMQ_ERR_UNSUPPORTED", 3: "SAMQ_ERR_CUDA",
    4: "SAMQ_ERR_OUT_OF_MEMORY", 5: "SAMQ_ERR_RANGE", 6: "SAMQ_ERR_TIMEOUT", 7: "SAMQ_ERR_PAYLOAD",
}

# Every symbol include/samq.h declares, with its ctypes signature.
_i64, _i32, _vp, _sz = ctypes.c_int64, ctypes.c_int, ctypes.c_void_p, ctypes.c_size_t


class Capabilities(ctypes.Structure):
    _fields_ = [("version", ctypes.c_uint32), ("device", ctypes.c_int32), ("cc_major", ctypes.c_int32),
                ("cc_minor", ctypes.c_int32), ("sm_count", ctypes.c_int32),
                ("global_memory_bytes", ctypes.c_uint64), ("max_shared_memory_per_block", ctypes.c_uint64),
                ("name", ctypes.c_char * 256)]


class Counters(ctypes.Structure):
    _fields_ = [("version", ctypes.c_uint32), ("path", ctypes.c_uint32), ("launches", ctypes.c_uint64),
                ("payload_bytes", ctypes.c_uint64), ("allocation_bytes", ctypes.c_uint64),
                ("weight_bytes", ctypes.c_uint64)]


class VitBlockDesc(ctypes.Structure):
    """struct samq_vit_block_v1."""
    _fields_ = [("version", ctypes.c_uint32), ("window", ctypes.c_int32), ("norm1_w", _vp), ("norm1_b", _vp),
                ("qkv", _vp), ("qkv_b", _vp), ("proj", _vp), ("proj_b", _vp), ("norm2_w", _vp), ("norm2_b", _vp),
                ("fc1", _vp), ("fc1_b", _vp), ("fc2", _vp), ("fc2_b", _vp), ("freqs_cis", _vp),
                ("compute", ctypes.c_int32)]


class TextBlockDesc(ctypes.Structure):
    """struct samq_text_block_v1."""
    _fields_ = [("version", ctypes.c_uint32), ("norm1_w", _vp), ("norm1_b", _vp), ("in_proj", _vp),
                ("in_proj_b", _vp), ("out_proj", _vp), ("out_proj_b", _vp), ("norm2_w", _vp), ("norm2_b", _vp),
                ("fc1", _vp), ("fc1_b", _vp), ("fc2", _vp), ("fc2_b", _vp)]


class LinearRef(ctypes.Structure):
    """struct samq_linear_ref_v1."""
    _fields_ = [("quantized", _vp), ("dense", _vp), ("bias", _vp)]


class FusionLayerDesc(ctypes.Structure):
    """struct samq_fusion_layer_v1."""
    _fields_ = [("version", ctypes.c_uint32), ("heads", ctypes.c_int32)] + \
        [(n, _vp) for n in ("norm1_w", "norm1_b", "norm2_w", "norm2_b", "norm3_w", "norm3_b")] + \
        [(n, LinearRef) for n in ("sa_in_proj", "sa_out_proj", "ca_in_proj", "ca_out_proj", "linear1", "linear2")]


DECODER_LAYER_LINEARS = ("sa_in_proj", "sa_out_proj", "ca_text_in_proj", "ca_text_out_proj", "ca_in_proj",
                         "ca_out_proj", "linear1", "linear2")
DECODER_LAYER_NORMS = ("norm1_w", "norm1_b", "norm2_w", "norm2_b", "norm_ca_text_w", "norm_ca_text_b", "norm3_w",
                       "norm3_b")


class DecoderLayerDesc(ctypes.Structure):
    """struct samq_decoder_layer_v1."""
    _fields_ = [(n, LinearRef) for n in DECODER_LAYER_LINEARS] + [(n, _vp) for n in DECODER_LAYER_NORMS]


class DecoderDesc(ctypes.Structure):
    """struct samq_decoder_v1."""
    _fields_ = [("version", ctypes.c_uint32), ("heads", ctypes.c_int32), ("layers", ctypes.c_int32),
                ("queries", ctypes.c_int32), ("layer", ctypes.POINTER(DecoderLayerDesc)),
                ("query_embed", _vp), ("presence_token", _vp), ("reference_points", _vp),
                ("ref_point_head", LinearRef * 2), ("bbox_embed", LinearRef * 3),
                ("rpb_x0_w", _vp), ("rpb_x0_b", _vp), ("rpb_y0_w", _vp), ("rpb_y0_b", _vp),
                ("rpb_x1", LinearRef), ("rpb_y1", LinearRef), ("norm_w", _vp), ("norm_b", _vp),
                ("presence_norm_w", _vp), ("presence_norm_b", _vp), ("presence_head", LinearRef * 3),
                ("prompt_mlp", LinearRef * 2), ("prompt_mlp_norm_w", _vp), ("prompt_mlp_norm_b", _vp),
                ("prompt_proj", LinearRef), ("hs_proj", LinearRef)]


GEOMETRY_LAYER_LINEARS = ("sa_in_proj", "sa_out_proj", "ca_in_proj", "ca_out_proj", "linear1", "linear2")
GEOMETRY_LAYER_NORMS = ("norm1_w", "norm1_b", "norm2_w", "norm2_b", "norm3_w", "norm3_b")


class GeometryLayerDesc(ctypes.Structure):
    """struct samq_geometry_layer_v1."""
    _fields_ = [(n, LinearRef) for n in GEOMETRY_LAYER_LINEARS] + [(n, _vp) for n in GEOMETRY_LAYER_NORMS]


class GeometryEncoderDesc(ctypes.Structure):
    """struct samq_geometry_encoder_v1."""
    _fields_ = [("version", ctypes.c_uint32), ("heads", ctypes.c_int32), ("layers", ctypes.c_int32),
                ("layer", ctypes.POINTER(GeometryLayerDesc)), ("cls_token", _vp), ("final_proj", LinearRef),
                ("norm_w", _vp), ("norm_b", _vp), ("encode_norm_w", _vp), ("encode_norm_b", _vp)]


class SegHeadDesc(ctypes.Structure):
    """struct samq_seg_head_v1."""
    _fields_ = [("version", ctypes.c_uint32), ("heads", ctypes.c_int32), ("cross_attn_norm_w", _vp),
                ("cross_attn_norm_b", _vp), ("ca_in_proj", LinearRef), ("ca_out_proj", LinearRef),
                ("conv", _vp * 2), ("conv_b", _vp * 2), ("norm_w", _vp * 2), ("norm_b", _vp * 2),
                ("instance", _vp), ("instance_b", _vp), ("mask_embed", LinearRef * 3)]


class NeckDesc(ctypes.Structure):
    """struct samq_neck_v1: (weights, bias) pairs in the order of NECK_LAYERS."""
    _fields_ = [("version", ctypes.c_uint32)] + [
        (f"{name}{suffix}", _vp) for name in ("s0_deconv1", "s0_deconv2", "s0_conv1x1", "s0_conv3x3", "s1_deconv1",
                                              "s1_conv1x1", "s1_conv3x3", "s2_conv1x1", "s2_conv3x3", "s3_conv1x1",
                                              "s3_conv3x3") for suffix in ("", "_b")]


NECK_LAYERS = ("s0_deconv1", "s0_deconv2", "s0_conv1x1", "s0_conv3x3", "s1_deconv1", "s1_conv1x1", "s1_conv3x3",
               "s2_conv1x1", "s2_conv3x3", "s3_conv1x1", "s3_conv3x3")

SIGNATURES = {
    "samq_last_error_v1": (ctypes.c_char_p, []),
    "samq_init_v1": (_i32, [_i32]),
    "samq_capabilities_v1": (_i32, [_i32, ctypes.POINTER(Capabilities)]),
    "samq_weights_create_v1": (_i32, [_i32, _i32, _i64, _i64, _vp, _sz, _vp, ctypes.POINTER(_vp)]),
    "samq_weights_destroy_v1": (_i32, [_vp]),
    "samq_weights_export_v1": (_i32, [_vp, _vp, _sz]),
    "samq_weights_packets_v1": (_i32, [_vp, ctypes.POINTER(_vp), ctypes.POINTER(_sz)]),
    "samq_quantize_q8_1_v1": (_i32, [_vp, _i64, _i64, _i64, _vp, _vp]),
    "samq_mmq_d4_bytes_v1": (_sz, [_i64, _i64]),
    "samq_quantize_mmq_q8_1_v1": (_i32, [_vp, _i64, _i64, _i64, _vp, _vp]),
    "samq_linear_v1": (_i32, [_vp, _vp, _i64, _i64, _vp, _i32, _vp, _i64, _vp]),
    "samq_linear_q8_1_v1": (_i32, [_vp, _vp, _i64, _vp, _i32, _vp, _i64, _vp]),
    "samq_stage_f16_v1": (_i32, [_vp, _i64, _i64, _i64, _vp, _vp]),
    "samq_linear_f16_v1": (_i32, [_vp, _vp, _i64, _i64, _vp, _i32, _vp, _i64, _vp]),
    "samq_query_v1": (_i32, [_vp, ctypes.POINTER(Counters)]),
    "samq_check_v1": (_i32, [_i32, _vp]),
    "samq_linear_static_v1": (_i32, [_vp, _vp, _i64, _i64, _vp, _i32, _vp, _i64, _vp]),
    "samq_vit_attention_v1": (_i32, [_vp, _i64, _i32, _i32, _i32, _i32, _i32, _vp, _vp, _i64, _vp]),
    "samq_vit_attention_v2": (_i32, [_vp, _i64, _i32, _i32, _i32, _i32, _i32, _vp, _vp, _i64, _i32, _vp]),
    "samq_vit_rope_v1": (_i32, [_vp, _i64, _i64, _i32, _vp, _vp, _vp]),
    "samq_vit_prefix_v2": (_i32, [_vp, _i32, _i32, _i32, _vp, _i64, _vp, _i32, _vp, _vp, _vp, _i32, _vp]),
    "samq_vit_block_forward_v1": (_i32, [ctypes.POINTER(VitBlockDesc), _vp, _i32, _i32, _vp]),
    "samq_vit_block_forward_batch_v1": (_i32, [ctypes.POINTER(VitBlockDesc), _vp, _i32, _i32, _i32, _vp]),
    "samq_vit_prefix_v1": (_i32, [_vp, _i32, _i32, _i32, _vp, _i64, _vp, _i32, _vp, _vp, _vp, _vp]),
    "samq_text_block_forward_v1": (_i32, [ctypes.POINTER(TextBlockDesc), _vp, _i32, _vp]),
    "samq_token_embed_v1": (_i32, [_vp, _i64, _i32, _vp, _i32, _vp, _vp, _vp]),
    "samq_layer_norm_v1": (_i32, [_vp, _i64, _i32, _i64, _vp, _vp, ctypes.c_float, _vp, _i64, _vp]),
    "samq_attention_v1": (_i32, [_vp, _i64, _vp, _i64, _vp, _i64, _i32, _i32, _i32, _i32, ctypes.c_float, _i32, _vp,
                                 _i64, _i64, _vp, _i64, _vp]),
    "samq_fusion_layer_forward_v1": (_i32, [ctypes.POINTER(FusionLayerDesc), _vp, _vp, _i32, _vp, _vp, _i32, _vp]),
    "samq_decoder_forward_v1": (_i32, [ctypes.POINTER(DecoderDesc), _vp, _vp, _i32, _vp, _vp, _vp, _i32, _vp, _vp,
                                       _vp, _vp, _vp]),
    "samq_geometry_encoder_forward_v1": (_i32, [ctypes.POINTER(GeometryEncoderDesc), _vp, _vp, _i32, _vp, _vp]),
    "samq_seg_head_forward_v1": (_i32, [ctypes.POINTER(SegHeadDesc), _vp, _i32, _vp, _vp, _vp, _i32, _vp, _vp, _i32,
                                        _vp, _vp]),
    "samq_sine_pe_2d_v1": (_i32, [_i32, _i32, _i32, _vp]),
    "samq_quantize_rows_v1": (_i32, [_i32, _i64, _i64, _vp, _vp, _sz]),
    "samq_mmq_weights_create_v1": (_i32, [_i32, _i32, _i32, _i64, _i64, _vp, _sz, _vp, ctypes.POINTER(_vp)]),
    "samq_mmq_weights_destroy_v1": (_i32, [_vp]),
    "samq_linear_mmq_v1": (_i32, [_vp, _vp, _i64, _i64, _vp, _i32, _vp, _i64, _vp]),
    "samq_dense_create_v1": (_i32, [_i32, _i32, _i32, _i32, _i32, _i64, _i64, _vp, _sz, _vp, ctypes.POINTER(_vp)]),
    "samq_dense_destroy_v1": (_i32, [_vp]),
    "samq_dense_linear_v1": (_i32, [_vp, _vp, _i64, _i64, _vp, _i32, _vp, _i64, _vp]),
    "samq_conv2d_v1": (_i32, [_vp, _vp, _i32, _i32, _vp, _i32, _vp, _vp]),
    "samq_maxpool2x2_v1": (_i32, [_vp, _i32, _i32, _i64, _vp, _vp]),
    "samq_neck_forward_v1": (_i32, [ctypes.POINTER(NeckDesc), _vp, _i32, _i32, ctypes.POINTER(_vp), _vp]),
}
STATIC_OPERAND_ELEMENTS = 16777216


class SamqError(RuntimeError):
    def __init__(self, status: int, message: str):
        self.status = status
        super().__init__(f"{STATUS_NAMES.get(status, status)}: {message}")


_lib = None


def library() -> ctypes.CDLL:
    """Load libsamq.so (raises if it has not been built)."""
    global _lib
    if _lib is None:
        if not LIB_PATH.exists():
            raise ImportError(f"{LIB_PATH} is missing; build it with `make -C {PACKAGE_DIR}` "
                              "(there is no non-CUDA fallback)")
        lib = ctypes.CDLL(str(LIB_PATH))
        for name, (res, args) in SIGNATURES.items():
            fn = getattr(lib, name)
            fn.restype = res
            fn.argtypes = args
        _lib = lib
    return _lib


def _check(status: int):
    if status != 0:
        raise SamqError(status, library().samq_last_error_v1().decode())


def _addr(obj) -> int | None:
    """Device address of a torch tensor / int / None."""
    if obj is None:
        return None
    if isinstance(obj, int):
        return obj
    if hasattr(obj, "data_ptr"):
        return obj.data_ptr()
    raise TypeError(f"expected a device tensor or address, got {type(obj)!r}")


def _stream(stream) -> int | None:
    if stream is None:
        try:
            import torch
            if torch.cuda.is_available():
                return torch.cuda.current_stream().cuda_stream
        except ImportError:
            pass
        return None
    if isinstance(stream, int):
        return stream
    return stream.cuda_stream


def init(device: int = 0):
    _check(library().samq_init_v1(device))


def capabilities(device: int = 0) -> Capabilities:
    info = Capabilities()
    _check(library().samq_capabilities_v1(device, ctypes.byref(info)))
    return info


def row_bytes(qtype: int, k: int) -> int:
    be, bb = BLOCK[qtype]
    if k % be:
        raise ValueError("width is not block aligned")
    return k // be * bb


class Weights:
    """A repacked weight matrix resident on one device (samq_weights*)."""

    def __init__(self, qtype: int, k: int, n: int, gguf_rows: np.ndarray, device: int = 0, stream=None):
        rows = np.ascontiguousarray(gguf_rows, dtype=np.uint8).reshape(-1)
        handle = ctypes.c_void_p()
        _check(library().samq_weights_create_v1(device, qtype, k, n, rows.ctypes.data, rows.nbytes,
                                                _stream(stream), ctypes.byref(handle)))
        self.handle = handle
        self.qtype, self.k, self.n, self.device = qtype, k, n, device

    def close(self):
        if self.handle:
            _check(library().samq_weights_destroy_v1(self.handle))
            self.handle = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def export(self) -> np.ndarray:
        out = np.empty(self.n * row_bytes(self.qtype, self.k), dtype=np.uint8)
        _check(library().samq_weights_export_v1(self.handle, out.ctypes.data, out.nbytes))
        return out

    def packets(self) -> tuple[int, int]:
        ptr, size = ctypes.c_void_p(), ctypes.c_size_t()
        _check(library().samq_weights_packets_v1(self.handle, ctypes.byref(ptr), ctypes.byref(size)))
        return ptr.value, size.value

    def query(self) -> Counters:
        c = Counters()
        _check(library().samq_query_v1(self.handle, ctypes.byref(c)))
        return c


def quantize_q8_1(x, rows: int, k: int, ld: int, out, stream=None):
    _check(library().samq_quantize_q8_1_v1(_addr(x), rows, k, ld, _addr(out), _stream(stream)))


def mmq_d4_bytes(rows: int, k: int) -> int:
    return library().samq_mmq_d4_bytes_v1(rows, k)


def quantize_mmq_q8_1(x, rows: int, k: int, ld: int, out, stream=None):
    _check(library().samq_quantize_mmq_q8_1_v1(_addr(x), rows, k, ld, _addr(out), _stream(stream)))


def linear(w: Weights, x, m: int, ldx: int, bias, epilogue: int, y, ldy: int, stream=None):
    _check(library().samq_linear_v1(w.handle, _addr(x), m, ldx, _addr(bias), epilogue, _addr(y), ldy,
                                    _stream(stream)))


def linear_q8_1(w: Weights, xq, m: int, bias, epilogue: int, y, ldy: int, stream=None):
    _check(library().samq_linear_q8_1_v1(w.handle, _addr(xq), m, _addr(bias), epilogue, _addr(y), ldy,
                                         _stream(stream)))


def stage_f16(x, rows: int, k: int, ld: int, out, stream=None):
    _check(library().samq_stage_f16_v1(_addr(x), rows, k, ld, _addr(out), _stream(stream)))


def linear_f16(w: Weights, x16, m: int, ldx: int, bias, epilogue: int, y, ldy: int, stream=None):
    _check(library().samq_linear_f16_v1(w.handle, _addr(x16), m, ldx, _addr(bias), epilogue, _addr(y), ldy,
                                        _stream(stream)))


def linear_static(w: Weights, x, m: int, ldx: int, bias, epilogue: int, y, ldy: int, stream=None):
    """samq_linear_static_v1: samq_linear_v1 without any device allocation."""
    _check(library().samq_linear_static_v1(w.handle, _addr(x), m, ldx, _addr(bias), epilogue, _addr(y), ldy,
                                           _stream(stream)))


def vit_attention(qkv, ldq: int, grid_w: int, grid_h: int, heads: int, window: int, freqs, out, ldo: int,
                  stream=None, head_dim: int = 64, compute: int = COMPUTE_F32):
    """samq_vit_attention_v2: RoPE + windowed (window > 0) or global attention,
    F32-precise (COMPUTE_F32, the reference's default) or on f16 tensor-core
    operands (COMPUTE_F16)."""
    _check(library().samq_vit_attention_v2(_addr(qkv), ldq, grid_w, grid_h, heads, head_dim, window, _addr(freqs),
                                           _addr(out), ldo, compute, _stream(stream)))


def vit_rope(x, tokens: int, head_batches: int, freqs, out, stream=None, head_dim: int = 64):
    """samq_vit_rope_v1: sam3_apply_rope on [head_batches][tokens][64] f32."""
    _check(library().samq_vit_rope_v1(_addr(x), tokens, head_batches, head_dim, _addr(freqs), _addr(out),
                                      _stream(stream)))


def check(device: int = 0, stream=None):
    _check(library().samq_check_v1(device, _stream(stream)))


class VitBlock:
    """One ViT block's device parameters (samq_vit_block_v1).

    The f32 parameters are device tensors (kept alive here); the four linears
    are Weights handles.  window is 24 for windowed blocks and 0 for global
    ones; freqs is [positions][32][2] (cos, sin); compute is COMPUTE_F32 (the
    reference's default: f32 qkv and F32-precise attention) or COMPUTE_F16."""

    def __init__(self, window: int, norm1_w, norm1_b, qkv: Weights, qkv_b, proj: Weights, proj_b, norm2_w, norm2_b,
                 fc1: Weights, fc1_b, fc2: Weights, fc2_b, freqs, compute: int = COMPUTE_F32):
        self._keep = (norm1_w, norm1_b, qkv, qkv_b, proj, proj_b, norm2_w, norm2_b, fc1, fc1_b, fc2, fc2_b, freqs)
        self.window = window
        self.compute = compute
        self.desc = VitBlockDesc(2, window, _addr(norm1_w), _addr(norm1_b), qkv.handle, _addr(qkv_b), proj.handle,
                                 _addr(proj_b), _addr(norm2_w), _addr(norm2_b), fc1.handle, _addr(fc1_b), fc2.handle,
                                 _addr(fc2_b), _addr(freqs), compute)


def vit_block_forward(block: VitBlock, x, grid_w: int, grid_h: int, stream=None, batch: int = 1):
    """samq_vit_block_forward_v1 (batch 1) / samq_vit_block_forward_batch_v1: one
    pre-LN ViT block in place on x [batch][tokens][E] f32."""
    if batch == 1:
        _check(library().samq_vit_block_forward_v1(ctypes.byref(block.desc), _addr(x), grid_w, grid_h,
                                                   _stream(stream)))
    else:
        _check(library().samq_vit_block_forward_batch_v1(ctypes.byref(block.desc), _addr(x), batch, grid_w, grid_h,
                                                         _stream(stream)))


def vit_prefix(image, width: int, height: int, patch: int, patch_w, embed: int, pos_embed, pos_grid: int, ln_w, ln_b,
               x, stream=None, compute: int = COMPUTE_F32):
    """samq_vit_prefix_v2: patch embedding + tiled pos_embed + ln_pre into x
    [tokens][E] f32 (F32 columns with F32 semantics, or f16 columns)."""
    _check(library().samq_vit_prefix_v2(_addr(image), width, height, patch, _addr(patch_w), embed, _addr(pos_embed),
                                        pos_grid, _addr(ln_w), _addr(ln_b), _addr(x), compute, _stream(stream)))


class TextBlock:
    """One text-encoder block's device parameters (samq_text_block_v1): f32
    device tensors and four Weights handles (kept alive here)."""

    def __init__(self, norm1_w, norm1_b, in_proj: Weights, in_proj_b, out_proj: Weights, out_proj_b, norm2_w, norm2_b,
                 fc1: Weights, fc1_b, fc2: Weights, fc2_b):
        self._keep = (norm1_w, norm1_b, in_proj, in_proj_b, out_proj, out_proj_b, norm2_w, norm2_b, fc1, fc1_b, fc2,
                      fc2_b)
        self.desc = TextBlockDesc(1, _addr(norm1_w), _addr(norm1_b), in_proj.handle, _addr(in_proj_b),
                                  out_proj.handle, _addr(out_proj_b), _addr(norm2_w), _addr(norm2_b), fc1.handle,
                                  _addr(fc1_b), fc2.handle, _addr(fc2_b))


def text_block_forward(block: TextBlock, x, tokens: int, stream=None):
    """samq_text_block_forward_v1: one causal pre-LN block in place on x [tokens][E]."""
    _check(library().samq_text_block_forward_v1(ctypes.byref(block.desc), _addr(x), tokens, _stream(stream)))


def token_embed(table, vocab: int, width: int, ids, pos, out, stream=None):
    """samq_token_embed_v1: out = table[ids] + pos; ids is a host sequence of ints."""
    arr = (ctypes.c_int32 * len(ids))(*[int(i) for i in ids])
    _check(library().samq_token_embed_v1(_addr(table), vocab, width, arr, len(ids), _addr(pos), _addr(out),
                                         _stream(stream)))


def layer_norm(x, rows: int, width: int, ldx: int, w, b, out, ldo: int, eps: float = 1e-5, stream=None):
    """samq_layer_norm_v1: f32 LayerNorm of rows."""
    _check(library().samq_layer_norm_v1(_addr(x), rows, width, ldx, _addr(w), _addr(b), eps, _addr(out), ldo,
                                        _stream(stream)))


def attention(q, ldq: int, k, ldk: int, v, ldv: int, lq: int, lk: int, heads: int, head_dim: int, scale: float, out,
              ldo: int, causal: bool = False, bias=None, bias_h: int = 0, bias_q: int = 0, stream=None):
    """samq_attention_v1: F32 multi-head attention with an optional causal or additive mask."""
    _check(library().samq_attention_v1(_addr(q), ldq, _addr(k), ldk, _addr(v), ldv, lq, lk, heads, head_dim, scale,
                                       1 if causal else 0, _addr(bias), bias_h, bias_q, _addr(out), ldo,
                                       _stream(stream)))


def linear_ref(weights, bias) -> LinearRef:
    """A samq_linear_ref_v1 for a Weights (quantized) or Dense handle."""
    if isinstance(weights, Weights):
        return LinearRef(weights.handle, None, _addr(bias))
    return LinearRef(None, weights.handle, _addr(bias))


class FusionLayer:
    """One fusion-encoder layer (samq_fusion_layer_v1); `linears` maps
    sa_in_proj, sa_out_proj, ca_in_proj, ca_out_proj, linear1, linear2 to
    (Weights or Dense, bias device tensor); norms to device tensors."""

    def __init__(self, heads: int, norms: dict, linears: dict):
        self._keep = (norms, linears)
        fields = [1, heads] + [_addr(norms[n]) for n in ("norm1_w", "norm1_b", "norm2_w", "norm2_b", "norm3_w",
                                                         "norm3_b")]
        fields += [linear_ref(*linears[n]) for n in ("sa_in_proj", "sa_out_proj", "ca_in_proj", "ca_out_proj",
                                                     "linear1", "linear2")]
        self.desc = FusionLayerDesc(*fields)


def fusion_layer_forward(layer: FusionLayer, x, pos, tokens: int, prompt, prompt_bias, prompt_tokens: int,
                         stream=None):
    """samq_fusion_layer_forward_v1 in place on x [tokens][D]."""
    _check(library().samq_fusion_layer_forward_v1(ctypes.byref(layer.desc), _addr(x), _addr(pos), tokens,
                                                  _addr(prompt), _addr(prompt_bias), prompt_tokens, _stream(stream)))


class Decoder:
    """The DETR decoder with scoring and presence head (samq_decoder_v1).
    `layers`: per layer a dict of DECODER_LAYER_LINEARS -> (Weights or Dense,
    bias) and DECODER_LAYER_NORMS -> device tensors.  `params`: device tensors
    query_embed, presence_token, reference_points, rpb_x0_w / b, rpb_y0_w / b,
    norm_w / b, presence_norm_w / b, prompt_mlp_norm_w / b; `heads_linears`:
    ref_point_head, bbox_embed, presence_head, prompt_mlp (lists of (handle,
    bias)), rpb_x1, rpb_y1, prompt_proj, hs_proj ((handle, bias))."""

    def __init__(self, heads: int, queries: int, layers: list, params: dict, heads_linears: dict):
        self._keep = (layers, params, heads_linears)
        arr = (DecoderLayerDesc * len(layers))()
        for i, ly in enumerate(layers):
            arr[i] = DecoderLayerDesc(*([linear_ref(*ly[n]) for n in DECODER_LAYER_LINEARS] +
                                        [_addr(ly[n]) for n in DECODER_LAYER_NORMS]))
        self._layers = arr
        d = DecoderDesc()
        d.version, d.heads, d.layers, d.queries = 1, heads, len(layers), queries
        d.layer = ctypes.cast(arr, ctypes.POINTER(DecoderLayerDesc))
        for n in ("query_embed", "presence_token", "reference_points", "rpb_x0_w", "rpb_x0_b", "rpb_y0_w", "rpb_y0_b",
                  "norm_w", "norm_b", "presence_norm_w", "presence_norm_b", "prompt_mlp_norm_w", "prompt_mlp_norm_b"):
            setattr(d, n, _addr(params[n]))
        for n in ("ref_point_head", "bbox_embed", "presence_head", "prompt_mlp"):
            field = getattr(d, n)
            for j, pair in enumerate(heads_linears[n]):
                field[j] = linear_ref(*pair)
        for n in ("rpb_x1", "rpb_y1", "prompt_proj", "hs_proj"):
            setattr(d, n, linear_ref(*heads_linears[n]))
        self.desc = d


def decoder_forward(decoder: Decoder, enc, enc_pos, grid: int, prompt, prompt_bias, prompt_valid, prompt_tokens: int,
                    queries_out, boxes, scores, presence, stream=None):
    """samq_decoder_forward_v1."""
    _check(library().samq_decoder_forward_v1(ctypes.byref(decoder.desc), _addr(enc), _addr(enc_pos), grid,
                                             _addr(prompt), _addr(prompt_bias), _addr(prompt_valid), prompt_tokens,
                                             _addr(queries_out), _addr(boxes), _addr(scores), _addr(presence),
                                             _stream(stream)))


class GeometryEncoder:
    """The text-only-prompt geometry encoder (samq_geometry_encoder_v1).
    `layers`: per layer a dict of GEOMETRY_LAYER_LINEARS -> (Weights or Dense,
    bias) and GEOMETRY_LAYER_NORMS -> device tensors; `params`: cls_token,
    norm_w / b, encode_norm_w / b device tensors; final_proj: (handle, bias)."""

    def __init__(self, heads: int, layers: list, params: dict, final_proj):
        self._keep = (layers, params, final_proj)
        arr = (GeometryLayerDesc * len(layers))()
        for i, ly in enumerate(layers):
            arr[i] = GeometryLayerDesc(*([linear_ref(*ly[n]) for n in GEOMETRY_LAYER_LINEARS] +
                                         [_addr(ly[n]) for n in GEOMETRY_LAYER_NORMS]))
        self._layers = arr
        self.desc = GeometryEncoderDesc(1, heads, len(layers), ctypes.cast(arr, ctypes.POINTER(GeometryLayerDesc)),
                                        _addr(params["cls_token"]), linear_ref(*final_proj), _addr(params["norm_w"]),
                                        _addr(params["norm_b"]), _addr(params["encode_norm_w"]),
                                        _addr(params["encode_norm_b"]))


def geometry_encoder_forward(encoder: GeometryEncoder, image, pos, tokens: int, out, stream=None):
    """samq_geometry_encoder_forward_v1: out [D] = the geometry prompt token."""
    _check(library().samq_geometry_encoder_forward_v1(ctypes.byref(encoder.desc), _addr(image), _addr(pos), tokens,
                                                      _addr(out), _stream(stream)))


class SegHead:
    """The segmentation head (samq_seg_head_v1): `params` holds device tensors
    cross_attn_norm_w / b, conv_b, norm_w, norm_b (pairs) and instance_b;
    convs: two 3x3 Dense CONV handles; instance: 1x1 Dense CONV; ca_in_proj,
    ca_out_proj: (handle, bias); mask_embed: three (handle, bias)."""

    def __init__(self, heads: int, params: dict, convs, instance, ca_in_proj, ca_out_proj, mask_embed):
        self._keep = (params, convs, instance, ca_in_proj, ca_out_proj, mask_embed)
        d = SegHeadDesc()
        d.version, d.heads = 1, heads
        d.cross_attn_norm_w, d.cross_attn_norm_b = _addr(params["cross_attn_norm_w"]), _addr(params["cross_attn_norm_b"])
        d.ca_in_proj, d.ca_out_proj = linear_ref(*ca_in_proj), linear_ref(*ca_out_proj)
        for i in range(2):
            d.conv[i] = convs[i].handle
            d.conv_b[i] = _addr(params["conv_b"][i])
            d.norm_w[i] = _addr(params["norm_w"][i])
            d.norm_b[i] = _addr(params["norm_b"][i])
        d.instance, d.instance_b = instance.handle, _addr(params["instance_b"])
        for j in range(3):
            d.mask_embed[j] = linear_ref(*mask_embed[j])
        self.desc = d


def seg_head_forward(head: SegHead, enc, grid: int, fpn0, fpn1, queries, nq: int, prompt, prompt_bias,
                     prompt_tokens: int, mask_logits, stream=None):
    """samq_seg_head_forward_v1: mask_logits [nq][(4 grid)^2]."""
    _check(library().samq_seg_head_forward_v1(ctypes.byref(head.desc), _addr(enc), grid, _addr(fpn0), _addr(fpn1),
                                              _addr(queries), nq, _addr(prompt), _addr(prompt_bias), prompt_tokens,
                                              _addr(mask_logits), _stream(stream)))


def quantize_rows(qtype: int, w):
    """samq_quantize_rows_v1: f32 [n][k] (numpy) -> packed GGUF rows (uint8, host)."""
    import numpy as np
    w = np.ascontiguousarray(w, dtype=np.float32)
    n, k = w.shape
    out = np.empty(n * row_bytes(qtype, k), np.uint8)
    _check(library().samq_quantize_rows_v1(qtype, k, n, w.ctypes.data, out.ctypes.data, out.nbytes))
    return out


MMQ_CODES_F16, MMQ_CODES_I8 = 0, 1


class MmqWeights:
    """Q8_0 weights for the exact MMQ path (samq_mmq_weights*): integer codes
    held as f16 (variant MMQ_CODES_F16) or int8 (MMQ_CODES_I8) plus f32 block
    scales."""

    def __init__(self, qtype: int, k: int, n: int, gguf_rows, variant: int = MMQ_CODES_F16, device: int = 0,
                 stream=None):
        import numpy as np
        rows = np.ascontiguousarray(gguf_rows, dtype=np.uint8).reshape(-1)
        handle = ctypes.c_void_p()
        _check(library().samq_mmq_weights_create_v1(device, qtype, variant, k, n, rows.ctypes.data, rows.nbytes,
                                                    _stream(stream), ctypes.byref(handle)))
        self.handle, self.k, self.n, self.variant, self.device = handle, k, n, variant, device

    def close(self):
        if self.handle:
            _check(library().samq_mmq_weights_destroy_v1(self.handle))
            self.handle = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


def linear_mmq(w: MmqWeights, x, m: int, ldx: int, bias, epilogue: int, y, ldy: int, stream=None):
    """samq_linear_mmq_v1: y = epilogue(x W^T + bias) with GGML MMQ's exact arithmetic."""
    _check(library().samq_linear_mmq_v1(w.handle, _addr(x), m, ldx, _addr(bias), epilogue, _addr(y), ldy,
                                        _stream(stream)))


def sine_pe_2d(h: int, w: int, d: int):
    """samq_sine_pe_2d_v1: the image positional encoding [h * w][d] (host f32 numpy)."""
    import numpy as np
    out = np.empty((h * w, d), np.float32)
    _check(library().samq_sine_pe_2d_v1(h, w, d, out.ctypes.data))
    return out


class Dense:
    """Dense F32 / F16 weights in their GGML layout (samq_dense*), used with
    F32 semantics.  kind DENSE_LINEAR: w is [n][k] (k = cin, n = cout);
    DENSE_CONV: [cout][cin][kh][kw] (kw == kh in {1, 3}); DENSE_DECONV2X2:
    [cin][cout][2][2]."""

    def __init__(self, kind: int, w: np.ndarray, device: int = 0, stream=None):
        w = np.ascontiguousarray(w)
        if w.dtype == np.float32:
            dtype = F32
        elif w.dtype == np.float16:
            dtype = F16
        else:
            raise TypeError("dense weights are float32 or float16")
        if kind == DENSE_LINEAR:
            cout, cin = w.shape
            kw = kh = 1
        elif kind == DENSE_CONV:
            cout, cin, kh, kw = w.shape
        elif kind == DENSE_DECONV2X2:
            cin, cout, kh, kw = w.shape
        else:
            raise ValueError("unknown dense kind")
        handle = ctypes.c_void_p()
        _check(library().samq_dense_create_v1(device, dtype, kind, kw, kh, cin, cout, w.ctypes.data, w.nbytes,
                                              _stream(stream), ctypes.byref(handle)))
        self.handle = handle
        self.kind, self.cin, self.cout, self.ks, self.device = kind, cin, cout, kw, device

    def close(self):
        if self.handle:
            _check(library().samq_dense_destroy_v1(self.handle))
            self.handle = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


def dense_linear(w: Dense, x, m: int, ldx: int, bias, epilogue: int, y, ldy: int, stream=None):
    """samq_dense_linear_v1: y = gelu?(x w^T + bias), F32 semantics."""
    _check(library().samq_dense_linear_v1(w.handle, _addr(x), m, ldx, _addr(bias), epilogue, _addr(y), ldy,
                                          _stream(stream)))


def conv2d(w: Dense, x, width: int, height: int, bias, epilogue: int, y, stream=None):
    """samq_conv2d_v1: NHWC convolution (stride 1, pad ks // 2) or 2x2 deconvolution."""
    _check(library().samq_conv2d_v1(w.handle, _addr(x), width, height, _addr(bias), epilogue, _addr(y),
                                    _stream(stream)))


def maxpool2x2(x, width: int, height: int, channels: int, y, stream=None):
    _check(library().samq_maxpool2x2_v1(_addr(x), width, height, channels, _addr(y), _stream(stream)))


class Neck:
    """The SimpleFPN neck (samq_neck_v1): layers maps each NECK_LAYERS name to
    (Dense, bias device tensor)."""

    def __init__(self, layers: dict):
        self._keep = layers
        vals = [1]
        for name in NECK_LAYERS:
            w, b = layers[name]
            vals += [w.handle, _addr(b)]
        self.desc = NeckDesc(*vals)


def neck_forward(neck: Neck, x, grid_w: int, grid_h: int, outs, stream=None):
    """samq_neck_forward_v1: the four NHWC feature maps of the ViT output x."""
    arr = (_vp * 4)(*[_addr(o) for o in outs])
    _check(library().samq_neck_forward_v1(ctypes.byref(neck.desc), _addr(x), grid_w, grid_h, arr, _stream(stream)))
