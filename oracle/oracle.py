"""ctypes binding of the CPU oracle (test infrastructure only).

Only tests/, __graft_entry__.smoke() and bench.py's CPU legs import this
module; it is the checker, never the measured or shipped path.  Every function
wraps one entry point of samq_oracle.c, which cites the reference file/line it
restates.
"""
from __future__ import annotations

import ctypes
import os
import subprocess
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
LIB_PATH = HERE / "libsamq_oracle.so"

Q8_0, Q8_1, Q4_K, Q5_K, Q6_K, Q8_K = 8, 9, 12, 13, 14, 15
TYPE_NAMES = {Q8_0: "Q8_0", Q4_K: "Q4_K", Q5_K: "Q5_K", Q6_K: "Q6_K"}
NAME_TYPES = {v: k for k, v in TYPE_NAMES.items()}
EPILOGUE_NONE, EPILOGUE_GELU_ERF = 0, 1

_lib = None


def build() -> Path:
    """Compile the oracle with its Makefile (gcc + OpenMP)."""
    subprocess.run(["make", "-C", str(HERE), "-s"], check=True)
    return LIB_PATH


def lib() -> ctypes.CDLL:
    global _lib
    if _lib is None:
        if not LIB_PATH.exists():
            build()
        _lib = ctypes.CDLL(str(LIB_PATH))
        i64, i32, vp = ctypes.c_int64, ctypes.c_int, ctypes.c_void_p
        sig = {
            "oracle_block_elements": (i64, [i32]),
            "oracle_block_bytes": (i64, [i32]),
            "oracle_row_bytes": (i64, [i32, i64]),
            "oracle_f32_to_f16": (ctypes.c_uint16, [ctypes.c_float]),
            "oracle_f16_to_f32": (ctypes.c_float, [ctypes.c_uint16]),
            "oracle_quantize_q8_0": (i32, [vp, i64, vp]),
            "oracle_quantize_kquant": (i32, [i32, vp, i64, vp]),
            "oracle_dequantize": (i32, [i32, vp, i64, vp]),
            "oracle_quantize_q8_1": (i32, [vp, i64, i64, i64, vp]),
            "oracle_mmq_d4_bytes": (i64, [i64, i64]),
            "oracle_quantize_mmq_d4": (i32, [vp, i64, i64, i64, vp]),
            "oracle_act_f16": (i32, [vp, i64, i64, i64, vp]),
            "oracle_q8_1_decode": (i32, [vp, i64, i64, vp]),
            "oracle_quantize_q8_k": (i32, [vp, i64, vp]),
            "oracle_packet_code_bytes": (i64, [i32]),
            "oracle_packet_bytes": (i64, [i32]),
            "oracle_packets_size": (i64, [i32, i64, i64]),
            "oracle_pack_packets": (i32, [i32, i64, i64, vp, vp]),
            "oracle_unpack_packets": (i32, [i32, i64, i64, vp, vp]),
            "oracle_weight_f16": (i32, [i32, i64, i64, vp, vp]),
            "oracle_gemm_f64": (i32, [vp, vp, i64, i64, i64, vp, i32, vp, i32]),
            "oracle_gemm_f16_f64": (i32, [vp, vp, i64, i64, i64, vp, i32, vp, i32]),
            "oracle_cpu_linear": (i32, [i32, vp, i64, i64, vp, i64, i64, vp, i32, vp, i64, i32]),
            "oracle_cpu_has_vnni": (i32, []),
            "oracle_vit_attention": (i32, [vp, i64, i32, i32, i32, i32, i32, vp, vp, i64, vp, i64, i32]),
            "oracle_flash_attn_f32": (i32, [vp, i64, vp, i64, vp, i64, i64, i64, i32, ctypes.c_float, vp, i64,
                                            i32]),
        }
        for name, (res, args) in sig.items():
            fn = getattr(_lib, name)
            fn.restype = res
            fn.argtypes = args
    return _lib


def _ptr(a: np.ndarray | None):
    return None if a is None else ctypes.c_void_p(a.ctypes.data)


def _check(rc: int, what: str):
    if rc != 0:
        raise ValueError(f"oracle {what} rejected its arguments")


def default_threads() -> int:
    return max(1, len(os.sched_getaffinity(0)))


def row_bytes(qtype: int, k: int) -> int:
    rb = lib().oracle_row_bytes(qtype, k)
    if rb < 0:
        raise ValueError("width is not block aligned for this type")
    return rb


def quantize_q8_0(x: np.ndarray) -> np.ndarray:
    x = np.ascontiguousarray(x, dtype=np.float32)
    out = np.empty(x.size // 32 * 34, dtype=np.uint8)
    _check(lib().oracle_quantize_q8_0(_ptr(x), x.size, _ptr(out)), "quantize_q8_0")
    return out


def quantize_kquant(qtype: int, x: np.ndarray) -> np.ndarray:
    x = np.ascontiguousarray(x, dtype=np.float32)
    out = np.empty(x.size // 256 * lib().oracle_block_bytes(qtype), dtype=np.uint8)
    _check(lib().oracle_quantize_kquant(qtype, _ptr(x), x.size, _ptr(out)), "quantize_kquant")
    return out


def quantize(qtype: int, w: np.ndarray) -> np.ndarray:
    """Pack an [n][k] f32 matrix row by row into GGUF blocks of `qtype`."""
    w = np.ascontiguousarray(w, dtype=np.float32)
    return quantize_q8_0(w) if qtype == Q8_0 else quantize_kquant(qtype, w)


def dequantize(qtype: int, blocks: np.ndarray, n_elements: int) -> np.ndarray:
    blocks = np.ascontiguousarray(blocks, dtype=np.uint8)
    out = np.empty(n_elements, dtype=np.float32)
    _check(lib().oracle_dequantize(qtype, _ptr(blocks), n_elements, _ptr(out)), "dequantize")
    return out


def quantize_q8_1(x: np.ndarray) -> np.ndarray:
    x = np.ascontiguousarray(x, dtype=np.float32)
    rows, k = x.shape
    out = np.empty(rows * (k // 32) * 36, dtype=np.uint8)
    _check(lib().oracle_quantize_q8_1(_ptr(x), rows, k, k, _ptr(out)), "quantize_q8_1")
    return out


def quantize_mmq_d4(x: np.ndarray) -> np.ndarray:
    x = np.ascontiguousarray(x, dtype=np.float32)
    rows, k = x.shape
    out = np.empty(lib().oracle_mmq_d4_bytes(rows, k), dtype=np.uint8)
    _check(lib().oracle_quantize_mmq_d4(_ptr(x), rows, k, k, _ptr(out)), "quantize_mmq_d4")
    return out


def act_f16(x: np.ndarray) -> np.ndarray:
    x = np.ascontiguousarray(x, dtype=np.float32)
    rows, k = x.shape
    out = np.empty((rows, k), dtype=np.uint16)
    _check(lib().oracle_act_f16(_ptr(x), rows, k, k, _ptr(out)), "act_f16")
    return out.view(np.float16)


def q8_1_decode(q: np.ndarray, rows: int, k: int) -> np.ndarray:
    q = np.ascontiguousarray(q, dtype=np.uint8)
    out = np.empty((rows, k), dtype=np.float32)
    _check(lib().oracle_q8_1_decode(_ptr(q), rows, k, _ptr(out)), "q8_1_decode")
    return out


def quantize_q8_k(x: np.ndarray) -> np.ndarray:
    x = np.ascontiguousarray(x, dtype=np.float32)
    out = np.empty(x.size // 256 * 292, dtype=np.uint8)
    _check(lib().oracle_quantize_q8_k(_ptr(x), x.size, _ptr(out)), "quantize_q8_k")
    return out


def packets_size(qtype: int, k: int, n: int) -> int:
    return lib().oracle_packets_size(qtype, k, n)


def pack_packets(qtype: int, k: int, n: int, rows: np.ndarray) -> np.ndarray:
    rows = np.ascontiguousarray(rows, dtype=np.uint8)
    out = np.empty(packets_size(qtype, k, n), dtype=np.uint8)
    _check(lib().oracle_pack_packets(qtype, k, n, _ptr(rows), _ptr(out)), "pack_packets")
    return out


def unpack_packets(qtype: int, k: int, n: int, packets: np.ndarray) -> np.ndarray:
    packets = np.ascontiguousarray(packets, dtype=np.uint8)
    out = np.empty(n * row_bytes(qtype, k), dtype=np.uint8)
    _check(lib().oracle_unpack_packets(qtype, k, n, _ptr(packets), _ptr(out)), "unpack_packets")
    return out


def weight_f16(qtype: int, k: int, n: int, rows: np.ndarray) -> np.ndarray:
    rows = np.ascontiguousarray(rows, dtype=np.uint8)
    out = np.empty((n, k), dtype=np.uint16)
    _check(lib().oracle_weight_f16(qtype, k, n, _ptr(rows), _ptr(out)), "weight_f16")
    return out.view(np.float16)


def gemm_f64(w: np.ndarray, x: np.ndarray, bias=None, epilogue=EPILOGUE_NONE, threads=None) -> np.ndarray:
    """Y = X . W^T with f64 accumulation over f32 (or f16) operands."""
    n, k = w.shape
    m = x.shape[0]
    y = np.empty((m, n), dtype=np.float32)
    b = None if bias is None else np.ascontiguousarray(bias, dtype=np.float32)
    t = threads or default_threads()
    if w.dtype == np.float16:
        w16 = np.ascontiguousarray(w).view(np.uint16)
        x16 = np.ascontiguousarray(x, dtype=np.float16).view(np.uint16)
        rc = lib().oracle_gemm_f16_f64(_ptr(w16), _ptr(x16), m, n, k, _ptr(b), epilogue, _ptr(y), t)
    else:
        w32 = np.ascontiguousarray(w, dtype=np.float32)
        x32 = np.ascontiguousarray(x, dtype=np.float32)
        rc = lib().oracle_gemm_f64(_ptr(w32), _ptr(x32), m, n, k, _ptr(b), epilogue, _ptr(y), t)
    _check(rc, "gemm")
    return y


def cpu_linear(qtype: int, rows: np.ndarray, k: int, n: int, x: np.ndarray, bias=None,
               epilogue=EPILOGUE_NONE, threads=None, out=None) -> np.ndarray:
    """Restated GGML CPU quantized mul_mat (+bias, +erf-GELU)."""
    rows = np.ascontiguousarray(rows, dtype=np.uint8)
    x = np.ascontiguousarray(x, dtype=np.float32)
    m = x.shape[0]
    y = out if out is not None else np.empty((m, n), dtype=np.float32)
    b = None if bias is None else np.ascontiguousarray(bias, dtype=np.float32)
    rc = lib().oracle_cpu_linear(qtype, _ptr(rows), k, n, _ptr(x), m, k, _ptr(b), epilogue, _ptr(y), n,
                                 threads or default_threads())
    _check(rc, "cpu_linear")
    return y


def vit_attention(qkv: np.ndarray, grid_w: int, grid_h: int, heads: int, head_dim: int, window: int,
                  freqs: np.ndarray, rows=None, threads=None) -> np.ndarray:
    """f64 windowed/global attention with RoPE for the query tokens `rows`."""
    qkv = np.ascontiguousarray(qkv, dtype=np.float32)
    freqs = np.ascontiguousarray(freqs, dtype=np.float32)
    E = heads * head_dim
    r = None if rows is None else np.ascontiguousarray(rows, dtype=np.int64)
    n = qkv.shape[0] if r is None else r.size
    out = np.empty((n, E), dtype=np.float32)
    rc = lib().oracle_vit_attention(_ptr(qkv), qkv.shape[1], grid_w, grid_h, heads, head_dim, window, _ptr(freqs),
                                    _ptr(r), n, _ptr(out), E, threads or default_threads())
    _check(rc, "vit_attention")
    return out


def flash_attn_f32(q: np.ndarray, k: np.ndarray, v: np.ndarray, scale: float, threads=None,
                   out: np.ndarray | None = None) -> np.ndarray:
    """Restated GGML CPU flash attention (f32 online softmax) of one head:
    q [n_q][hd], k / v [n_kv][hd] f32 (rows may be strided views of a
    contiguous last axis)."""
    for a in (q, k, v):
        assert a.dtype == np.float32 and a.strides[1] == 4
    n_q, hd = q.shape
    y = out if out is not None else np.empty((n_q, hd), dtype=np.float32)
    rc = lib().oracle_flash_attn_f32(_ptr(q), q.strides[0] // 4, _ptr(k), k.strides[0] // 4, _ptr(v),
                                     v.strides[0] // 4, n_q, k.shape[0], hd, scale, _ptr(y), y.strides[0] // 4,
                                     threads or default_threads())
    _check(rc, "flash_attn_f32")
    return y


def rope_freqs(positions: int, head_dim: int = 64, seed: int = 0) -> np.ndarray:
    """Unit-modulus (cos, sin) pairs [positions][head_dim/2][2] (any such table is a valid freqs_cis)."""
    rng = np.random.default_rng(seed)
    ang = rng.uniform(-np.pi, np.pi, (positions, head_dim // 2))
    return np.stack([np.cos(ang), np.sin(ang)], axis=-1).astype(np.float32)


def has_vnni() -> bool:
    return bool(lib().oracle_cpu_has_vnni())


def gelu_erf(v: np.ndarray) -> np.ndarray:
    from math import erf, sqrt
    f = np.vectorize(lambda t: 0.5 * t * (1.0 + erf(t / sqrt(2.0))))
    return f(v.astype(np.float64)).astype(np.float32)


def layer_norm(x: np.ndarray, w: np.ndarray, b: np.ndarray, eps: float = 1e-5) -> np.ndarray:
    """ggml_norm(eps) * w + b in f64 (src/models/sam3/ops.hpp:56-66), rounded to f32."""
    x64 = np.asarray(x, dtype=np.float64)
    c = x64 - x64.mean(axis=1, keepdims=True)
    var = (c * c).mean(axis=1, keepdims=True)
    return (c / np.sqrt(var + eps) * np.asarray(w, np.float64) + np.asarray(b, np.float64)).astype(np.float32)


_EXACT_OPERANDS = [False]


def staged_linear(w: np.ndarray, x: np.ndarray, bias=None, epilogue=EPILOGUE_NONE) -> np.ndarray:
    """A quantized linear with GGML MMQ's operand semantics: x is staged to
    Q8_1 (quantize_q8_1 restated) and the product runs over the DECODED
    operands, d_x * q_x for the activations and the weight's f32 dequantized
    values (w = dequantize(...), [n][k] f32, no f16 rounding), in f64; then
    bias and erf-GELU, rounded to f32 (the reference's F32 output tensor).
    Inside `exact_operands()` both operands are first rounded to f16 as the
    device's tensor-core operands are (act_f16, and the f16 rounding of the
    decoded weight that weight_f16 produces)."""
    x = np.ascontiguousarray(x, dtype=np.float32)
    m, k = x.shape
    if _EXACT_OPERANDS[0]:
        w16 = np.ascontiguousarray(np.asarray(w, np.float32).astype(np.float16))
        return gemm_f64(w16, act_f16(x), bias=bias, epilogue=epilogue)
    xd = q8_1_decode(quantize_q8_1(x), m, k).astype(np.float64)
    y = xd @ np.asarray(w, np.float64).T
    if bias is not None:
        y += np.asarray(bias, np.float64)
    if epilogue == EPILOGUE_GELU_ERF:
        y = gelu_erf64(y)
    return y.astype(np.float32)


def win_part_index(grid_w: int, grid_h: int, window: int) -> np.ndarray:
    """ggml_win_part as an index map (src/models/sam3/vision.hpp:170-173):
    the [C, W, H] grid, zero-padded up to multiples of `window`, cut into
    window x window tiles ordered row-major over the tile grid, each tile's
    tokens row-major.  Returns [windows][window * window] raster token indices
    (y * grid_w + x), -1 where the tile covers padding."""
    nx, ny = -(-grid_w // window), -(-grid_h // window)
    ly, lx = np.divmod(np.arange(window * window), window)
    out = np.empty((nx * ny, window * window), dtype=np.int64)
    for wy in range(ny):
        for wx in range(nx):
            y, x = wy * window + ly, wx * window + lx
            out[wy * nx + wx] = np.where((x < grid_w) & (y < grid_h), y * grid_w + x, -1)
    return out


def win_part(x: np.ndarray, grid_w: int, grid_h: int, window: int) -> np.ndarray:
    """x [grid_h * grid_w][C] (raster) -> [windows][window * window][C] with
    zeros in the padding (ggml_win_part)."""
    idx = win_part_index(grid_w, grid_h, window)
    x = np.asarray(x)
    out = np.zeros(idx.shape + x.shape[1:], dtype=x.dtype)
    valid = idx >= 0
    out[valid] = x[idx[valid]]
    return out


def win_unpart(parts: np.ndarray, grid_w: int, grid_h: int, window: int) -> np.ndarray:
    """Inverse of win_part (ggml_win_unpart, vision.hpp:225-227): drops the padding."""
    idx = win_part_index(grid_w, grid_h, window)
    out = np.empty((grid_w * grid_h,) + parts.shape[2:], dtype=parts.dtype)
    valid = idx >= 0
    out[idx[valid]] = parts[valid]
    return out


def rope64(x: np.ndarray, freqs: np.ndarray) -> np.ndarray:
    """sam3_apply_rope (vision.hpp:100-148) in f64: channel pairs (2i, 2i+1)
    of x [n][head_dim] rotated by freqs [n][head_dim/2] (cos, sin)."""
    x = np.asarray(x, np.float64)
    f = np.asarray(freqs, np.float64)
    re, im = x[:, 0::2], x[:, 1::2]
    c, s = f[..., 0], f[..., 1]
    out = np.empty_like(x)
    out[:, 0::2] = re * c - im * s
    out[:, 1::2] = re * s + im * c
    return out


def attention_np(qkv: np.ndarray, grid_w: int, grid_h: int, heads: int, window: int, freqs: np.ndarray,
                 rows=None, pad_qkv=None) -> np.ndarray:
    """f64 RoPE + windowed / global attention of one ViT block
    (vision.hpp:170-227): qkv [tokens][3E] f32 (Q | K | V, heads of 64),
    windows from win_part (padding tokens carry `pad_qkv`, the qkv of a zero
    LayerNorm row, as GGML's zero-padded partition does), RoPE by local
    position, softmax(Q K^T / 8) V per head, win_unpart.  Returns [rows][E]
    f32 for the query tokens `rows` (all when None)."""
    qkv = np.asarray(qkv, np.float32)
    E = heads * 64
    tokens = grid_w * grid_h
    groups = win_part_index(grid_w, grid_h, window) if window else np.arange(tokens)[None, :]
    want = np.zeros(tokens, dtype=bool)
    want[np.arange(tokens) if rows is None else np.asarray(rows, np.int64)] = True
    out = np.zeros((tokens, E), dtype=np.float32)
    freqs = np.asarray(freqs, np.float64).reshape(groups.shape[1], 32, 2)
    for g in groups:
        valid = g >= 0
        if not want[g[valid]].any():
            continue
        rows_g = np.empty((g.size, 3 * E), dtype=np.float64)
        rows_g[valid] = qkv[g[valid]]
        if not valid.all():
            rows_g[~valid] = np.asarray(pad_qkv, np.float64).reshape(3 * E)
        qsel = np.nonzero(valid & want[np.where(valid, g, 0)])[0]
        for h in range(heads):
            q = rope64(rows_g[qsel, h * 64:(h + 1) * 64], freqs[qsel])
            k = rope64(rows_g[:, E + h * 64:E + (h + 1) * 64], freqs)
            v = rows_g[:, 2 * E + h * 64:2 * E + (h + 1) * 64]
            s = (q @ k.T) * 0.125
            s -= s.max(axis=1, keepdims=True)
            p = np.exp(s)
            o = (p @ v) / p.sum(axis=1, keepdims=True)
            out[g[qsel], h * 64:(h + 1) * 64] = o
    sel = np.arange(tokens) if rows is None else np.asarray(rows, np.int64)
    return out[sel]


def cpu_path_linear(blk: dict, name: str, x: np.ndarray, bias=None, epilogue=EPILOGUE_NONE) -> np.ndarray:
    """The block linear `name` as the reference's GGML CPU backend computes it
    (cpu_linear: Q8_0 / Q8_K activation packing, integer block dots, f32
    scales); blk[name + "_q"] = (type, packed GGUF rows)."""
    qtype, rows = blk[name + "_q"]
    n, k = blk[name + "_w"].shape
    return cpu_linear(qtype, rows, k, n, x, bias=bias, epilogue=epilogue)


def vit_block(x: np.ndarray, blk: dict, grid_w: int, grid_h: int, rows=None, threads=None,
              cpu_path: bool = False) -> np.ndarray:
    """One SAM 3 ViT block (src/models/sam3/vision.hpp:152-243) with GGML's
    arithmetic for every quantized linear (staged_linear: Q8_1-staged input,
    f32-decoded weights, f64 dots) and f64 LayerNorm / attention:
      x1 = x + proj(attn(RoPE(qkv(LN1(x)))));  out = x1 + fc2(GELU(fc1(LN2(x1)))).
    blk holds window, norm1_w/b, norm2_w/b, the decoded f32 weights qkv_w,
    proj_w, fc1_w, fc2_w ([n][k], from dequantize), the biases and freqs.  x
    is [tokens][E] f32 in raster order; the residual adds are f32 as in GGML.
    Returns the block output for the tokens in `rows` (all when None): K and V
    cover every token, the rest only `rows`.  cpu_path=True computes the
    linears as the reference's CPU backend does instead (cpu_path_linear),
    the yardstick for how far two of the reference's own backends drift apart."""
    del threads

    def linear(name, v, epilogue=EPILOGUE_NONE):
        if cpu_path:
            return cpu_path_linear(blk, name, v, blk[name + "_b"], epilogue)
        return staged_linear(blk[name + "_w"], v, blk[name + "_b"], epilogue)

    x = np.ascontiguousarray(x, dtype=np.float32)
    E = x.shape[1]
    heads = E // 64
    h = layer_norm(x, blk["norm1_w"], blk["norm1_b"])
    qkv = linear("qkv", h)
    pad = linear("qkv", np.zeros((1, E), np.float32))
    sel = np.arange(x.shape[0]) if rows is None else np.asarray(rows, dtype=np.int64)
    att = attention_np(qkv, grid_w, grid_h, heads, blk["window"], blk["freqs"], rows=sel, pad_qkv=pad)
    x1 = x[sel] + linear("proj", att)
    h2 = layer_norm(x1, blk["norm2_w"], blk["norm2_b"])
    f = linear("fc1", h2, EPILOGUE_GELU_ERF)
    return x1 + linear("fc2", f)


def vit_prefix(image: np.ndarray, patch: int, patch_w: np.ndarray, pos_embed: np.ndarray, ln_w: np.ndarray,
               ln_b: np.ndarray, threads=None) -> np.ndarray:
    """Backbone prefix (src/models/sam3/vision.hpp:252-282) in f64: unpadded
    patch x patch convolution without bias (image [3][H][W], weight
    [E][3][patch][patch]), + pos_embed [pg][pg][E] tiled over the grid, then
    ln_pre.  Returns [tokens][E] f32, tokens in raster order."""
    image = np.asarray(image, dtype=np.float64)
    C, H, W = image.shape
    gh, gw = H // patch, W // patch
    cols = image.reshape(C, gh, patch, gw, patch).transpose(1, 3, 0, 2, 4).reshape(gh * gw, C * patch * patch)
    E = patch_w.shape[0]
    y = cols @ np.asarray(patch_w, np.float64).reshape(E, -1).T
    pg = pos_embed.shape[0]
    py, px = np.divmod(np.arange(gh * gw), gw)
    y += np.asarray(pos_embed, np.float64)[py % pg, px % pg]
    return layer_norm(y, ln_w, ln_b)


# ---- dense F32 modules (neck, fusion / decoder linears in F32 profiles) -----
# f64 restatements; the device path is held to F32-level error against them.

def gelu_erf64(v: np.ndarray) -> np.ndarray:
    """ggml_gelu_erf, 0.5 v (1 + erf(v / sqrt 2)), in f64."""
    from scipy.special import erf
    v = np.asarray(v, np.float64)
    return 0.5 * v * (1.0 + erf(v / np.sqrt(2.0)))


def dense_linear(x: np.ndarray, w: np.ndarray, bias=None, gelu: bool = False) -> np.ndarray:
    """ggml_mul_mat on an F32 / F16 weight [n][k] at GGML_PREC_F32, which the
    reference's CUDA path runs as cuBLAS COMPUTE_32F_PEDANTIC
    (cmake/patches/ggml-precise-cuda.patch:288-356): x [m][k] . w^T (+ bias)
    (then erf-GELU), f64."""
    y = np.asarray(x, np.float64) @ np.asarray(w, np.float64).T
    if bias is not None:
        y = y + np.asarray(bias, np.float64)
    return gelu_erf64(y) if gelu else y


def conv2d_nhwc(x: np.ndarray, w: np.ndarray, bias=None, stride: int = 1, pad: int | None = None) -> np.ndarray:
    """sam3_conv_2d (src/models/sam3/ops.hpp:67-84): im2col + mul_mat over F32
    columns.  x [H][W][Cin] (the reference's [W, H, C] tensor), w
    [Cout][Cin][kh][kw] (GGML [kw, kh, Cin, Cout]).  Default stride 1 and pad
    k // 2 is sam3_conv_2d_s1_ph (:91-94); stride = k, pad = 0 is
    sam3_conv_2d_sk_p0 (:86-89).  f64 [Ho][Wo][Cout]."""
    x = np.asarray(x, np.float64)
    w = np.asarray(w, np.float64)
    H, W, C = x.shape
    co, ci, kh, kw = w.shape
    assert ci == C
    p = kh // 2 if pad is None else pad
    xp = np.zeros((H + 2 * p, W + 2 * p, C))
    xp[p:p + H, p:p + W] = x
    ho = (H + 2 * p - kh) // stride + 1
    wo = (W + 2 * p - kw) // stride + 1
    out = np.zeros((ho, wo, co))
    for ky in range(kh):
        for kx in range(kw):
            patch = xp[ky:ky + stride * (ho - 1) + 1:stride, kx:kx + stride * (wo - 1) + 1:stride]
            out += patch @ w[:, :, ky, kx].T
    if bias is not None:
        out = out + np.asarray(bias, np.float64)
    return out


def deconv2x2_nhwc(x: np.ndarray, w: np.ndarray, bias=None) -> np.ndarray:
    """sam3_deconv_2x2 (src/models/sam3/ops.hpp:96-117), the stride-2 2x2
    ConvTranspose2d as one matrix product: x [H][W][Cin], w [Cin][Cout][2][2]
    (GGML [2, 2, Cout, Cin]); y[2i + ky][2j + kx][co] = sum_c x[i][j][c]
    w[c][co][ky][kx] (+ bias[co]).  f64 [2H][2W][Cout]."""
    x = np.asarray(x, np.float64)
    w = np.asarray(w, np.float64)
    H, W, C = x.shape
    ci, co = w.shape[:2]
    assert ci == C
    out = np.zeros((2 * H, 2 * W, co))
    for ky in range(2):
        for kx in range(2):
            out[ky::2, kx::2] = x @ w[:, :, ky, kx]
    if bias is not None:
        out = out + np.asarray(bias, np.float64)
    return out


def maxpool2x2_nhwc(x: np.ndarray) -> np.ndarray:
    """ggml_pool_2d(MAX, 2, 2, 2, 2, 0, 0) of an NHWC image (floor sizes)."""
    H, W, C = x.shape
    h2, w2 = H // 2, W // 2
    return np.asarray(x)[:2 * h2, :2 * w2].reshape(h2, 2, w2, 2, C).max(axis=(1, 3))


def neck(x: np.ndarray, layers: dict) -> list:
    """sam3_build_neck_graph (src/models/sam3/vision.hpp:307-366) in f64:
    x [gh][gw][E]; layers[name] = (weight, bias) with the samq_neck_v1 names.
    Returns the four NHWC maps (4x, 2x, 1x, 0.5x)."""
    L = layers
    s0 = deconv2x2_nhwc(x, *L["s0_deconv1"])
    s0 = gelu_erf64(s0)
    s0 = deconv2x2_nhwc(s0, *L["s0_deconv2"])
    s0 = conv2d_nhwc(s0, *L["s0_conv1x1"])
    s0 = conv2d_nhwc(s0, *L["s0_conv3x3"])
    s1 = deconv2x2_nhwc(x, *L["s1_deconv1"])
    s1 = conv2d_nhwc(s1, *L["s1_conv1x1"])
    s1 = conv2d_nhwc(s1, *L["s1_conv3x3"])
    s2 = conv2d_nhwc(x, *L["s2_conv1x1"])
    s2 = conv2d_nhwc(s2, *L["s2_conv3x3"])
    s3 = maxpool2x2_nhwc(np.asarray(x, np.float64))
    s3 = conv2d_nhwc(s3, *L["s3_conv1x1"])
    s3 = conv2d_nhwc(s3, *L["s3_conv3x3"])
    return [s0, s1, s2, s3]


# ---- text encoder / general attention (f64) ----------------------------------

def attention_gen(q: np.ndarray, k: np.ndarray, v: np.ndarray, heads: int, head_dim: int, scale: float,
                  causal: bool = False, bias=None) -> np.ndarray:
    """ggml_flash_attn_ext semantics in f64: per head h, softmax(scale Q_h K_h^T
    + bias_h) V_h; q [lq][>= heads*hd], k / v [lk][...]; bias broadcastable to
    [heads][lq][lk] (additive, -inf masks); causal masks keys k > q.  A query
    with every key masked gets 0."""
    q, k, v = (np.asarray(a, np.float64) for a in (q, k, v))
    lq, lk = q.shape[0], k.shape[0]
    out = np.zeros((lq, heads * head_dim), np.float64)
    b = None if bias is None else np.broadcast_to(np.asarray(bias, np.float64), (heads, lq, lk))
    for h in range(heads):
        sl = slice(h * head_dim, (h + 1) * head_dim)
        s = (q[:, sl] @ k[:, sl].T) * scale
        if b is not None:
            s = s + b[h]
        if causal:
            s = np.where(np.arange(lk)[None, :] > np.arange(lq)[:, None], -np.inf, s)
        mx = s.max(axis=1, keepdims=True)
        mx = np.where(np.isfinite(mx), mx, 0.0)
        p = np.exp(s - mx)
        den = p.sum(axis=1, keepdims=True)
        out[:, sl] = np.where(den > 0, (p @ v[:, sl]) / np.where(den > 0, den, 1.0), 0.0)
    return out.astype(np.float32)


def text_block(x: np.ndarray, blk: dict) -> np.ndarray:
    """One SAM 3 text-encoder block (src/models/sam3/text_encoder.hpp:68-150):
    x1 = x + out_proj(attn_causal(in_proj(LN1(x)))); out = x1 + fc2(GELU(fc1(LN2(x1)))),
    every quantized linear with MMQ operand semantics (staged_linear), attention
    in f64 with the causal mask and scale 1/8 (heads of 64)."""
    x = np.ascontiguousarray(x, dtype=np.float32)
    E = x.shape[1]
    heads = E // 64
    h = layer_norm(x, blk["norm1_w"], blk["norm1_b"])
    qkv = staged_linear(blk["in_proj_w"], h, blk["in_proj_b"])
    att = attention_gen(qkv[:, :E], qkv[:, E:2 * E], qkv[:, 2 * E:], heads, 64, 0.125, causal=True)
    x1 = x + staged_linear(blk["out_proj_w"], att, blk["out_proj_b"])
    h2 = layer_norm(x1, blk["norm2_w"], blk["norm2_b"])
    f = staged_linear(blk["fc1_w"], h2, blk["fc1_b"], EPILOGUE_GELU_ERF)
    return x1 + staged_linear(blk["fc2_w"], f, blk["fc2_b"])


def text_encoder(ids, token_embed: np.ndarray, pos_embed: np.ndarray, blocks: list, ln_w, ln_b, resizer_w,
                 resizer_b) -> np.ndarray:
    """sam3_build_text_encoder_graph (text_encoder.hpp:151-180): token rows +
    pos_embed, the blocks, the final LayerNorm and the quantized resizer."""
    x = (np.asarray(token_embed, np.float32)[np.asarray(ids)] + np.asarray(pos_embed, np.float32)).astype(np.float32)
    for blk in blocks:
        x = text_block(x, blk)
    return staged_linear(resizer_w, layer_norm(x, ln_w, ln_b), resizer_b)


class exact_operands:
    """Context in which every quantized linear (staged_linear, and through it
    module_linear, vit_block, text_block ...) runs over the device GEMM's
    exact f16 operands instead of GGML MMQ's decoded operands.  The distance
    between the two is the operand precision of the f16 tensor-core path; the
    device is held tightly to this mode."""

    def __enter__(self):
        _EXACT_OPERANDS[0] = True
        return self

    def __exit__(self, *exc):
        _EXACT_OPERANDS[0] = False
        return False


def module_linear(lin: dict, x: np.ndarray, rows=None, epilogue=EPILOGUE_NONE) -> np.ndarray:
    """A linear of the fusion / decoder modules: lin = {"w": f32 [n][k] (the
    decoded weight), "b": [n] or None, "quantized": bool}.  Quantized: MMQ
    operand semantics (staged_linear); dense: the F32 product in f64.  `rows`
    selects a row slice of the weight (the in_proj views)."""
    w = lin["w"] if rows is None else lin["w"][rows]
    b = None if lin["b"] is None else (lin["b"] if rows is None else lin["b"][rows])
    if lin["quantized"]:
        return staged_linear(w, x, b, epilogue)
    return dense_linear(x, w, b, gelu=epilogue == EPILOGUE_GELU_ERF).astype(np.float32)


def fusion_layer(x: np.ndarray, pos: np.ndarray, prompt: np.ndarray, prompt_bias, ly: dict, heads: int) -> np.ndarray:
    """sam3_fenc_layer_forward (src/models/sam3/fusion_encoder.hpp:38-150) with
    f64 LayerNorm / attention; ly holds norm{1,2,3}_{w,b} and the module_linear
    dicts sa_in_proj, sa_out_proj, ca_in_proj, ca_out_proj, linear1, linear2."""
    x = np.asarray(x, np.float32)
    D = x.shape[1]
    hd = D // heads
    scale = 1.0 / np.sqrt(hd)
    h = layer_norm(x, ly["norm1_w"], ly["norm1_b"])
    qk_in = (h + np.asarray(pos, np.float32)).astype(np.float32)
    qk = module_linear(ly["sa_in_proj"], qk_in, slice(0, 2 * D))
    v = module_linear(ly["sa_in_proj"], h, slice(2 * D, 3 * D))
    att = attention_gen(qk[:, :D], qk[:, D:], v, heads, hd, scale)
    x = x + module_linear(ly["sa_out_proj"], att)
    h = layer_norm(x, ly["norm2_w"], ly["norm2_b"])
    q = module_linear(ly["ca_in_proj"], h, slice(0, D))
    kv = module_linear(ly["ca_in_proj"], np.asarray(prompt, np.float32), slice(D, 3 * D))
    bias = None if prompt_bias is None else np.asarray(prompt_bias, np.float32)[None, None, :]
    att = attention_gen(q, kv[:, :D], kv[:, D:], heads, hd, scale, bias=bias)
    x = x + module_linear(ly["ca_out_proj"], att)
    h = layer_norm(x, ly["norm3_w"], ly["norm3_b"])
    f = np.maximum(module_linear(ly["linear1"], h), 0.0).astype(np.float32)
    return x + module_linear(ly["linear2"], f)


# ---- DETR decoder + scoring (src/models/sam3/detector.hpp) -------------------

def sine_dim_t() -> np.ndarray:
    """The 64 angle multipliers execution.hpp:223-226 uploads: 2 pi / 10000^(2i/128), f32."""
    i = np.arange(64, dtype=np.float32)
    return (np.float32(2.0) * np.float32(np.pi) / np.power(np.float32(10000.0), np.float32(2.0) * i / np.float32(128.0))
            ).astype(np.float32)


def sine_pos_embed_4d(ref: np.ndarray) -> np.ndarray:
    """sam3_build_sine_pos_embed_4d (detector.hpp:67-104): ref [NQ][4]
    (cx, cy, w, h); coordinates in the order cy, cx, w, h, each as 64
    (sin, cos) pairs of ref * dim_t -> [NQ][512] (f64)."""
    ref = np.asarray(ref, np.float32)
    parts = []
    for ci in (1, 0, 2, 3):
        a = (ref[:, ci:ci + 1] * sine_dim_t()[None, :]).astype(np.float64)  # the f32 product GGML forms
        pair = np.stack([np.sin(a), np.cos(a)], axis=-1).reshape(ref.shape[0], 128)
        parts.append(pair)
    return np.concatenate(parts, axis=1)


def box_rpb(ref: np.ndarray, grid: int, x0_w, x0_b, x1: dict, y0_w, y0_b, y1: dict, heads: int) -> np.ndarray:
    """sam3_compute_box_rpb (detector.hpp:160-305): the additive image
    cross-attention bias [heads][NQ + 1][grid * grid] (row 0, the presence
    token, zero).  Deltas coord - edge with coord = i / grid, log transform
    sign(8d) log2(|8d| + 1) / 3, per axis MLP Linear(2 -> 256) + ReLU, Linear(256 -> heads),
    outer sum over (h, w) with key index h * grid + w."""
    ref = np.asarray(ref, np.float64)
    nq = ref.shape[0]
    coords = (np.arange(grid, dtype=np.float32) / np.float32(grid)).astype(np.float64)
    cx, cy, w, h = ref[:, 0], ref[:, 1], ref[:, 2], ref[:, 3]

    def logt(d):
        d8 = 8.0 * d
        return np.sign(d8) * np.log2(np.abs(d8) + 1.0) / 3.0

    def mlp(lo, hi, w0, b0, l1):
        d = np.stack([logt(coords[None, :] - lo[:, None]), logt(coords[None, :] - hi[:, None])], axis=-1)  # [NQ][G][2]
        hdn = np.maximum(d @ np.asarray(w0, np.float64).T + np.asarray(b0, np.float64), 0.0)
        flat = hdn.reshape(nq * grid, -1).astype(np.float32)
        return module_linear(l1, flat).astype(np.float64).reshape(nq, grid, heads)

    rx = mlp(cx - 0.5 * w, cx + 0.5 * w, x0_w, x0_b, x1)
    ry = mlp(cy - 0.5 * h, cy + 0.5 * h, y0_w, y0_b, y1)
    bias = np.zeros((heads, nq + 1, grid * grid), np.float64)
    # key h * grid + w: ry[q][h] + rx[q][w]
    bias[:, 1:, :] = (ry.transpose(2, 0, 1)[:, :, :, None] + rx.transpose(2, 0, 1)[:, :, None, :]).reshape(
        heads, nq, grid * grid)
    return bias.astype(np.float32)


def inverse_sigmoid(x):
    x = np.clip(x, 0.0, 1.0)
    return np.log(np.clip(x, 1e-3, 1.0)) - np.log(np.clip(1.0 - x, 1e-3, 1.0))


def sigmoid(x):
    return 1.0 / (1.0 + np.exp(-np.asarray(x, np.float64)))


def mlp_chain(lins: list, x, relu_last=False):
    for j, lin in enumerate(lins):
        x = module_linear(lin, np.asarray(x, np.float32))
        if j < len(lins) - 1 or relu_last:
            x = np.maximum(x, 0.0)
    return np.asarray(x, np.float32)


def decoder_layer(q, qpos, enc, enc_pos, text, text_bias, rpb, ly: dict, heads: int):
    """sam3_ddec_layer_forward (detector.hpp:307-478): post-norm self-attention
    (norm2), text cross-attention (norm_ca_text), image cross-attention with
    the box bias (norm1), ReLU FFN (norm3)."""
    D = q.shape[1]
    hd = D // heads
    scale = 1.0 / np.sqrt(hd)
    qin = (q + qpos).astype(np.float32)
    qk = module_linear(ly["sa_in_proj"], qin, slice(0, 2 * D))
    v = module_linear(ly["sa_in_proj"], q, slice(2 * D, 3 * D))
    att = attention_gen(qk[:, :D], qk[:, D:], v, heads, hd, scale)
    q = layer_norm(q + module_linear(ly["sa_out_proj"], att), ly["norm2_w"], ly["norm2_b"])
    qin = (q + qpos).astype(np.float32)
    qq = module_linear(ly["ca_text_in_proj"], qin, slice(0, D))
    kv = module_linear(ly["ca_text_in_proj"], text, slice(D, 3 * D))
    tb = None if text_bias is None else np.asarray(text_bias, np.float32)[None, None, :]
    att = attention_gen(qq, kv[:, :D], kv[:, D:], heads, hd, scale, bias=tb)
    q = layer_norm(q + module_linear(ly["ca_text_out_proj"], att), ly["norm_ca_text_w"], ly["norm_ca_text_b"])
    qin = (q + qpos).astype(np.float32)
    kin = (np.asarray(enc, np.float32) + np.asarray(enc_pos, np.float32)).astype(np.float32)
    qq = module_linear(ly["ca_in_proj"], qin, slice(0, D))
    kk = module_linear(ly["ca_in_proj"], kin, slice(D, 2 * D))
    vv = module_linear(ly["ca_in_proj"], enc, slice(2 * D, 3 * D))
    att = attention_gen(qq, kk, vv, heads, hd, scale, bias=rpb)
    q = layer_norm(q + module_linear(ly["ca_out_proj"], att), ly["norm1_w"], ly["norm1_b"])
    f = np.maximum(module_linear(ly["linear1"], q), 0.0).astype(np.float32)
    return layer_norm(q + module_linear(ly["linear2"], f), ly["norm3_w"], ly["norm3_b"])


def decoder(enc, enc_pos, text, text_bias, text_valid, dec: dict, grid: int, heads: int):
    """sam3_build_ddec_graph + sam3_dot_product_scoring (detector.hpp:507-713):
    returns (queries_for_seg [NQ + 1][D], boxes [NQ][4], scores [NQ], presence logit)."""
    qe = np.asarray(dec["query_embed"], np.float32)
    nq, D = qe.shape
    q = np.concatenate([np.asarray(dec["presence_token"], np.float32).reshape(1, D), qe], axis=0)
    ref = sigmoid(np.asarray(dec["reference_points"], np.float32)).astype(np.float32)
    last_presence = q[:1]
    for ly in dec["layers"]:
        sine = sine_pos_embed_4d(ref).astype(np.float32)
        qpos = np.zeros((nq + 1, D), np.float32)
        qpos[1:] = mlp_chain(dec["ref_point_head"], sine)
        rpb = box_rpb(ref, grid, dec["rpb_x0_w"], dec["rpb_x0_b"], dec["rpb_x1"], dec["rpb_y0_w"], dec["rpb_y0_b"],
                      dec["rpb_y1"], heads)
        q = decoder_layer(q, qpos, enc, enc_pos, text, text_bias, rpb, ly, heads)
        last_presence = q[:1]
        normed = layer_norm(q[1:], dec["norm_w"], dec["norm_b"])
        bd = mlp_chain(dec["bbox_embed"], normed).astype(np.float64)
        ref = sigmoid(inverse_sigmoid(ref.astype(np.float64)) + bd).astype(np.float32)
    obj = layer_norm(q[1:], dec["norm_w"], dec["norm_b"])
    text = np.asarray(text, np.float32)
    tm = mlp_chain(dec["prompt_mlp"], text)
    tm = layer_norm(tm + text, dec["prompt_mlp_norm_w"], dec["prompt_mlp_norm_b"])
    valid = np.asarray(text_valid, np.float64)
    pooled = ((tm.astype(np.float64) * valid[:, None]).sum(axis=0) / tm.shape[0]).astype(np.float32)[None, :]
    pp = module_linear(dec["prompt_proj"], pooled).astype(np.float64)
    hs = module_linear(dec["hs_proj"], obj).astype(np.float64)
    scores = np.clip((hs @ pp[0]) / np.sqrt(D), -12.0, 12.0).astype(np.float32)
    pres = layer_norm(last_presence, dec["presence_norm_w"], dec["presence_norm_b"])
    presence = float(mlp_chain(dec["presence_head"], pres)[0, 0])
    return np.concatenate([last_presence, obj], axis=0), ref, scores, presence


# ---- image positional encoding, geometry encoder, segmentation head -----------

def sine_pe_2d(h: int, w: int, d: int) -> np.ndarray:
    """sam3_sinusoidal_pe_2d (src/models/sam3/vision.hpp:39-75), the image
    positional encoding, [h * w][d] f32 rows (token y * w + x): channel i < d/2
    is the y encoding, channel d/2 + i the x encoding; pos = (p + 1) / n * 2 pi,
    dim_t = 10000^((i & ~1) / (d/2)), sin at even i, cos at odd i.  Evaluated
    in f64 from the f32 arguments the reference forms."""
    half = d // 2
    i = np.arange(half)
    dim_t = np.power(np.float32(10000.0), (i & ~1).astype(np.float32) / np.float32(half)).astype(np.float32)
    scale = np.float32(2.0 * np.pi)
    py = ((np.arange(h, dtype=np.float32) + 1) / np.float32(h) * scale).astype(np.float32)
    px = ((np.arange(w, dtype=np.float32) + 1) / np.float32(w) * scale).astype(np.float32)
    ay = (py[:, None] / dim_t[None, :]).astype(np.float32).astype(np.float64)  # [h][half]
    ax = (px[:, None] / dim_t[None, :]).astype(np.float32).astype(np.float64)  # [w][half]
    even = (i % 2 == 0)[None, :]
    vy = np.where(even, np.sin(ay), np.cos(ay))
    vx = np.where(even, np.sin(ax), np.cos(ax))
    out = np.empty((h, w, d), np.float64)
    out[:, :, :half] = vy[:, None, :]
    out[:, :, half:] = vx[None, :, :]
    return out.reshape(h * w, d).astype(np.float32)


def geometry_encoder(image: np.ndarray, pos: np.ndarray, ge: dict, heads: int = 8) -> np.ndarray:
    """sam3_build_geom_enc_graph (src/models/sam3/prompt_encoder.hpp:44-160)
    for a text-only prompt: the learned CLS token through final_proj and norm,
    three pre-norm layers (self-attention over the single token, cross-attention
    to the image with keys image + pos, ReLU FFN), then encode_norm.  Returns
    the geometry prompt token [1][D] f32."""
    cls = np.asarray(ge["cls"], np.float32).reshape(1, -1)
    D = cls.shape[1]
    hd = D // heads
    scale = 1.0 / np.sqrt(hd)
    x = layer_norm(module_linear(ge["final_proj"], cls), ge["norm_w"], ge["norm_b"])
    kin = (np.asarray(image, np.float32) + np.asarray(pos, np.float32)).astype(np.float32)
    for ly in ge["layers"]:
        xn = layer_norm(x, ly["norm1_w"], ly["norm1_b"])
        qkv = module_linear(ly["sa_in_proj"], xn)
        att = attention_gen(qkv[:, :D], qkv[:, D:2 * D], qkv[:, 2 * D:], heads, hd, scale)
        x = (x.astype(np.float64) + module_linear(ly["sa_out_proj"], att)).astype(np.float32)
        xn = layer_norm(x, ly["norm2_w"], ly["norm2_b"])
        q = module_linear(ly["ca_in_proj"], xn, slice(0, D))
        k = module_linear(ly["ca_in_proj"], kin, slice(D, 2 * D))
        v = module_linear(ly["ca_in_proj"], image, slice(2 * D, 3 * D))
        att = attention_gen(q, k, v, heads, hd, scale)
        x = (x.astype(np.float64) + module_linear(ly["ca_out_proj"], att)).astype(np.float32)
        xn = layer_norm(x, ly["norm3_w"], ly["norm3_b"])
        f = np.maximum(module_linear(ly["linear1"], xn), 0.0).astype(np.float32)
        x = (x.astype(np.float64) + module_linear(ly["linear2"], f)).astype(np.float32)
    return layer_norm(x, ge["encode_norm_w"], ge["encode_norm_b"])


def group_norm_nhwc(x: np.ndarray, groups: int, w, b, eps: float = 1e-5) -> np.ndarray:
    """ggml_group_norm(groups, eps) of an NHWC map followed by the per-channel
    affine (src/models/sam3/mask_decoder.hpp:75-83): statistics over all pixels
    and the C / groups channels of a group, f64."""
    x = np.asarray(x, np.float64)
    H, W, C = x.shape
    g = x.reshape(H * W, groups, C // groups)
    mean = g.mean(axis=(0, 2), keepdims=True)
    var = ((g - mean) ** 2).mean(axis=(0, 2), keepdims=True)
    y = ((g - mean) / np.sqrt(var + eps)).reshape(H, W, C)
    return y * np.asarray(w, np.float64) + np.asarray(b, np.float64)


def upsample2x_nhwc(x: np.ndarray) -> np.ndarray:
    """ggml_upscale(x, 2, NEAREST): out[y][x] = in[y / 2][x / 2]."""
    return np.repeat(np.repeat(np.asarray(x), 2, axis=0), 2, axis=1)


def seg_head(enc: np.ndarray, fpn0: np.ndarray, fpn1: np.ndarray, queries: np.ndarray, prompt: np.ndarray,
             prompt_bias, sh: dict, grid: int, heads: int = 8) -> np.ndarray:
    """sam3_build_seg_head_graph + sam3_pixel_decoder
    (src/models/sam3/mask_decoder.hpp:57-202): prompt cross-attention on the
    fusion output (residual, no positions), pixel decoder over (fusion output,
    fpn1, fpn0) with nearest 2x upsampling, 3x3 conv, GroupNorm(8) and ReLU,
    the 1x1 instance head, the 3-layer mask-embedding MLP on the object queries
    and the einsum: mask logits [Q][(4 grid)^2] (f64)."""
    enc = np.asarray(enc, np.float32)
    D = enc.shape[1]
    hd = D // heads
    ln = layer_norm(enc, sh["cross_attn_norm_w"], sh["cross_attn_norm_b"])
    q = module_linear(sh["ca_in_proj"], ln, slice(0, D))
    kv = module_linear(sh["ca_in_proj"], prompt, slice(D, 3 * D))
    tb = None if prompt_bias is None else np.asarray(prompt_bias, np.float32)[None, None, :]
    att = attention_gen(q, kv[:, :D], kv[:, D:], heads, hd, 1.0 / np.sqrt(hd), bias=tb)
    enc = (enc.astype(np.float64) + module_linear(sh["ca_out_proj"], att)).astype(np.float32)
    prev = enc.reshape(grid, grid, D)
    for i, fpn in enumerate((fpn1, fpn0)):
        size = grid * (2 << i)
        merged = (np.asarray(fpn, np.float32).reshape(size, size, D) + upsample2x_nhwc(prev)).astype(np.float32)
        y = conv2d_nhwc(merged, sh["conv_w"][i], sh["conv_b"][i])
        prev = np.maximum(group_norm_nhwc(y, 8, sh["norm_w"][i], sh["norm_b"][i]), 0.0).astype(np.float32)
    pe = conv2d_nhwc(prev, sh["instance_w"], sh["instance_b"], stride=1, pad=0).reshape(-1, D)
    me = mlp_chain(sh["mask_embed"], queries).astype(np.float64)
    return me @ pe.T
