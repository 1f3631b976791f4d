"""The CPU oracle pinned against golden vectors and the reference's test rules.

Sources: gguf-py 0.19.0 fixtures (tests/golden/make_golden.py), the MMQ scale
known-answer test (tests/runtime/ggml/test_cuda_q8_mmq_scale.cpp:33-93 in the
reference), the CPU matmul tolerance 5e-4 + 5e-5|ref| against decoded
operands (tools/benchmark/cpu_quantized_matmul.hpp:195-222) and the
quantized-math tolerance 0.025 + 0.005|ref| (tests/runtime/ggml/
test_quantization.cpp:469-494).
"""
import numpy as np
import pytest

from conftest import load_golden


def test_f16_conversion_matches_numpy(oracle):
    rng = np.random.default_rng(1)
    vals = np.concatenate([
        rng.normal(0, 1, 4000), rng.normal(0, 1e-5, 2000), rng.normal(0, 3e4, 2000),
        [0.0, -0.0, 65504.0, 65519.99, 65520.0, 1e-8, 5.96e-8, 2.98e-8, 6.1e-5, np.inf, -np.inf],
    ]).astype(np.float32)
    ours = np.array([oracle.lib().oracle_f32_to_f16(float(v)) for v in vals], dtype=np.uint16)
    np.testing.assert_array_equal(ours, vals.astype(np.float16).view(np.uint16))
    halves = np.arange(0, 65536, 7, dtype=np.uint16)
    halves = halves[(halves & 0x7c00) != 0x7c00]
    back = np.array([oracle.lib().oracle_f16_to_f32(int(h)) for h in halves], dtype=np.float32)
    np.testing.assert_array_equal(back, halves.view(np.float16).astype(np.float32))


def test_q8_0_quantizer_is_gguf_bit_exact(oracle):
    g = load_golden("q8_0_quantize")
    np.testing.assert_array_equal(oracle.quantize_q8_0(g["source"]), g["blocks"])


@pytest.mark.parametrize("name", ["q8_0", "q4_k", "q5_k", "q6_k"])
def test_dequantize_is_gguf_bit_exact(oracle, name):
    g = load_golden(f"dequant_{name}")
    qtype = oracle.NAME_TYPES[name.upper()]
    ours = oracle.dequantize(qtype, g["blocks"], g["values"].size)
    np.testing.assert_array_equal(ours.view(np.uint32), g["values"].view(np.uint32))


def test_q8_staging_matches_verified_fixture(oracle):
    g = load_golden("q8_staging")
    np.testing.assert_array_equal(oracle.quantize_q8_1(g["source"]), g["q8_1"])
    np.testing.assert_array_equal(oracle.quantize_mmq_d4(g["source"]), g["mmq_d4"])


def mmq_kat_input():
    """Inputs of the reference MMQ scale KAT (test_cuda_q8_mmq_scale.cpp:33-41)."""
    width, rows = 160, 65
    x = np.zeros((rows, width), dtype=np.float32)
    x[0, 0] = 3.0e38
    x[1, 32] = -3.0e38
    x[2, 64] = 2000.0
    x[2, 80] = -800.0
    x[3, 128] = -2000.0
    return x


def check_mmq_kat(x, payload):
    """Assertions of test_cuda_q8_mmq_scale.cpp:59-92 on a D4 payload."""
    rows, width = x.shape
    blocks = payload.reshape(4, rows, 144)
    for b in range(4):
        for r in range(rows):
            scales = blocks[b, r, :16].copy().view(np.float32)
            codes = blocks[b, r, 16:].view(np.int8)
            assert np.all((codes >= -127) & (codes <= 127))
            for s in range(4):
                lo, hi = b * 128 + s * 32, b * 128 + s * 32 + 32
                seg = x[r, lo:min(hi, width)] if lo < width else np.zeros(0, np.float32)
                maximum = float(np.max(np.abs(seg.astype(np.float64)))) if seg.size else 0.0
                expected = np.float32(maximum / 127.0)
                if expected == 0:
                    assert scales[s] == 0
                else:
                    ulp = float(np.spacing(expected))
                    assert np.isfinite(scales[s]) and scales[s] >= 0
                    assert abs(float(scales[s]) - maximum / 127.0) <= 4 * ulp
    assert blocks[0, 0, 16 + 0].view(np.int8) == 127
    assert blocks[0, 1, 16 + 32].view(np.int8) == -127
    assert blocks[0, 2, 16 + 64].view(np.int8) == 127
    assert blocks[0, 2, 16 + 80].view(np.int8) == -51
    assert blocks[1, 3, 16 + 0].view(np.int8) == -127


def test_mmq_d4_known_answers(oracle):
    x = mmq_kat_input()
    check_mmq_kat(x, oracle.quantize_mmq_d4(x))


def test_q8_1_rules_hold_on_random_rows(oracle):
    """Independent restatement of verify_q8_rhs_staging.check_blocks without allowances."""
    rng = np.random.default_rng(7)
    x = (rng.normal(0, 1, (37, 256)) * rng.uniform(0.01, 100, (37, 1))).astype(np.float32)
    payload = oracle.quantize_q8_1(x).reshape(-1, 36)
    vals = x.reshape(-1, 32)
    scale = payload[:, :2].copy().view(np.float16).reshape(-1)
    amax = np.max(np.abs(vals), axis=1).astype(np.float64)
    np.testing.assert_array_equal(scale, (amax / 127.0).astype(np.float32).astype(np.float16))
    codes = payload[:, 4:].view(np.int8).astype(np.int64)
    target = vals.astype(np.float64) * 127.0 / amax[:, None]
    assert np.all(np.abs(codes - target) <= 0.5 + 1e-4)
    lanes = np.arange(32)
    red = vals.copy()
    for off in (16, 8, 4, 2, 1):
        red = (red + red[:, lanes ^ off]).astype(np.float32)
    np.testing.assert_array_equal(payload[:, 2:4].copy().view(np.float16).reshape(-1), red[:, 0].astype(np.float16))


@pytest.mark.parametrize("qtype", [8, 12, 13, 14])
def test_packets_round_trip_and_layout(oracle, qtype):
    rng = np.random.default_rng(qtype)
    for n, k in [(1, 256), (130, 512), (257, 1024)]:
        rows = oracle.quantize(qtype, rng.normal(0, 0.02, (n, k)).astype(np.float32))
        packets = oracle.pack_packets(qtype, k, n, rows)
        assert packets.size == (n + 127) // 128 * ((k + 63) // 64) * oracle.lib().oracle_packet_bytes(qtype)
        np.testing.assert_array_equal(oracle.unpack_packets(qtype, k, n, packets), rows)


def test_q8_0_packets_with_half_chunk(oracle):
    rng = np.random.default_rng(3)
    for k in (32, 96, 4736):
        rows = oracle.quantize(8, rng.normal(0, 0.02, (5, k)).astype(np.float32))
        p = oracle.pack_packets(8, k, 5, rows)
        np.testing.assert_array_equal(oracle.unpack_packets(8, k, 5, p), rows)


@pytest.mark.parametrize("qtype", [8, 12, 13, 14])
def test_weight_f16_is_rounded_dequant(oracle, qtype):
    rng = np.random.default_rng(11)
    n, k = 9, 512
    rows = oracle.quantize(qtype, rng.normal(0, 0.02, (n, k)).astype(np.float32))
    ref = oracle.dequantize(qtype, rows, n * k).reshape(n, k).astype(np.float16)
    np.testing.assert_array_equal(oracle.weight_f16(qtype, k, n, rows).view(np.uint16), ref.view(np.uint16))


def test_act_f16_is_rounded_q8_1_decode(oracle):
    rng = np.random.default_rng(5)
    x = rng.normal(0, 2, (13, 320)).astype(np.float32)
    dec = oracle.q8_1_decode(oracle.quantize_q8_1(x), 13, 320)
    np.testing.assert_array_equal(oracle.act_f16(x).view(np.uint16), dec.astype(np.float16).view(np.uint16))


def _decoded_rhs(oracle, qtype, x):
    if qtype == 8:
        return oracle.dequantize(8, oracle.quantize_q8_0(x), x.size).reshape(x.shape)
    q = oracle.quantize_q8_k(x).reshape(-1, 292)
    d = q[:, :4].copy().view(np.float32)
    return (d * q[:, 4:260].view(np.int8).astype(np.float32)).reshape(x.shape)


@pytest.mark.parametrize("qtype", [8, 12, 13, 14])
@pytest.mark.parametrize("m", [1, 8, 17])
def test_cpu_linear_matches_decoded_reference(oracle, qtype, m):
    """tools/benchmark/cpu_quantized_matmul.hpp:195-222 tolerance."""
    rng = np.random.default_rng(100 + qtype + m)
    n, k = 48, 1024
    w = rng.normal(0, 0.02, (n, k)).astype(np.float32)
    rows = oracle.quantize(qtype, w)
    x = rng.normal(0, 1, (m, k)).astype(np.float32)
    x[0, 3] = 17.1   # outlier scenario (cpu_quantized_matmul.hpp:70-75)
    y = oracle.cpu_linear(qtype, rows, k, n, x, threads=2)
    ref = oracle.gemm_f64(oracle.dequantize(qtype, rows, n * k).reshape(n, k), _decoded_rhs(oracle, qtype, x))
    assert np.all(np.abs(y - ref) <= 5e-4 + 5e-5 * np.abs(ref))


def test_cpu_linear_q8_0_wide_k_and_epilogue(oracle):
    rng = np.random.default_rng(9)
    n, k, m = 17, 4736, 3
    rows = oracle.quantize(8, rng.normal(0, 0.02, (n, k)).astype(np.float32))
    x = rng.normal(0, 1, (m, k)).astype(np.float32)
    bias = rng.normal(0, 0.1, n).astype(np.float32)
    y = oracle.cpu_linear(8, rows, k, n, x, bias=bias, epilogue=oracle.EPILOGUE_GELU_ERF, threads=2)
    ref = oracle.gemm_f64(oracle.dequantize(8, rows, n * k).reshape(n, k), _decoded_rhs(oracle, 8, x),
                          bias=bias, epilogue=oracle.EPILOGUE_GELU_ERF)
    assert np.all(np.abs(y - ref) <= 5e-4 + 5e-5 * np.abs(ref))


def test_cpu_linear_zero_input(oracle):
    rows = oracle.quantize(12, np.ones((16, 256), np.float32) * 0.01)
    y = oracle.cpu_linear(12, rows, 256, 16, np.zeros((4, 256), np.float32), threads=1)
    assert np.all(y == 0)


def test_gemm_f64_epilogue(oracle):
    rng = np.random.default_rng(2)
    w = rng.normal(0, 0.1, (5, 64)).astype(np.float32)
    x = rng.normal(0, 1, (3, 64)).astype(np.float32)
    b = rng.normal(0, 0.1, 5).astype(np.float32)
    y = oracle.gemm_f64(w, x, bias=b, epilogue=oracle.EPILOGUE_GELU_ERF)
    ref = oracle.gelu_erf(x.astype(np.float64) @ w.astype(np.float64).T + b)
    np.testing.assert_allclose(y, ref, rtol=1e-6, atol=1e-7)


def test_kquant_packer_is_close_to_source(oracle):
    """Own packer sanity: decoded weights track the source within format noise."""
    rng = np.random.default_rng(4)
    w = rng.normal(0, 0.02, (32, 1024)).astype(np.float32)
    for qtype, bound in [(12, 0.12), (13, 0.06), (14, 0.04)]:
        dq = oracle.dequantize(qtype, oracle.quantize(qtype, w), w.size).reshape(w.shape)
        assert np.linalg.norm(dq - w) / np.linalg.norm(w) < bound


# ---- ViT window partition / attention restatements ---------------------------

def _iota_grid(channels, width, height):
    """1, 2, 3, ... in GGML [C, W, H] order (channels fastest) as raster token rows."""
    return np.arange(1, channels * width * height + 1, dtype=np.float32).reshape(height * width, channels)


@pytest.mark.parametrize("shape,golden", [
    ((2, 3, 2, 2), [1, 2, 3, 4, 7, 8, 9, 10, 5, 6, 0, 0, 11, 12, 0, 0]),
    ((1, 3, 3, 2), [1, 2, 4, 5, 3, 0, 6, 0, 7, 8, 0, 0, 9, 0, 0, 0]),
])
def test_win_part_matches_reference_golden_layouts(oracle, shape, golden):
    """The handwritten layouts of tests/runtime/ggml/test_window.cpp:44-51
    (channel order, window order, zero padding) for ggml_win_part."""
    c, w, h, win = shape
    x = _iota_grid(c, w, h)
    parts = oracle.win_part(x, w, h, win)
    np.testing.assert_array_equal(parts.ravel(), np.asarray(golden, dtype=np.float32))
    np.testing.assert_array_equal(oracle.win_unpart(parts, w, h, win), x)


@pytest.mark.parametrize("shape", [(3, 1, 1, 4), (37, 7, 5, 4), (33, 2, 5, 1), (8, 72, 72, 24)])
def test_win_part_round_trip(oracle, shape):
    """The other shapes of test_window.cpp:54-56: win_unpart restores the image
    exactly, and every non-padding slot holds its own token."""
    c, w, h, win = shape
    x = _iota_grid(c, w, h)
    parts = oracle.win_part(x, w, h, win)
    nx, ny = -(-w // win), -(-h // win)
    assert parts.shape == (nx * ny, win * win, c)
    np.testing.assert_array_equal(oracle.win_unpart(parts, w, h, win), x)
    idx = oracle.win_part_index(w, h, win)
    assert np.count_nonzero(idx >= 0) == w * h and np.all(parts[idx < 0] == 0)


def test_attention_restatements_agree(oracle):
    """The numpy attention (used by the block oracle) and the C one
    (oracle_vit_attention) are independent restatements of the same graph."""
    rng = np.random.default_rng(3)
    for grid, heads, window in ((16, 2, 8), (12, 1, 0)):
        E = heads * 64
        qkv = rng.normal(0, 1, (grid * grid, 3 * E)).astype(np.float32)
        freqs = oracle.rope_freqs(window * window if window else grid * grid, seed=grid)
        a = oracle.attention_np(qkv, grid, grid, heads, window, freqs)
        b = oracle.vit_attention(qkv, grid, grid, heads, 64, window, freqs)
        np.testing.assert_allclose(a, b, rtol=0, atol=2e-6)
        rows = np.array([0, 5, grid * grid - 1])
        np.testing.assert_array_equal(oracle.attention_np(qkv, grid, grid, heads, window, freqs, rows=rows), a[rows])


def test_rope_matches_reference_scalar_formula(oracle):
    """sam3_apply_rope against the independent scalar complex formula of
    tests/runtime/ggml/test_rope.cpp:76-93, with its identity and quarter-turn
    tables: (re cos - im sin, re sin + im cos) within 2e-6 (1 + |expected|)."""
    rng = np.random.default_rng(0)
    x = rng.normal(0, 1, (37, 64)).astype(np.float32)
    for c, s in ((1.0, 0.0), (0.0, 1.0)):
        f = np.zeros((37, 32, 2), np.float32)
        f[..., 0], f[..., 1] = c, s
        out = oracle.rope64(x, f)
        re, im = x[:, 0::2].astype(np.float64), x[:, 1::2].astype(np.float64)
        exp_re, exp_im = re * c - im * s, re * s + im * c
        tol = 2e-6 * (1 + np.maximum(np.abs(exp_re), np.abs(exp_im)))
        assert np.all(np.abs(out[:, 0::2] - exp_re) <= tol) and np.all(np.abs(out[:, 1::2] - exp_im) <= tol)
