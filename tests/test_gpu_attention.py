"""GPU parity of K3 (RoPE + windowed / global ViT attention) against the f64 oracle.

The tests at the top exercise the F16 compute mode (the tcgen05 kernel); the
ones at the end cover both modes, the reference's RoPE patterns and its
closed-form attention probe.

Reference semantics: src/models/sam3/vision.hpp:100-148 (RoPE), :170-227
(window partition, flash_attn_ext with scale 1/8, window unpartition).  The
kernel computes on f16 operands with f32 accumulation and an f32 online
softmax; the bar is cosine >= 0.9999 and normalized max error <= 2e-3 against
the f64 oracle over the same f32 qkv input.  The f16 rounding of Q and K
makes the logit error grow with the logit magnitude (|s| * 2^-11): at logit
standard deviations around 36 the normalized error reaches ~9e-3, while the
scales exercised here (and LayerNorm-fed activations) stay near 5e-4.
"""
import numpy as np
import pytest

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu

COS_MIN = 0.9999
MAX_REL = 2e-3


@pytest.fixture(scope="module")
def samq():
    import samq as module
    assert torch.cuda.is_available(), "GPU tests need a CUDA device"
    module.init(0)
    return module


def metrics(y, ref):
    y64, r64 = y.astype(np.float64).ravel(), ref.astype(np.float64).ravel()
    cos = float(np.dot(y64, r64) / (np.linalg.norm(y64) * np.linalg.norm(r64)))
    return cos, float(np.max(np.abs(y64 - r64)) / np.max(np.abs(r64)))


def run(samq, qkv, grid_w, grid_h, heads, window, freqs):
    E = heads * 64
    out = torch.full((grid_w * grid_h, E), -5.0, dtype=torch.float32, device="cuda")
    samq.vit_attention(torch.from_numpy(qkv).cuda(), qkv.shape[1], grid_w, grid_h, heads, window,
                       torch.from_numpy(freqs).cuda(), out, E, compute=samq.COMPUTE_F16)
    samq.check(0)
    return out.cpu().numpy()


@pytest.mark.parametrize("grid,heads,window,scale", [
    (24, 2, 0, 1.0),     # global, 576 tokens: 4.5 key blocks (masked tail)
    (48, 2, 24, 1.0),    # 4 windows of 576
    (16, 3, 8, 2.0),     # 4 windows of 64 tokens: a single partial key block
    (24, 1, 0, 2.0),     # logits ~4x larger: online-softmax rescaling across blocks
])
def test_attention_parity_small(samq, oracle, grid, heads, window, scale):
    rng = np.random.default_rng(grid * 10 + heads + window)
    E = heads * 64
    qkv = (rng.normal(0, 1, (grid * grid, 3 * E)) * scale).astype(np.float32)
    positions = window * window if window else grid * grid
    freqs = oracle.rope_freqs(positions, seed=grid)
    y = run(samq, qkv, grid, grid, heads, window, freqs)
    ref = oracle.vit_attention(qkv, grid, grid, heads, 64, window, freqs)
    cos, rel = metrics(y, ref)
    assert cos >= COS_MIN and rel <= MAX_REL, (cos, rel)


@pytest.mark.parametrize("window", [24, 0])
def test_attention_full_size_sampled_rows(samq, oracle, window):
    """SAM 3 ViT geometry: 72x72 tokens, 16 heads, windowed (24) or global."""
    rng = np.random.default_rng(window)
    grid, heads = 72, 16
    E = heads * 64
    qkv = rng.normal(0, 1, (grid * grid, 3 * E)).astype(np.float32)
    positions = window * window if window else grid * grid
    freqs = oracle.rope_freqs(positions, seed=3)
    y = run(samq, qkv, grid, grid, heads, window, freqs)
    rows = np.sort(rng.choice(grid * grid, 40, replace=False))
    rows[-1] = grid * grid - 1
    ref = oracle.vit_attention(qkv, grid, grid, heads, 64, window, freqs, rows=rows)
    cos, rel = metrics(y[rows], ref)
    assert cos >= COS_MIN and rel <= MAX_REL, (cos, rel)
    assert np.isfinite(y).all()


# ---- compute modes, RoPE patterns and the closed-form attention probe -------

@pytest.mark.parametrize("grid,heads,window", [(24, 2, 0), (48, 2, 24), (16, 3, 8)])
def test_attention_f32_mode_parity(samq, oracle, grid, heads, window):
    """SAMQ_COMPUTE_F32 keeps Q, K, V and P in f32: against the f64 oracle the
    error is at f32 level (cosine >= 1 - 1e-10, normalized max error <= 1e-5),
    and the F16 mode stays within its own 2e-3 bar on the same input."""
    rng = np.random.default_rng(700 + grid + window)
    E = heads * 64
    qkv = rng.normal(0, 1, (grid * grid, 3 * E)).astype(np.float32)
    freqs = oracle.rope_freqs(window * window if window else grid * grid, seed=grid + 1)
    ref = oracle.vit_attention(qkv, grid, grid, heads, 64, window, freqs)
    for compute, cos_min, rel_max in ((samq.COMPUTE_F32, 1 - 1e-10, 1e-5), (samq.COMPUTE_F16, COS_MIN, MAX_REL)):
        out = torch.full((grid * grid, E), -5.0, dtype=torch.float32, device="cuda")
        samq.vit_attention(torch.from_numpy(qkv).cuda(), 3 * E, grid, grid, heads, window,
                           torch.from_numpy(freqs).cuda(), out, E, compute=compute)
        samq.check(0)
        cos, rel = metrics(out.cpu().numpy(), ref)
        assert cos >= cos_min and rel <= rel_max, (compute, cos, rel)


def _rope_input(tokens, heads, batch, salt):
    """tests/runtime/ggml/test_rope.cpp:23-40 (make_input): [head_batch][token][64]."""
    hb = np.arange(heads * batch)[:, None, None].astype(np.float64)
    tok = np.arange(tokens)[None, :, None].astype(np.float64)
    pair = np.arange(32)[None, None, :].astype(np.float64)
    phase = 0.17 * (hb + 1) + 0.011 * (tok + 1) + 0.031 * (pair + 1) + salt
    x = np.empty((heads * batch, tokens, 64), dtype=np.float32)
    x[..., 0::2] = (0.1234567 + 0.7 * np.sin(phase) + 0.01 * hb).astype(np.float32)
    x[..., 1::2] = (-0.7654321 + 0.6 * np.cos(phase * 0.73) - 0.005 * hb).astype(np.float32)
    x[0, 0, 0] = np.float32(0.1234567) + np.float32(salt)
    x[0, 0, 1] = np.float32(-0.7654321) - np.float32(salt)
    return x


def _rope_freqs(tokens, pattern, salt):
    """tests/runtime/ggml/test_rope.cpp:42-68 (make_frequencies): [token][32][2]."""
    f = np.empty((tokens, 32, 2), dtype=np.float32)
    tok = np.arange(tokens)[:, None]
    pair = np.arange(32)[None, :]
    if pattern == "identity":
        f[..., 0], f[..., 1] = 1.0, 0.0
    elif pattern == "quarter_turn":
        f[..., 0], f[..., 1] = 0.0, 1.0
    elif pattern == "arbitrary":
        phase = 0.19 * (pair + 1) + 0.027 * (tok + 1) + 0.013 * (((pair + 3) * (tok + 5)) % 19) + salt
        f[..., 0] = (0.71 + 0.13 * np.cos(phase)).astype(np.float32)
        f[..., 1] = (-0.23 + 0.17 * np.sin(phase * 0.61)).astype(np.float32)
    else:
        phase = 0.21 * (pair + 1) + 0.0007 * (tok + 1) + 0.003 * ((pair + 2) * (tok % 97 + 1)) + salt
        f[..., 0] = np.cos(phase).astype(np.float32)
        f[..., 1] = np.sin(phase).astype(np.float32)
    return f


@pytest.mark.parametrize("tokens,heads,batch,patterns", [
    (1, 1, 1, ("identity", "quarter_turn")),
    (37, 3, 2, ("arbitrary", "arbitrary", "identity", "quarter_turn")),
    (576, 16, 1, ("trigonometric",)),
    (5184, 16, 1, ("trigonometric",)),
])
def test_rope_matches_reference_patterns(samq, tokens, heads, batch, patterns):
    """The shapes and tables of tests/runtime/ggml/test_rope.cpp:150-170 through
    samq_vit_rope_v1: within 2e-6 (1 + |expected|) of the scalar complex
    formula (test_rope.cpp:70-93), and bit-identical to GGML's f32 op sequence
    (two products, then one subtraction / addition, each rounded to f32)."""
    previous = None
    for p, pattern in enumerate(patterns):
        salt = np.float32(p * 0.137)
        x = _rope_input(tokens, heads, batch, float(salt))
        f = _rope_freqs(tokens, pattern, float(salt))
        xd = torch.from_numpy(x).cuda()
        out = torch.empty_like(xd)
        samq.vit_rope(xd, tokens, heads * batch, torch.from_numpy(f).cuda(), out)
        samq.check(0)
        got = out.cpu().numpy()
        re, im = x[..., 0::2], x[..., 1::2]
        c, s = f[None, ..., 0], f[None, ..., 1]
        ggml_re = np.subtract(np.multiply(re, c, dtype=np.float32), np.multiply(im, s, dtype=np.float32),
                              dtype=np.float32)
        ggml_im = np.add(np.multiply(re, s, dtype=np.float32), np.multiply(im, c, dtype=np.float32), dtype=np.float32)
        np.testing.assert_array_equal(got[..., 0::2], ggml_re)
        np.testing.assert_array_equal(got[..., 1::2], ggml_im)
        r64, i64 = re.astype(np.float64), im.astype(np.float64)
        exp_re = r64 * c.astype(np.float64) - i64 * s.astype(np.float64)
        exp_im = r64 * s.astype(np.float64) + i64 * c.astype(np.float64)
        tol = 2e-6 * (1.0 + np.maximum(np.abs(exp_re), np.abs(exp_im)))
        assert np.all(np.abs(got[..., 0::2] - exp_re) <= tol) and np.all(np.abs(got[..., 1::2] - exp_im) <= tol)
        if previous is not None:  # fresh inputs change the output (test_rope.cpp:128-133)
            assert np.any(np.abs(got - previous) > 1e-5)
        previous = got


@pytest.mark.parametrize("grid_w,grid_h,window", [(16, 8, 0), (24, 24, 0), (72, 72, 0), (48, 48, 24)])
def test_attention_precision_probe(samq, grid_w, grid_h, window):
    """The closed-form probe of tests/runtime/ggml/test_precision.cpp:68-126 at
    head_dim 64: Q = 1.0003 + (query % 7) 1e-5 in every channel, half of the
    keys K = 0.0625 / V = 1 and the other half K = -0.0625 / V = -1, identity
    RoPE, so each output channel is tanh(64 * 0.0625 * (1/8) * q).  The F32
    mode must be within 1e-5 (the reference's precise bar); the F16 mode loses
    Q's low bits to f16 (the reference measured 1.18e-4 for its half-Q path)
    and is only bounded by 5e-4."""
    tokens = grid_w * grid_h
    group_n = window * window if window else tokens
    qkv = np.empty((tokens, 3 * 64), dtype=np.float32)
    t = np.arange(tokens)
    # position inside the token's attention group (window-local raster, or global)
    local = ((t // grid_w) % window) * window + (t % grid_w) % window if window else t
    qv = (np.float32(1.0003) + (local % 7).astype(np.float32) * np.float32(0.00001)).astype(np.float32)
    positive = local < group_n // 2
    qkv[:, :64] = qv[:, None]
    qkv[:, 64:128] = np.where(positive, np.float32(0.0625), np.float32(-0.0625))[:, None]
    qkv[:, 128:] = np.where(positive, np.float32(1.0), np.float32(-1.0))[:, None]
    freqs = np.zeros((group_n, 32, 2), dtype=np.float32)
    freqs[..., 0] = 1.0
    expected = np.tanh(64 * 0.0625 * 0.125 * qv.astype(np.float64))[:, None]
    errors = {}
    for compute in (samq.COMPUTE_F32, samq.COMPUTE_F16):
        out = torch.empty((tokens, 64), dtype=torch.float32, device="cuda")
        samq.vit_attention(torch.from_numpy(qkv).cuda(), 3 * 64, grid_w, grid_h, 1, window,
                           torch.from_numpy(freqs).cuda(), out, 64, compute=compute)
        samq.check(0)
        got = out.cpu().numpy().astype(np.float64)
        assert np.all(np.isfinite(got))
        errors[compute] = float(np.abs(got - expected).max())
    print("precision probe", grid_w, grid_h, window, errors)
    assert errors[samq.COMPUTE_F32] <= 1e-5, errors
    assert errors[samq.COMPUTE_F16] <= 5e-4, errors
