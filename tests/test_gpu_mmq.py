"""The quantized linear with GGML MMQ's exact arithmetic (samq_linear_mmq_v1,
csrc/gemm_mmq.cu): activations staged with the MMQ-D4 rule
(tools/validation/verify_q8_mmq_rhs_staging.py:24-67: f32 scale amax / 127,
codes round(x * 127 / amax)), Q8_0 weight codes and f16 scales, the integer
block dots on the tensor cores and the per-block rescale in f32
(verify_q8_mmq_dots.py:54-105).

Reference: the f64 product of the oracle's D4-staged operands (oracle
quantize_mmq_d4, pinned to the reference's own verifier) and the decoded Q8_0
weights.  Only f32 rounding separates the two, so the bar is tight: max error
<= 2e-6 of max |ref| (+ GELU on the same sums).  Both code variants (f16 codes
on kind::f16, int8 codes on kind::i8) are checked.  Activations far beyond the
f16 range (amax 1e20) stay exact (no operand range limit); a non-finite
activation is reported through samq_check_v1.
"""
import numpy as np
import pytest
import torch

import samq
from oracle import oracle as o

pytestmark = pytest.mark.gpu


def d4_decode(blob, rows, k):
    """[block of 128][row] x {f32 d[4], int8 q[128]} -> decoded [rows][k] f64."""
    padded = (k + 511) // 512 * 512
    b = np.frombuffer(blob.tobytes(), dtype=np.uint8).reshape(padded // 128, rows, 144)
    d = b[:, :, :16].copy().view(np.float32).reshape(padded // 128, rows, 4)
    q = b[:, :, 16:].view(np.int8).reshape(padded // 128, rows, 4, 32).astype(np.float64)
    dec = (q * d[..., None].astype(np.float64)).reshape(padded // 128, rows, 128)
    return dec.transpose(1, 0, 2).reshape(rows, padded)[:, :k]


def reference(w32, x, bias=None, gelu=False):
    xd = d4_decode(o.quantize_mmq_d4(x), x.shape[0], x.shape[1])
    y = xd @ w32.astype(np.float64).T
    if bias is not None:
        y += bias.astype(np.float64)
    return o.gelu_erf64(y) if gelu else y


def run(w, x, bias=None, epilogue=0):
    m, k = x.shape
    y = torch.zeros((m, w.n), dtype=torch.float32, device="cuda")
    b = None if bias is None else torch.from_numpy(bias).cuda()
    samq.linear_mmq(w, torch.from_numpy(x).cuda(), m, k, b, epilogue, y, w.n)
    samq.check(0)
    return y.cpu().numpy()


@pytest.mark.parametrize("variant", [samq.MMQ_CODES_F16, samq.MMQ_CODES_I8])
@pytest.mark.parametrize("m,n,k", [(1, 128, 128), (33, 256, 512), (257, 384, 1024), (130, 100, 1024),
                                   (700, 1024, 4736)])
def test_mmq_exact_parity(variant, m, n, k):
    rng = np.random.default_rng(m + n + k + variant)
    w = rng.normal(0, 0.02, (n, k)).astype(np.float32)
    w[rng.random(w.shape) < 0.01] *= 8
    rows = o.quantize(o.Q8_0, w)
    w32 = o.dequantize(o.Q8_0, rows, n * k).reshape(n, k)
    x = (rng.normal(0, 1, (m, k)) * rng.uniform(0.01, 10, (m, 1))).astype(np.float32)
    bias = rng.normal(0, 0.5, n).astype(np.float32)
    h = samq.MmqWeights(o.Q8_0, k, n, rows, variant=variant)
    got = run(h, x, bias)
    ref = reference(w32, x, bias)
    err = float(np.abs(got - ref).max() / np.abs(ref).max())
    assert err <= 2e-6, err
    got = run(h, x, bias, epilogue=1)
    ref = reference(w32, x, bias, gelu=True)
    assert float(np.abs(got - ref).max() / np.abs(ref).max()) <= 2e-6
    h.close()


def test_mmq_wide_activation_range():
    """Activation blocks with amax up to 1e20 (beyond the f16 operand of the
    other path) keep their exact result; a NaN is flagged, not silently used."""
    rng = np.random.default_rng(9)
    m, n, k = 64, 256, 512
    w = rng.normal(0, 0.02, (n, k)).astype(np.float32)
    rows = o.quantize(o.Q8_0, w)
    w32 = o.dequantize(o.Q8_0, rows, n * k).reshape(n, k)
    x = rng.normal(0, 1, (m, k)).astype(np.float32)
    x[::3] *= np.float32(1e20)
    h = samq.MmqWeights(o.Q8_0, k, n, rows)
    got = run(h, x)
    ref = reference(w32, x)
    for r in range(m):
        assert np.abs(got[r] - ref[r]).max() <= 2e-6 * np.abs(ref[r]).max(), r
    x[5, 7] = np.nan
    y = torch.zeros((m, n), dtype=torch.float32, device="cuda")
    samq.linear_mmq(h, torch.from_numpy(x).cuda(), m, k, None, 0, y, n)
    with pytest.raises(samq.SamqError):
        samq.check(0)
    h.close()


def test_mmq_matches_f16_path_within_its_operand_precision():
    """The f16-operand K2 path sits within its stated 2e-3 of the exact path."""
    rng = np.random.default_rng(4)
    m, n, k = 300, 1024, 1024
    w = rng.normal(0, 0.02, (n, k)).astype(np.float32)
    rows = o.quantize(o.Q8_0, w)
    x = rng.normal(0, 1, (m, k)).astype(np.float32)
    exact = run(samq.MmqWeights(o.Q8_0, k, n, rows), x)
    wf = samq.Weights(o.Q8_0, k, n, rows)
    y = torch.zeros((m, n), dtype=torch.float32, device="cuda")
    samq.linear(wf, torch.from_numpy(x).cuda(), m, k, None, 0, y, n)
    samq.check(0)
    err = float(np.abs(y.cpu().numpy() - exact).max() / np.abs(exact).max())
    assert 1e-6 < err <= 2e-3, err
