"""Small-M linears (M <= 64): samq_linear_v1 / samq_linear_f16_v1 stream the K4
packets and decode them in the producer (stream.cu).

Shapes are the SAM 3 text encoder's (M = 32 tokens: in_proj 1024 -> 3072,
out_proj 1024 -> 1024, fc1 1024 -> 4096 + GELU, fc2 4096 -> 1024, resizer
1024 -> 256; src/models/sam3/text_encoder.hpp:83-174) plus ragged and
split-K cases.  Bars are the linear's: cosine >= 0.9999 and max error <= 2e-3
of max |ref| against the decoded-operand f64 product, and <= 5e-5 against the
f64 product of the exact f16 tensor-core operands (the decoded weights must
equal K2's f16 weights bit for bit, so an indexing error shows here).
"""
import numpy as np
import pytest

from test_gpu_kernels import (COS_MIN, EXACT_OPERAND_REL, MAX_REL, dev, host, metrics, references, run_linear,
                              weights_matrix)

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def samq():
    import samq as module
    assert torch.cuda.is_available(), "GPU tests need a CUDA device"
    module.init(0)
    return module


TEXT_SHAPES = [(3072, 1024, 0), (1024, 1024, 0), (4096, 1024, 1), (1024, 4096, 0), (256, 1024, 0)]


@pytest.mark.parametrize("n,k,epilogue", TEXT_SHAPES)
@pytest.mark.parametrize("m", [32, 33])
def test_text_encoder_linears_q8_0(samq, oracle, n, k, epilogue, m):
    rng = np.random.default_rng(n + k + m)
    rows = oracle.quantize(8, weights_matrix(rng, n, k))
    x = rng.normal(0, 1, (m, k)).astype(np.float32)
    bias = rng.normal(0, 0.5, n).astype(np.float32)
    w = samq.Weights(8, k, n, rows)
    y = run_linear(samq, w, x, bias=bias, epilogue=epilogue)
    semantic, exact = references(oracle, 8, rows, x, n, k, bias=bias, epilogue=epilogue)
    cos, rel = metrics(y, semantic)
    assert cos >= COS_MIN and rel <= MAX_REL, (cos, rel)
    assert metrics(y, exact)[1] <= EXACT_OPERAND_REL
    w.close()


@pytest.mark.parametrize("qtype", [8, 12, 13, 14])
@pytest.mark.parametrize("m,n,k", [(1, 1000, 2048), (17, 384, 1024), (64, 640, 512)])
def test_stream_formats_and_ragged_shapes(samq, oracle, qtype, m, n, k):
    """All four formats; n not a multiple of 128 (zero rows of the last
    packet tile), single rows, the 64-token variant, 1..16-way split-K."""
    rng = np.random.default_rng(qtype * 7 + m + n)
    rows = oracle.quantize(qtype, weights_matrix(rng, n, k))
    x = rng.normal(0, 1, (m, k)).astype(np.float32)
    w = samq.Weights(qtype, k, n, rows)
    y = run_linear(samq, w, x, ldy=n + 4)
    semantic, exact = references(oracle, qtype, rows, x, n, k)
    cos, rel = metrics(y, semantic)
    assert cos >= COS_MIN and rel <= MAX_REL, (cos, rel)
    assert metrics(y, exact)[1] <= EXACT_OPERAND_REL
    w.close()


def test_stream_f16_entry_and_determinism(samq, oracle):
    """samq_linear_f16_v1 takes the same path from a caller-staged operand
    (row stride > k); two calls give identical bits (fixed split-K order)."""
    rng = np.random.default_rng(77)
    m, n, k = 32, 1024, 4096
    rows = oracle.quantize(12, weights_matrix(rng, n, k))
    x = rng.normal(0, 1, (m, k)).astype(np.float32)
    w = samq.Weights(12, k, n, rows)
    a16 = torch.zeros((m, k + 16), dtype=torch.float16, device="cuda")
    samq.stage_f16(dev(x), m, k, k, a16[:, :k].contiguous())
    staged = torch.empty((m, k), dtype=torch.float16, device="cuda")
    samq.stage_f16(dev(x), m, k, k, staged)
    a16[:, :k] = staged
    ys = []
    for _ in range(2):
        y = torch.empty((m, n), dtype=torch.float32, device="cuda")
        samq.linear_f16(w, a16, m, k + 16, None, 0, y, n)
        ys.append(host(y))
    np.testing.assert_array_equal(ys[0], ys[1])
    np.testing.assert_array_equal(ys[0], run_linear(samq, w, x))
    _, exact = references(oracle, 12, rows, x, n, k)
    assert metrics(ys[0], exact)[1] <= EXACT_OPERAND_REL
    w.close()
