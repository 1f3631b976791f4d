"""GPU parity of the sm_100a kernels against the CPU oracle, through the C ABI.

Bars (BASELINE north star and the reference's own tests):
  * K1 activation staging (Q8_1 36-byte blocks, MMQ-D4 144-byte blocks):
    bit-exact against the oracle and the committed, reference-verified
    fixture; MMQ-D4 also passes the reference KAT
    (tests/runtime/ggml/test_cuda_q8_mmq_scale.cpp:33-93).
  * K4 repack: packets bit-exact against the oracle; export round trip
    bit-exact against the GGUF input.
  * K2 linear: against the f64 product of the decoded weights and the decoded
    Q8_1 activations, cosine >= 0.9999 and normalized max error
    max|y - ref| / max|ref| <= 2e-3 (north star, "fp32 accumulate"); against
    the f64 product of the exact f16 tensor-core operands, normalized max
    error <= 5e-5 (only f32 accumulation order differs).
"""
import numpy as np
import pytest

from conftest import load_golden
from test_oracle import check_mmq_kat, mmq_kat_input

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu

COS_MIN = 0.9999
MAX_REL = 2e-3
EXACT_OPERAND_REL = 5e-5


@pytest.fixture(scope="module")
def samq():
    import samq as module
    assert torch.cuda.is_available(), "GPU tests need a CUDA device"
    module.init(0)
    return module


def dev(a):
    return torch.from_numpy(np.ascontiguousarray(a)).cuda()


def host(t):
    torch.cuda.synchronize()
    return t.cpu().numpy()


def metrics(y, ref):
    y64, r64 = y.astype(np.float64).ravel(), ref.astype(np.float64).ravel()
    cos = float(np.dot(y64, r64) / (np.linalg.norm(y64) * np.linalg.norm(r64)))
    rel = float(np.max(np.abs(y64 - r64)) / np.max(np.abs(r64)))
    return cos, rel


def weights_matrix(rng, n, k):
    w = rng.normal(0.0, 0.02, (n, k)).astype(np.float32)
    mask = rng.random(w.shape) < 0.01
    w[mask] *= 8
    return w


# ------------------------------------------------------------------ K1

def test_q8_1_staging_matches_verified_fixture(samq):
    g = load_golden("q8_staging")
    x = g["source"]
    out = torch.zeros(g["q8_1"].size, dtype=torch.uint8, device="cuda")
    samq.quantize_q8_1(dev(x), x.shape[0], x.shape[1], x.shape[1], out)
    np.testing.assert_array_equal(host(out), g["q8_1"])


@pytest.mark.parametrize("rows,k,ld", [(1, 32, 32), (7, 96, 100), (300, 1024, 1024), (33, 4736, 4740)])
def test_q8_1_staging_matches_oracle(samq, oracle, rows, k, ld):
    rng = np.random.default_rng(rows * 7 + k)
    x = (rng.normal(0, 1, (rows, ld)) * rng.uniform(1e-3, 1e3, (rows, 1))).astype(np.float32)
    out = torch.zeros(rows * (k // 32) * 36, dtype=torch.uint8, device="cuda")
    samq.quantize_q8_1(dev(x), rows, k, ld, out)
    np.testing.assert_array_equal(host(out), oracle.quantize_q8_1(x[:, :k]))


def test_mmq_d4_matches_fixture_and_kat(samq, oracle):
    g = load_golden("q8_staging")
    x = g["source"]
    out = torch.zeros(samq.mmq_d4_bytes(*x.shape), dtype=torch.uint8, device="cuda")
    samq.quantize_mmq_q8_1(dev(x), x.shape[0], x.shape[1], x.shape[1], out)
    np.testing.assert_array_equal(host(out), g["mmq_d4"])
    kat = mmq_kat_input()
    out = torch.zeros(samq.mmq_d4_bytes(*kat.shape), dtype=torch.uint8, device="cuda")
    samq.quantize_mmq_q8_1(dev(kat), kat.shape[0], kat.shape[1], kat.shape[1], out)
    payload = host(out)
    check_mmq_kat(kat, payload)
    np.testing.assert_array_equal(payload, oracle.quantize_mmq_d4(kat))


# ------------------------------------------------------------------ K4

FORMATS = [8, 12, 13, 14]


@pytest.mark.parametrize("qtype", FORMATS)
@pytest.mark.parametrize("n,k", [(1, 256), (130, 512), (300, 1024)])
def test_repack_packets_and_round_trip(samq, oracle, qtype, n, k):
    rng = np.random.default_rng(qtype * 1000 + n)
    rows = oracle.quantize(qtype, weights_matrix(rng, n, k))
    w = samq.Weights(qtype, k, n, rows)
    ptr, size = w.packets()
    expected = oracle.pack_packets(qtype, k, n, rows)
    assert size == expected.size
    got = torch.empty(size, dtype=torch.uint8, device="cuda")
    cudart_copy(got.data_ptr(), ptr, size)
    np.testing.assert_array_equal(host(got), expected)
    np.testing.assert_array_equal(w.export(), rows)
    w.close()


def cudart_copy(dst, src, size):
    """Device-to-device cudaMemcpy through the CUDA runtime torch has loaded."""
    import ctypes
    rt = ctypes.CDLL("libcudart.so.12")
    rt.cudaMemcpy.restype = ctypes.c_int
    rt.cudaMemcpy.argtypes = [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_size_t, ctypes.c_int]
    torch.cuda.synchronize()
    assert rt.cudaMemcpy(dst, src, size, 3) == 0  # cudaMemcpyDeviceToDevice


def test_q8_0_repack_odd_widths(samq, oracle):
    rng = np.random.default_rng(17)
    for k in (32, 96, 4736):
        rows = oracle.quantize(8, weights_matrix(rng, 5, k))
        w = samq.Weights(8, k, 5, rows)
        np.testing.assert_array_equal(w.export(), rows)
        w.close()


@pytest.mark.parametrize("qtype", FORMATS)
def test_repack_rejects_nonfinite_scale(samq, oracle, qtype):
    rng = np.random.default_rng(5)
    rows = oracle.quantize(qtype, weights_matrix(rng, 3, 256)).reshape(3, -1).copy()
    off = 208 if qtype == 14 else 0
    rows[1, off:off + 2] = np.array([0x00, 0x7c], dtype=np.uint8)  # f16 +inf
    with pytest.raises(samq.SamqError) as err:
        samq.Weights(qtype, 256, 3, rows)
    assert err.value.status == 7
    if qtype in (12, 13):  # non-finite dmin (test_quantization.cpp:99-104)
        rows = oracle.quantize(qtype, weights_matrix(rng, 3, 256)).reshape(3, -1).copy()
        rows[2, 2:4] = np.array([0x00, 0x7e], dtype=np.uint8)
        with pytest.raises(samq.SamqError):
            samq.Weights(qtype, 256, 3, rows)


# ------------------------------------------------------------------ K2

def run_linear(samq, w, x, bias=None, epilogue=0, ldx=None, ldy=None):
    m, k = x.shape
    ldx = ldx or k
    ldy = ldy or w.n
    xs = np.zeros((m, ldx), np.float32)
    xs[:, :k] = x
    y = torch.full((max(m, 1), ldy), -7.0, dtype=torch.float32, device="cuda")
    b = dev(bias) if bias is not None else None
    samq.linear(w, dev(xs), m, ldx, b, epilogue, y, ldy)
    out = host(y)
    if ldy > w.n:
        assert np.all(out[:m, w.n:] == -7.0), "wrote outside the n output columns"
    return out[:m, :w.n]


def references(oracle, qtype, rows, x, n, k, bias=None, epilogue=0):
    w32 = oracle.dequantize(qtype, rows, n * k).reshape(n, k)
    x_dec = oracle.q8_1_decode(oracle.quantize_q8_1(x), x.shape[0], k)
    semantic = oracle.gemm_f64(w32, x_dec, bias=bias, epilogue=epilogue)
    exact = oracle.gemm_f64(oracle.weight_f16(qtype, k, n, rows), oracle.act_f16(x), bias=bias, epilogue=epilogue)
    return semantic, exact


@pytest.mark.parametrize("qtype", FORMATS)
@pytest.mark.parametrize("m,n,k", [(1, 128, 256), (33, 256, 512), (257, 384, 1024), (130, 100, 1024), (200, 1024, 256)])
def test_linear_parity(samq, oracle, qtype, m, n, k):
    rng = np.random.default_rng(qtype + 13 * m + n)
    rows = oracle.quantize(qtype, weights_matrix(rng, n, k))
    x = rng.normal(0, 1, (m, k)).astype(np.float32)
    w = samq.Weights(qtype, k, n, rows)
    y = run_linear(samq, w, x)
    semantic, exact = references(oracle, qtype, rows, x, n, k)
    cos, rel = metrics(y, semantic)
    assert cos >= COS_MIN and rel <= MAX_REL, (cos, rel)
    _, rel_exact = metrics(y, exact)
    assert rel_exact <= EXACT_OPERAND_REL, rel_exact
    w.close()


@pytest.mark.parametrize("epilogue,bias_scale", [(0, 0.5), (1, 0.5), (1, 8.0)])
def test_linear_bias_gelu_and_strides(samq, oracle, epilogue, bias_scale):
    """bias_scale 8 drives GELU arguments across the whole erf range (|x| up to ~30)."""
    rng = np.random.default_rng(31 + epilogue)
    qtype, m, n, k = 12, 70, 320, 512
    rows = oracle.quantize(qtype, weights_matrix(rng, n, k))
    x = rng.normal(0, 1, (m, k)).astype(np.float32)
    bias = rng.normal(0, bias_scale, n).astype(np.float32)
    w = samq.Weights(qtype, k, n, rows)
    y = run_linear(samq, w, x, bias=bias, epilogue=epilogue, ldx=k + 12, ldy=n + 8)
    semantic, exact = references(oracle, qtype, rows, x, n, k, bias=bias, epilogue=epilogue)
    cos, rel = metrics(y, semantic)
    assert cos >= COS_MIN and rel <= MAX_REL, (cos, rel)
    assert metrics(y, exact)[1] <= EXACT_OPERAND_REL
    w.close()


def test_linear_q8_0_wide_k(samq, oracle):
    """fc2 shape class: K = 4736 is Q8_0 even in K-quant profiles (weights.hpp:148-164)."""
    rng = np.random.default_rng(47)
    m, n, k = 96, 256, 4736
    rows = oracle.quantize(8, weights_matrix(rng, n, k))
    x = rng.normal(0, 1, (m, k)).astype(np.float32)
    w = samq.Weights(8, k, n, rows)
    y = run_linear(samq, w, x)
    semantic, exact = references(oracle, 8, rows, x, n, k)
    cos, rel = metrics(y, semantic)
    assert cos >= COS_MIN and rel <= MAX_REL
    assert metrics(y, exact)[1] <= EXACT_OPERAND_REL
    w.close()


@pytest.mark.parametrize("qtype,m,n,k,epilogue", [
    (8, 2000, 4736, 1056, 0),   # ragged M (7.8 pair tiles), ragged N (BN 192), K % 64 == 32
    (8, 2000, 4736, 1056, 1),   # the same with erf-GELU (16 epilogue warps per CTA)
    (12, 1300, 6144, 1024, 0),  # the last pair tile's second CTA holds only rows past M
])
def test_linear_cta_pair_ragged_shapes(samq, oracle, qtype, m, n, k, epilogue):
    """Shapes whose CTA-pair tiling runs three or more waves (gemm_f16_pair_kernel,
    cta_group::2), with ragged edges in M, N and K; checked on the first 64 and
    the last 150 rows against the oracle (every other row lies in a tile of the
    same kind)."""
    rng = np.random.default_rng(qtype + m + n + epilogue)
    rows = oracle.quantize(qtype, weights_matrix(rng, n, k))
    x = rng.normal(0, 1, (m, k)).astype(np.float32)
    bias = rng.normal(0, 0.02, n).astype(np.float32)
    w = samq.Weights(qtype, k, n, rows)
    y = run_linear(samq, w, x, bias=bias, epilogue=epilogue)
    pick = np.r_[0:64, m - 150:m]
    semantic, exact = references(oracle, qtype, rows, x[pick], n, k, bias=bias, epilogue=epilogue)
    cos, rel = metrics(y[pick], semantic)
    assert cos >= COS_MIN and rel <= MAX_REL, (cos, rel)
    assert metrics(y[pick], exact)[1] <= EXACT_OPERAND_REL
    assert np.isfinite(y).all()
    w.close()


def test_linear_from_staged_q8_1_matches_linear(samq, oracle):
    rng = np.random.default_rng(8)
    m, n, k = 150, 512, 1024
    rows = oracle.quantize(13, weights_matrix(rng, n, k))
    x = rng.normal(0, 1, (m, k)).astype(np.float32)
    w = samq.Weights(13, k, n, rows)
    xq = torch.zeros(m * (k // 32) * 36, dtype=torch.uint8, device="cuda")
    samq.quantize_q8_1(dev(x), m, k, k, xq)
    y1 = torch.empty((m, n), dtype=torch.float32, device="cuda")
    samq.linear_q8_1(w, xq, m, None, 0, y1, n)
    y2 = run_linear(samq, w, x)
    np.testing.assert_array_equal(host(y1), y2)
    w.close()


def test_stage_f16_and_linear_f16_compose_to_linear(samq, oracle):
    rng = np.random.default_rng(21)
    m, n, k = 77, 256, 512
    rows = oracle.quantize(14, weights_matrix(rng, n, k))
    x = rng.normal(0, 1, (m, k)).astype(np.float32)
    w = samq.Weights(14, k, n, rows)
    a16 = torch.empty((m, k), dtype=torch.float16, device="cuda")
    samq.stage_f16(dev(x), m, k, k, a16)
    np.testing.assert_array_equal(host(a16).view(np.uint16), oracle.act_f16(x).view(np.uint16))
    padded = torch.zeros((m, k + 8), dtype=torch.float16, device="cuda")
    padded[:, :k] = a16
    y = torch.empty((m, n), dtype=torch.float32, device="cuda")
    samq.linear_f16(w, padded, m, k + 8, None, 0, y, n)
    np.testing.assert_array_equal(host(y), run_linear(samq, w, x))
    w.close()


def test_linear_zero_rows_and_counters(samq, oracle):
    rng = np.random.default_rng(3)
    rows = oracle.quantize(8, weights_matrix(rng, 64, 256))
    w = samq.Weights(8, 256, 64, rows)
    before = w.query().launches
    y = torch.empty((1, 64), dtype=torch.float32, device="cuda")
    samq.linear(w, dev(np.zeros((1, 256), np.float32)), 0, 256, None, 0, y, 64)
    run_linear(samq, w, rng.normal(0, 1, (5, 256)).astype(np.float32))
    c = w.query()
    assert c.version == 1 and c.path == 1 and c.launches == before + 1
    assert c.payload_bytes == 5 * 256 * 2 and c.allocation_bytes >= c.payload_bytes
    w.close()


def test_range_check_rejects_then_recovers(samq, oracle):
    """Mirrors the invalid-RHS rejection and recovery of test_native_activation.cpp:186-198."""
    rng = np.random.default_rng(12)
    rows = oracle.quantize(8, weights_matrix(rng, 32, 256))
    w = samq.Weights(8, 256, 32, rows)
    samq.check(0)
    bad = rng.normal(0, 1, (4, 256)).astype(np.float32)
    bad[2, 7] = np.float32(1e6)
    run_linear(samq, w, bad)
    with pytest.raises(samq.SamqError) as err:
        samq.check(0)
    assert err.value.status == 5
    x = rng.normal(0, 1, (4, 256)).astype(np.float32)
    y = run_linear(samq, w, x)
    samq.check(0)
    semantic, _ = references(oracle, 8, rows, x, 32, 256)
    assert metrics(y, semantic)[0] >= COS_MIN
    w.close()


@pytest.mark.parametrize("qtype", [8, 12])
def test_full_size_fc1_sampled_rows(samq, oracle, qtype):
    """Config 1 / 2 shape (M=5184, N=4736, K=1024); rows are independent, so a
    sample of rows is checked against the oracle at full size."""
    rng = np.random.default_rng(0)
    n, k, m = 4736, 1024, 5184
    w32 = weights_matrix(rng, n, k)
    rows = oracle.quantize(qtype, w32)
    x = rng.normal(0, 1, (m, k)).astype(np.float32)
    bias = rng.normal(0, 0.02, n).astype(np.float32)
    w = samq.Weights(qtype, k, n, rows)
    y = run_linear(samq, w, x, bias=bias, epilogue=1)
    pick = np.sort(rng.choice(m, 48, replace=False))
    pick[-1] = m - 1
    semantic, exact = references(oracle, qtype, rows, x[pick], n, k, bias=bias, epilogue=1)
    cos, rel = metrics(y[pick], semantic)
    assert cos >= COS_MIN and rel <= MAX_REL, (cos, rel)
    assert metrics(y[pick], exact)[1] <= EXACT_OPERAND_REL
    assert np.isfinite(y).all()
    w.close()
