"""Dense F32 modules on the GPU (dense.cu) against the f64 oracle.

The reference multiplies F32 / F16 weights with F32 semantics (cuBLAS
COMPUTE_32F_PEDANTIC, cmake/patches/ggml-precise-cuda.patch:288-356); the
device path gets there with a three-term TF32 split on the tensor cores.  Bars:
  - the reference's golden vectors (tests/runtime/ggml/test_graph.cpp:55-140):
    the 2x2 deconvolution layout within 1e-6 and the padded 3x3 convolution
    of 1.0003 within 1e-5 (F32 activations must not be narrowed), the
    single-channel cases embedded in 32 channels with zero weights;
  - random shapes: max |y - ref| no worse than 4x the error of an f32 SGEMM
    (numpy float32 matmul) of the same operands against the same f64 oracle,
    plus 1e-6 of max |ref| (the f64 oracle keeps its intermediates in f64,
    the device rounds them to f32 as cuBLAS does), and cosine >= 1 - 1e-9.
"""
import numpy as np
import pytest

from oracle import oracle as o

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def samq():
    import samq as module
    assert torch.cuda.is_available(), "GPU tests need a CUDA device"
    module.init(0)
    return module


def dev(a):
    return torch.from_numpy(np.ascontiguousarray(a, dtype=np.float32)).cuda()


def check_close(y, ref, ref_f32=None, rel=1e-6, factor=4.0):
    y = np.asarray(y, np.float64)
    ref = np.asarray(ref, np.float64)
    err = np.abs(y - ref).max()
    bound = rel * np.abs(ref).max()
    if ref_f32 is not None:
        bound += factor * np.abs(np.asarray(ref_f32, np.float64) - ref).max()
    cos = float((y.ravel() @ ref.ravel()) / (np.linalg.norm(y) * np.linalg.norm(ref)))
    assert err <= bound and cos >= 1 - 1e-9, (err, bound, cos)


def test_golden_deconv(samq):
    w = np.zeros((32, 32, 2, 2), np.float32)
    w[0, 0] = np.array([[1, 2], [3, 4]], np.float32)
    x = np.zeros((1, 2, 32), np.float32)
    x[0, :, 0] = [10, 20]
    wd = samq.Dense(samq.DENSE_DECONV2X2, w)
    y = torch.empty(2 * 4 * 32, device="cuda")
    samq.conv2d(wd, dev(x), 2, 1, None, 0, y)
    samq.check(0)
    out = y.cpu().numpy().reshape(2, 4, 32)
    np.testing.assert_allclose(out[..., 0].ravel(), [10, 20, 20, 40, 30, 40, 60, 80], atol=1e-6)
    assert not out[..., 1:].any()


@pytest.mark.parametrize("half", [False, True])
def test_golden_padded_conv(samq, half):
    w = np.zeros((1, 32, 3, 3), np.float32)
    w[0, 0] = np.arange(1, 10, dtype=np.float32).reshape(3, 3)
    wd = samq.Dense(samq.DENSE_CONV, w.astype(np.float16) if half else w)
    x = np.zeros((4, 4, 32), np.float32)
    x[..., 0] = 1.0003
    y = torch.empty(16, device="cuda")
    samq.conv2d(wd, dev(x), 4, 4, None, 0, y)
    samq.check(0)
    expected = o.conv2d_nhwc(x[..., :1], w[:, :1])[..., 0]
    assert np.abs(y.cpu().numpy().reshape(4, 4) - expected).max() <= 1e-5


@pytest.mark.parametrize("m,n,k", [(200, 256, 256), (5184, 256, 256), (33, 2048, 256), (1000, 300, 100),
                                   (7, 40, 36)])
@pytest.mark.parametrize("half", [False, True])
def test_dense_linear(samq, m, n, k, half):
    rng = np.random.default_rng(m + n + k + half)
    w = (rng.normal(size=(n, k)) / np.sqrt(k)).astype(np.float16 if half else np.float32)
    x = rng.normal(size=(m, k)).astype(np.float32)
    b = rng.normal(0, 0.02, n).astype(np.float32)
    gelu = (m + n) % 2 == 1
    wd = samq.Dense(samq.DENSE_LINEAR, w)
    ldx, ldy = k + 4, n + 8
    xd = torch.zeros((m, ldx), device="cuda")
    xd[:, :k] = dev(x)
    y = torch.full((m, ldy), 7.0, device="cuda")
    samq.dense_linear(wd, xd, m, ldx, dev(b), 1 if gelu else 0, y, ldy)
    samq.check(0)
    out = y.cpu().numpy()
    assert (out[:, n:] == 7.0).all()  # row padding untouched
    w32 = w.astype(np.float32)
    ref = o.dense_linear(x, w32, b, gelu)
    f32 = x @ w32.T + b
    if gelu:
        f32 = o.gelu_erf64(f32)
    check_close(out[:, :n], ref, f32)


@pytest.mark.parametrize("width,height,cin,cout,ks", [(20, 12, 64, 96, 3), (72, 72, 256, 256, 3), (36, 36, 256, 256, 3),
                                                      (13, 9, 32, 40, 3), (24, 10, 512, 256, 1)])
def test_conv2d(samq, width, height, cin, cout, ks):
    rng = np.random.default_rng(width * height + cin)
    w = (rng.normal(size=(cout, cin, ks, ks)) / np.sqrt(cin * ks * ks)).astype(np.float32)
    b = rng.normal(0, 0.02, cout).astype(np.float32)
    x = rng.normal(size=(height, width, cin)).astype(np.float32)
    wd = samq.Dense(samq.DENSE_CONV, w)
    y = torch.empty(height * width * cout, device="cuda")
    samq.conv2d(wd, dev(x), width, height, dev(b), 0, y)
    samq.check(0)
    ref = o.conv2d_nhwc(x, w, b)
    xp = np.pad(x, ((ks // 2, ks // 2), (ks // 2, ks // 2), (0, 0)))
    f32 = np.zeros((height, width, cout), np.float32)
    for ky in range(ks):
        for kx in range(ks):
            f32 += xp[ky:ky + height, kx:kx + width] @ w[:, :, ky, kx].T
    check_close(y.cpu().numpy().reshape(height, width, cout), ref, f32 + b)


@pytest.mark.parametrize("gelu", [False, True])
def test_deconv2x2(samq, gelu):
    rng = np.random.default_rng(11 + gelu)
    width, height, cin, cout = 9, 7, 96, 64
    w = (rng.normal(size=(cin, cout, 2, 2)) / np.sqrt(cin)).astype(np.float32)
    b = rng.normal(0, 0.02, cout).astype(np.float32)
    x = rng.normal(size=(height, width, cin)).astype(np.float32)
    wd = samq.Dense(samq.DENSE_DECONV2X2, w)
    y = torch.empty(4 * height * width * cout, device="cuda")
    samq.conv2d(wd, dev(x), width, height, dev(b), 1 if gelu else 0, y)
    samq.check(0)
    ref = o.deconv2x2_nhwc(x, w, b)
    f32 = np.zeros((2 * height, 2 * width, cout), np.float32)
    for ky in range(2):
        for kx in range(2):
            f32[ky::2, kx::2] = x @ w[:, :, ky, kx] + b
    if gelu:
        ref, f32 = o.gelu_erf64(ref), o.gelu_erf64(f32)
    check_close(y.cpu().numpy().reshape(2 * height, 2 * width, cout), ref, f32)


def test_maxpool_is_exact(samq):
    rng = np.random.default_rng(12)
    x = rng.normal(size=(9, 11, 64)).astype(np.float32)
    y = torch.empty(4 * 5 * 64, device="cuda")
    samq.maxpool2x2(dev(x), 11, 9, 64, y)
    samq.check(0)
    np.testing.assert_array_equal(y.cpu().numpy().reshape(4, 5, 64), o.maxpool2x2_nhwc(x))


def make_neck(samq, rng, E=1024, mid=512, D=256):
    """Random-init neck with fan-in scaled weights (SAM 3 shapes by default)."""
    shapes = {"s0_deconv1": (samq.DENSE_DECONV2X2, (E, mid, 2, 2)), "s0_deconv2": (samq.DENSE_DECONV2X2, (mid, D, 2, 2)),
              "s0_conv1x1": (samq.DENSE_CONV, (D, D, 1, 1)), "s0_conv3x3": (samq.DENSE_CONV, (D, D, 3, 3)),
              "s1_deconv1": (samq.DENSE_DECONV2X2, (E, mid, 2, 2)), "s1_conv1x1": (samq.DENSE_CONV, (D, mid, 1, 1)),
              "s1_conv3x3": (samq.DENSE_CONV, (D, D, 3, 3)), "s2_conv1x1": (samq.DENSE_CONV, (D, E, 1, 1)),
              "s2_conv3x3": (samq.DENSE_CONV, (D, D, 3, 3)), "s3_conv1x1": (samq.DENSE_CONV, (D, E, 1, 1)),
              "s3_conv3x3": (samq.DENSE_CONV, (D, D, 3, 3))}
    host, layers = {}, {}
    for name, (kind, shape) in shapes.items():
        fan_in = shape[0] if kind == samq.DENSE_DECONV2X2 else shape[1] * shape[2] * shape[3]
        w = (rng.normal(size=shape) / np.sqrt(fan_in)).astype(np.float32)
        b = rng.normal(0, 0.02, shape[1] if kind == samq.DENSE_DECONV2X2 else shape[0]).astype(np.float32)
        host[name] = (w, b)
        layers[name] = (samq.Dense(kind, w), dev(b))
    return host, samq.Neck(layers)


def run_neck(samq, neck, x, gw, gh, D=256):
    sizes = [(4 * gh, 4 * gw), (2 * gh, 2 * gw), (gh, gw), (gh // 2, gw // 2)]
    outs = [torch.empty(h * w * D, device="cuda") for h, w in sizes]
    samq.neck_forward(neck, dev(x), gw, gh, outs)
    samq.check(0)
    return [o_.cpu().numpy().reshape(h, w, D) for o_, (h, w) in zip(outs, sizes)]


def test_neck_small_grid(samq):
    """All four scales at a 10 x 6 grid with the SAM 3 channel counts."""
    rng = np.random.default_rng(21)
    host, neck = make_neck(samq, rng)
    gw, gh = 10, 6
    x = rng.normal(size=(gh, gw, 1024)).astype(np.float32)
    outs = run_neck(samq, neck, x.reshape(-1, 1024), gw, gh)
    refs = o.neck(x, host)
    for out, ref in zip(outs, refs):
        check_close(out, ref, rel=2e-6)


def test_neck_full_grid_low_scales(samq):
    """72 x 72 (the backbone's grid): scales 2 and 3 against the oracle, and
    all four maps finite."""
    rng = np.random.default_rng(22)
    host, neck = make_neck(samq, rng)
    x = rng.normal(size=(72, 72, 1024)).astype(np.float32)
    outs = run_neck(samq, neck, x.reshape(-1, 1024), 72, 72)
    assert all(np.isfinite(a).all() for a in outs)
    s2 = o.conv2d_nhwc(o.conv2d_nhwc(x, *host["s2_conv1x1"]), *host["s2_conv3x3"])
    s3 = o.conv2d_nhwc(o.conv2d_nhwc(o.maxpool2x2_nhwc(x), *host["s3_conv1x1"]), *host["s3_conv3x3"])
    check_close(outs[2], s2, rel=2e-6)
    check_close(outs[3], s3, rel=2e-6)


def test_neck_odd_grid(samq):
    """A 7 x 5 grid: the 0.5x scale floors to 3 x 2 (ggml_pool_2d without
    padding), the other maps are 28 x 20, 14 x 10 and 7 x 5."""
    rng = np.random.default_rng(23)
    host, neck = make_neck(samq, rng, E=256, mid=128, D=64)
    gw, gh = 7, 5
    x = rng.normal(size=(gh, gw, 256)).astype(np.float32)
    outs = run_neck(samq, neck, x.reshape(-1, 256), gw, gh, D=64)
    refs = o.neck(x, host)
    assert outs[3].shape == (2, 3, 64)
    for out, ref in zip(outs, refs):
        check_close(out, ref, rel=2e-6)
