"""Dense F32 modules on the CPU: the f64 oracle pinned to the reference's
golden vectors, and the C ABI rejecting malformed dense arguments before any
device work.

Golden vectors: tests/runtime/ggml/test_graph.cpp:55-140 of the reference --
a 2x2 deconvolution of a 2 x 1 image ({10, 20}) by kernel {1, 2, 3, 4} gives
{10, 20, 20, 40, 30, 40, 60, 80}, and 3x3 convolutions (kernel 1..9, F32 and
F16 storage) of a 4 x 4 image of 1.0003 give sum(kernel taps in range) *
1.0003 within 1e-5, unpadded stride 3 (sam3_conv_2d_sk_p0) and padded stride 1
(sam3_conv_2d_s1_ph); 1.0003 checks that F32 activations are not narrowed
(F16 staging rounds it to 1).
"""
import ctypes
import subprocess

import numpy as np
import pytest

from conftest import PACKAGE
from oracle import oracle as o

GOLDEN_DECONV = np.array([10, 20, 20, 40, 30, 40, 60, 80], np.float32)


def golden_conv_expected(padded: bool) -> np.ndarray:
    kernel = np.arange(1, 10, dtype=np.float64)
    width = 4 if padded else 1
    out = np.zeros((width, width))
    for y in range(width):
        for x in range(width):
            for ky in range(3):
                for kx in range(3):
                    iy, ix = y + ky - (1 if padded else 0), x + kx - (1 if padded else 0)
                    if 0 <= ix < 4 and 0 <= iy < 4:
                        out[y, x] += kernel[ky * 3 + kx] * float(np.float32(1.0003))
    return out


def test_oracle_deconv_golden():
    w = np.array([1, 2, 3, 4], np.float32).reshape(1, 1, 2, 2)  # GGML [2, 2, 1, 1]: index kx + 2 ky
    x = np.array([10, 20], np.float32).reshape(1, 2, 1)          # [H=1][W=2][C=1]
    out = o.deconv2x2_nhwc(x, w)
    assert out.shape == (2, 4, 1)
    np.testing.assert_allclose(out.ravel(), GOLDEN_DECONV, atol=1e-6)


@pytest.mark.parametrize("half", [False, True])
@pytest.mark.parametrize("padded", [False, True])
def test_oracle_conv_golden(padded, half):
    kernel = np.arange(1, 10, dtype=np.float32).reshape(1, 1, 3, 3)
    if half:
        kernel = kernel.astype(np.float16).astype(np.float32)  # exact for 1..9
    image = np.full((4, 4, 1), 1.0003, np.float32)
    out = o.conv2d_nhwc(image, kernel) if padded else o.conv2d_nhwc(image, kernel, stride=3, pad=0)
    expected = golden_conv_expected(padded)
    assert out.shape[:2] == expected.shape
    assert np.abs(out[..., 0] - expected).max() <= 1e-5


def test_oracle_deconv_matches_transposed_convolution_definition():
    """deconv2x2 against the scatter form of ConvTranspose2d(stride 2, k 2)."""
    rng = np.random.default_rng(3)
    x = rng.normal(size=(3, 5, 4))
    w = rng.normal(size=(4, 6, 2, 2))
    out = np.zeros((6, 10, 6))
    for i in range(3):
        for j in range(5):
            for ky in range(2):
                for kx in range(2):
                    out[2 * i + ky, 2 * j + kx] += x[i, j] @ w[:, :, ky, kx]
    np.testing.assert_allclose(o.deconv2x2_nhwc(x, w), out, rtol=1e-12, atol=1e-12)


def test_oracle_conv_matches_direct_sum():
    rng = np.random.default_rng(4)
    x = rng.normal(size=(5, 6, 3))
    w = rng.normal(size=(2, 3, 3, 3))
    b = rng.normal(size=2)
    ref = np.zeros((5, 6, 2))
    for y in range(5):
        for xx in range(6):
            for co in range(2):
                s = b[co]
                for ky in range(3):
                    for kx in range(3):
                        iy, ix = y + ky - 1, xx + kx - 1
                        if 0 <= iy < 5 and 0 <= ix < 6:
                            s += x[iy, ix] @ w[co, :, ky, kx]
                ref[y, xx, co] = s
    np.testing.assert_allclose(o.conv2d_nhwc(x, w, b), ref, rtol=1e-12, atol=1e-12)


def test_oracle_maxpool_floor_sizes():
    x = np.arange(5 * 7 * 2, dtype=np.float32).reshape(5, 7, 2)
    out = o.maxpool2x2_nhwc(x)
    assert out.shape == (2, 3, 2)
    assert out[1, 2, 1] == x[3, 5, 1]


def test_oracle_neck_shapes():
    rng = np.random.default_rng(5)
    E, mid, D, g = 64, 32, 32, 4
    lay = {
        "s0_deconv1": (rng.normal(size=(E, mid, 2, 2)), None), "s0_deconv2": (rng.normal(size=(mid, D, 2, 2)), None),
        "s0_conv1x1": (rng.normal(size=(D, D, 1, 1)), None), "s0_conv3x3": (rng.normal(size=(D, D, 3, 3)), None),
        "s1_deconv1": (rng.normal(size=(E, mid, 2, 2)), None), "s1_conv1x1": (rng.normal(size=(D, mid, 1, 1)), None),
        "s1_conv3x3": (rng.normal(size=(D, D, 3, 3)), None), "s2_conv1x1": (rng.normal(size=(D, E, 1, 1)), None),
        "s2_conv3x3": (rng.normal(size=(D, D, 3, 3)), None), "s3_conv1x1": (rng.normal(size=(D, E, 1, 1)), None),
        "s3_conv3x3": (rng.normal(size=(D, D, 3, 3)), None)}
    outs = o.neck(rng.normal(size=(g, g + 2, E)), lay)
    assert [x.shape for x in outs] == [(16, 24, D), (8, 12, D), (4, 6, D), (2, 3, D)]


@pytest.fixture(scope="module")
def samq():
    lib = PACKAGE / "libsamq.so"
    if not lib.exists():
        subprocess.run(["make", "-C", str(PACKAGE), "-s", "-j4"], check=True)
    import samq as module
    module.library()
    return module


def test_invalid_dense_arguments_are_rejected(samq):
    lib = samq.library()
    h = ctypes.c_void_p()
    w = np.zeros(64 * 9 * 32, np.float32)
    # unknown type (Q8_0 is not dense)
    rc = lib.samq_dense_create_v1(0, 8, samq.DENSE_CONV, 3, 3, 64, 32, w.ctypes.data, w.nbytes, None, ctypes.byref(h))
    assert rc == 1 and b"F32 or F16" in lib.samq_last_error_v1()
    # 5x5 kernels are not a neck shape
    rc = lib.samq_dense_create_v1(0, 0, samq.DENSE_CONV, 5, 5, 64, 32, w.ctypes.data, w.nbytes, None, ctypes.byref(h))
    assert rc == 1 and b"1x1 or 3x3" in lib.samq_last_error_v1()
    # input channels not a multiple of 32
    rc = lib.samq_dense_create_v1(0, 0, samq.DENSE_CONV, 3, 3, 48, 32, w.ctypes.data, w.nbytes, None, ctypes.byref(h))
    assert rc == 1 and b"multiple of 32" in lib.samq_last_error_v1()
    # payload size
    rc = lib.samq_dense_create_v1(0, 0, samq.DENSE_CONV, 3, 3, 64, 32, w.ctypes.data, w.nbytes - 4, None,
                                  ctypes.byref(h))
    assert rc == 1 and b"size" in lib.samq_last_error_v1()
    # deconvolution output channels must be a multiple of 32
    rc = lib.samq_dense_create_v1(0, 0, samq.DENSE_DECONV2X2, 2, 2, 64, 16, w.ctypes.data, 64 * 16 * 16, None,
                                  ctypes.byref(h))
    assert rc == 1 and b"multiples of 32" in lib.samq_last_error_v1()
    assert h.value is None
    rc = lib.samq_dense_linear_v1(None, None, 4, 32, None, 0, None, 32, None)
    assert rc == 1 and b"LINEAR" in lib.samq_last_error_v1()
    rc = lib.samq_conv2d_v1(None, None, 4, 4, None, 0, None, None)
    assert rc == 1 and b"CONV" in lib.samq_last_error_v1()
    rc = lib.samq_maxpool2x2_v1(None, 4, 4, 6, None, None)
    assert rc == 1 and b"multiple of 4" in lib.samq_last_error_v1()
    rc = lib.samq_neck_forward_v1(None, None, 8, 8, None, None)
    assert rc == 1 and b"version 1" in lib.samq_last_error_v1()
