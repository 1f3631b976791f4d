"""Host-side checks of the C ABI (no GPU needed).

The library must load, export every entry point include/samq.h declares and
reject malformed arguments with a status code and a message before any
device work (the reference's boundary validates shapes the same way,
src/runtime/ggml/backends/cpu.hpp:26-34, src/models/sam3/weights.hpp:384-425).
"""
import ctypes
import re
import subprocess

import numpy as np
import pytest

from conftest import PACKAGE, ROOT


def header_functions():
    text = (ROOT / "include" / "samq.h").read_text()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"\b(samq_[a-z0-9_]+_v[0-9]+)\s*\(", text)))


@pytest.fixture(scope="module")
def samq():
    lib = PACKAGE / "libsamq.so"
    if not lib.exists():
        subprocess.run(["make", "-C", str(PACKAGE), "-s", "-j4"], check=True)
    import samq as module
    module.library()
    return module


def test_header_declares_the_expected_surface():
    names = header_functions()
    assert "samq_linear_v1" in names and "samq_weights_create_v1" in names
    assert len(names) >= 14


def test_library_exports_every_declared_symbol(samq):
    lib = samq.library()
    for name in header_functions():
        assert hasattr(lib, name), name
    out = subprocess.run(["nm", "-D", "--defined-only", str(samq.LIB_PATH)], capture_output=True, text=True,
                         check=True).stdout
    exported = set(re.findall(r"\bT (samq_[a-z0-9_]+)", out))
    assert set(header_functions()) <= exported


def test_binding_covers_the_header(samq):
    assert set(samq.SIGNATURES) == set(header_functions())


def test_invalid_weight_arguments_are_rejected(samq):
    lib = samq.library()
    handle = ctypes.c_void_p()
    rows = np.zeros(34, dtype=np.uint8)
    # unsupported type id (Q4_0 = 2)
    rc = lib.samq_weights_create_v1(0, 2, 32, 1, rows.ctypes.data, rows.nbytes, None, ctypes.byref(handle))
    assert rc == 1 and b"Q8_0" in lib.samq_last_error_v1()
    # width not block aligned for Q4_K
    rc = lib.samq_weights_create_v1(0, 12, 128, 1, rows.ctypes.data, rows.nbytes, None, ctypes.byref(handle))
    assert rc == 1 and b"block" in lib.samq_last_error_v1()
    # payload size differs from n rows
    rc = lib.samq_weights_create_v1(0, 8, 32, 2, rows.ctypes.data, rows.nbytes, None, ctypes.byref(handle))
    assert rc == 1 and b"size" in lib.samq_last_error_v1()
    assert handle.value is None


def test_invalid_linear_arguments_are_rejected(samq):
    lib = samq.library()
    rc = lib.samq_linear_v1(None, None, 4, 32, None, 0, None, 32, None)
    assert rc == 1 and b"null weights" in lib.samq_last_error_v1()
    rc = lib.samq_quantize_q8_1_v1(None, 4, 48, 48, None, None)
    assert rc == 1 and b"multiple of 32" in lib.samq_last_error_v1()
    rc = lib.samq_quantize_q8_1_v1(None, 4, 64, 62, None, None)
    assert rc == 1


def test_mmq_d4_sizes(samq):
    assert samq.mmq_d4_bytes(65, 160) == 65 * 4 * 144
    assert samq.mmq_d4_bytes(1, 512) == 4 * 144
    assert samq.mmq_d4_bytes(2, 513) == 2 * 8 * 144
    assert samq.mmq_d4_bytes(0, 32) == 0


def test_last_error_is_thread_local(samq):
    import threading
    lib = samq.library()
    lib.samq_linear_v1(None, None, 4, 32, None, 0, None, 32, None)
    seen = []
    t = threading.Thread(target=lambda: seen.append(lib.samq_last_error_v1()))
    t.start()
    t.join()
    assert seen == [b""]
    assert lib.samq_last_error_v1() != b""


def test_invalid_block_arguments_are_rejected(samq):
    """The ViT block entries check the descriptor before any device work."""
    lib = samq.library()
    x = ctypes.c_void_p(16)
    rc = lib.samq_vit_block_forward_v1(None, x, 72, 72, None)
    assert rc == 1 and b"version 1" in lib.samq_last_error_v1()
    rc = lib.samq_vit_block_forward_batch_v1(None, x, 8, 72, 72, None)
    assert rc == 1 and b"version 1" in lib.samq_last_error_v1()
    desc = samq.VitBlockDesc()
    desc.version = 3
    rc = lib.samq_vit_block_forward_batch_v1(ctypes.byref(desc), x, 8, 72, 72, None)
    assert rc == 1 and b"version 1" in lib.samq_last_error_v1()
    desc.version = 2
    desc.compute = 7  # neither SAMQ_COMPUTE_F32 nor _F16
    rc = lib.samq_vit_block_forward_v1(ctypes.byref(desc), x, 72, 72, None)
    assert rc == 1 and b"compute" in lib.samq_last_error_v1()


def test_module_descriptors_are_checked_before_device_work(samq):
    """The fusion, decoder, geometry and segmentation entries reject a missing
    or wrongly versioned descriptor without touching a device."""
    lib = samq.library()
    x = ctypes.c_void_p(16)
    assert lib.samq_fusion_layer_forward_v1(None, x, x, 16, x, None, 1, None) == 1
    assert b"version 1" in lib.samq_last_error_v1()
    assert lib.samq_decoder_forward_v1(None, x, x, 8, x, None, None, 1, x, x, x, x, None) == 1
    assert b"version 1" in lib.samq_last_error_v1()
    dec = samq.DecoderDesc()
    dec.version = 2
    assert lib.samq_decoder_forward_v1(ctypes.byref(dec), x, x, 8, x, None, None, 1, x, x, x, x, None) == 1
    assert lib.samq_geometry_encoder_forward_v1(None, x, x, 16, x, None) == 1
    assert b"version 1" in lib.samq_last_error_v1()
    geo = samq.GeometryEncoderDesc()
    geo.version = 1
    geo.layers = 0
    assert lib.samq_geometry_encoder_forward_v1(ctypes.byref(geo), x, x, 16, x, None) == 1
    assert b"layer count" in lib.samq_last_error_v1()
    assert lib.samq_seg_head_forward_v1(None, x, 8, x, x, x, 4, x, None, 1, x, None) == 1
    assert b"version 1" in lib.samq_last_error_v1()


def test_sine_pe_2d_host(samq):
    """samq_sine_pe_2d_v1 (host f32, the reference's own arithmetic) against
    the oracle's f64 evaluation of the same f32 arguments, and its layout:
    y encoding in the first half, x in the second, sin at even channels."""
    import sys
    sys.path.insert(0, str(ROOT))
    from oracle import oracle as o
    pe = samq.sine_pe_2d(72, 72, 256)
    ref = o.sine_pe_2d(72, 72, 256)
    assert np.abs(pe.astype(np.float64) - ref).max() <= 1e-6
    assert abs(float(pe[0, 0]) - np.sin(2 * np.pi / 72)) <= 1e-6 and abs(float(pe[0, 1]) - np.cos(2 * np.pi / 72)) <= 1e-6
    assert np.array_equal(pe[5 * 72 + 3, :128], pe[5 * 72 + 40, :128])  # y half depends on the row only
    assert np.array_equal(pe[3 * 72 + 9, 128:], pe[60 * 72 + 9, 128:])  # x half on the column only
    pe2 = samq.sine_pe_2d(24, 36, 64)
    assert np.abs(pe2.astype(np.float64) - o.sine_pe_2d(24, 36, 64)).max() <= 1e-6
    with pytest.raises(samq.SamqError):
        samq.sine_pe_2d(0, 4, 8)


@pytest.mark.parametrize("qtype", [8, 12, 13, 14])
def test_quantize_rows_host(samq, qtype):
    """samq_quantize_rows_v1: Q8_0 bit-exact with the oracle's restatement of
    the reference converter's quantizer; every format decodes (oracle
    dequantizer, pinned to gguf-py) to within its step of the source."""
    import sys
    sys.path.insert(0, str(ROOT))
    from oracle import oracle as o
    rng = np.random.default_rng(qtype)
    n, k = 7, 512
    w = rng.normal(0, 0.02, (n, k)).astype(np.float32)
    w[rng.random(w.shape) < 0.01] *= 8.0
    w[3] = 0.0  # an all-zero row
    rows = samq.quantize_rows(qtype, w)
    assert rows.nbytes == n * samq.row_bytes(qtype, k)
    if qtype == 8:
        assert np.array_equal(rows, o.quantize(8, w).ravel())
    dec = o.dequantize(qtype, rows, n * k).reshape(n, k)
    assert np.all(dec[3] == 0.0)
    # the decoded error is no worse than that of the oracle's own packer for the format
    ref = o.dequantize(qtype, o.quantize(qtype, w), n * k).reshape(n, k)
    err, ref_err = np.linalg.norm(dec - w), np.linalg.norm(ref - w)
    assert err <= 1.05 * ref_err + 1e-9, (err, ref_err)
    assert err <= {8: 0.01, 12: 0.12, 13: 0.06, 14: 0.04}[qtype] * np.linalg.norm(w)
    with pytest.raises(samq.SamqError):
        samq.quantize_rows(qtype, np.full((1, 256), np.nan, np.float32))
