"""The C++ host layer (sam.cpp_b200/host/samq_backend.hpp) driven by a C++
test program, the way the reference's runtime tests drive its backend."""
import os
import subprocess

import numpy as np
import pytest

from conftest import PACKAGE, ROOT

CXX = "/usr/bin/g++" if os.path.exists("/usr/bin/g++") else "g++"
CUDA = "/usr/local/cuda"


def compile_test(out):
    cmd = [CXX, "-std=c++17", "-O2", "-Wall", "-Wextra", f"-I{ROOT / 'include'}", f"-I{PACKAGE / 'host'}",
           f"-I{CUDA}/include", str(ROOT / "tests" / "cpp" / "test_samq_backend.cpp"), "-o", str(out),
           f"-L{PACKAGE}", "-lsamq", f"-L{CUDA}/lib64", "-lcudart", f"-Wl,-rpath,{PACKAGE}",
           f"-Wl,-rpath,{CUDA}/lib64"]
    subprocess.run(cmd, check=True)


def test_host_header_compiles(tmp_path):
    """Syntax/type check of the C++ host layer against include/samq.h (no GPU)."""
    src = tmp_path / "inc.cpp"
    src.write_text('#include "samq_backend.hpp"\nint main() { return 0; }\n')
    subprocess.run([CXX, "-std=c++17", "-fsyntax-only", "-Wall", "-Wextra", f"-I{ROOT / 'include'}",
                    f"-I{PACKAGE / 'host'}", f"-I{CUDA}/include", str(src)], check=True)


@pytest.mark.gpu
@pytest.mark.parametrize("qtype,epilogue", [(8, 0), (12, 1), (14, 0)])
def test_cpp_host_layer_on_gpu(tmp_path, oracle, qtype, epilogue):
    rng = np.random.default_rng(qtype)
    k, n, m = 1024, 384, 150
    w = rng.normal(0, 0.02, (n, k)).astype(np.float32)
    rows = oracle.quantize(qtype, w)
    x = rng.normal(0, 1, (m, k)).astype(np.float32)
    bias = rng.normal(0, 0.1, n).astype(np.float32)
    ref = oracle.gemm_f64(oracle.dequantize(qtype, rows, n * k).reshape(n, k),
                          oracle.q8_1_decode(oracle.quantize_q8_1(x), m, k), bias=bias, epilogue=epilogue)
    (tmp_path / "meta.txt").write_text(f"{qtype} {k} {n} {m} {epilogue}\n")
    rows.tofile(tmp_path / "rows.bin")
    x.tofile(tmp_path / "x.bin")
    bias.tofile(tmp_path / "bias.bin")
    ref.astype(np.float32).tofile(tmp_path / "ref.bin")
    exe = tmp_path / "test_samq_backend"
    compile_test(exe)
    run = subprocess.run([str(exe), str(tmp_path)], capture_output=True, text=True, timeout=120)
    assert run.returncode == 0, run.stdout + run.stderr


def compile_program(name, out):
    cmd = [CXX, "-std=c++17", "-O2", "-Wall", "-Wextra", f"-I{ROOT / 'include'}", f"-I{PACKAGE / 'host'}",
           f"-I{CUDA}/include", str(ROOT / "tests" / "cpp" / name), "-o", str(out),
           f"-L{PACKAGE}", "-lsamq", f"-L{CUDA}/lib64", "-lcudart", f"-Wl,-rpath,{PACKAGE}",
           f"-Wl,-rpath,{CUDA}/lib64"]
    subprocess.run(cmd, check=True)


def test_vit_backbone_host_program_compiles(tmp_path):
    compile_program("test_vit_backbone.cpp", tmp_path / "test_vit_backbone")


@pytest.mark.gpu
def test_cpp_vit_backbone_on_gpu(tmp_path, oracle):
    """VitBackbone::encode (prefix + one windowed block) from C++, its linears
    loaded from a gguf-py checkpoint by the host GGUF reader, against the f64
    oracle; same bar as the block test on the block's contribution."""
    rng = np.random.default_rng(11)
    size, patch, pos_grid, E, MLP, window = 336, 14, 8, 1024, 4736, 24
    files = {}
    files["image"] = ((rng.random((3, size, size)) - 0.5) / 0.5).astype(np.float32)
    files["patch_w"] = rng.normal(0, 0.02, (E, 3, patch, patch)).astype(np.float32)
    files["pos"] = rng.normal(0, 0.02, (pos_grid, pos_grid, E)).astype(np.float32)
    files["ln_w"] = (1 + rng.normal(0, 0.02, E)).astype(np.float32)
    files["ln_b"] = rng.normal(0, 0.02, E).astype(np.float32)
    blk = {"window": window}
    import gguf
    writer = gguf.GGUFWriter(str(tmp_path / "weights.gguf"), "sam3")
    for name, gname, n, k, t in (("qkv", "attn.qkv", 3 * E, E, 12), ("proj", "attn.proj", E, E, 12),
                                 ("fc1", "mlp.lin1", MLP, E, 12), ("fc2", "mlp.lin2", E, MLP, 8)):
        w = rng.normal(0, 0.02, (n, k)).astype(np.float32)
        rows = oracle.quantize(t, w)
        writer.add_tensor(f"vit.blocks.0.{gname}.weight", rows.reshape(n, -1), raw_dtype=gguf.GGMLQuantizationType(t))
        blk[name + "_w"] = oracle.dequantize(t, rows, n * k).reshape(n, k)
        blk[name + "_b"] = files[name + "_b"] = rng.normal(0, 0.02, n).astype(np.float32)
    writer.write_header_to_file()
    writer.write_kv_data_to_file()
    writer.write_tensors_to_file()
    writer.close()
    for name in ("norm1", "norm2"):
        blk[name + "_w"] = files[name + "_w"] = (1 + rng.normal(0, 0.02, E)).astype(np.float32)
        blk[name + "_b"] = files[name + "_b"] = rng.normal(0, 0.02, E).astype(np.float32)
    blk["freqs"] = files["freqs"] = oracle.rope_freqs(window * window, seed=3)
    for name, arr in files.items():
        np.ascontiguousarray(arr).tofile(tmp_path / f"{name}.bin")
    (tmp_path / "meta.txt").write_text(f"{size} {patch} {pos_grid} {E} {MLP} {window} 12 8\n")
    exe = tmp_path / "test_vit_backbone"
    compile_program("test_vit_backbone.cpp", exe)
    run = subprocess.run([str(exe), str(tmp_path)], capture_output=True, text=True, timeout=180)
    assert run.returncode == 0, run.stdout + run.stderr
    grid = size // patch
    out = np.fromfile(tmp_path / "out.bin", dtype=np.float32).reshape(grid * grid, E)
    x0 = oracle.vit_prefix(files["image"], patch, files["patch_w"], files["pos"], files["ln_w"], files["ln_b"])
    ref = oracle.vit_block(x0, blk, grid, grid)
    # Prefix and block errors add up here; the bars are those of one block of
    # the whole-depth backbone test: the full output's normalized L2 <= 1e-2
    # and cosine >= 0.99995, the block contribution's cosine >= 0.9998 (it
    # also carries the prefix error).
    o64, r64 = out.astype(np.float64).ravel(), ref.astype(np.float64).ravel()
    nl2 = float(np.linalg.norm(o64 - r64) / np.linalg.norm(r64))
    cos = float(o64 @ r64 / (np.linalg.norm(o64) * np.linalg.norm(r64)))
    d_gpu = (out - x0).astype(np.float64).ravel()
    d_ref = (ref - x0).astype(np.float64).ravel()
    dcos = float(d_gpu @ d_ref / (np.linalg.norm(d_gpu) * np.linalg.norm(d_ref)))
    assert nl2 <= 1e-2 and cos >= 0.99995 and dcos >= 0.9998, (nl2, cos, dcos)


def test_neck_host_program_compiles(tmp_path):
    compile_program("test_neck.cpp", tmp_path / "test_neck")


@pytest.mark.gpu
def test_cpp_neck_on_gpu(tmp_path, oracle):
    """SimpleFpnNeck::forward from C++, its 11 F32 layers and biases loaded from
    a gguf-py checkpoint by the host GGUF reader (reduced widths E = 64, mid =
    D = 32), against the f64 oracle at a 6 x 4 grid."""
    import gguf
    rng = np.random.default_rng(31)
    gw, gh, E, mid, D = 6, 4, 64, 32, 32
    shapes = {"0.dconv_2x2_0": (E, mid, 2, 2), "0.dconv_2x2_1": (mid, D, 2, 2), "0.conv_1x1": (D, D, 1, 1),
              "0.conv_3x3": (D, D, 3, 3), "1.dconv_2x2": (E, mid, 2, 2), "1.conv_1x1": (D, mid, 1, 1),
              "1.conv_3x3": (D, D, 3, 3), "2.conv_1x1": (D, E, 1, 1), "2.conv_3x3": (D, D, 3, 3),
              "3.conv_1x1": (D, E, 1, 1), "3.conv_3x3": (D, D, 3, 3)}
    keys = ("s0_deconv1", "s0_deconv2", "s0_conv1x1", "s0_conv3x3", "s1_deconv1", "s1_conv1x1", "s1_conv3x3",
            "s2_conv1x1", "s2_conv3x3", "s3_conv1x1", "s3_conv3x3")
    writer = gguf.GGUFWriter(str(tmp_path / "weights.gguf"), "sam3")
    layers = {}
    for key, (name, shape) in zip(keys, shapes.items()):
        deconv = "dconv" in name
        fan_in = shape[0] if deconv else shape[1] * shape[2] * shape[3]
        w = (rng.normal(size=shape) / np.sqrt(fan_in)).astype(np.float32)
        b = rng.normal(0, 0.02, shape[1] if deconv else shape[0]).astype(np.float32)
        writer.add_tensor(f"neck.det.{name}.weight", w)
        writer.add_tensor(f"neck.det.{name}.bias", b)
        layers[key] = (w, b)
    writer.write_header_to_file()
    writer.write_kv_data_to_file()
    writer.write_tensors_to_file()
    writer.close()
    x = rng.normal(size=(gh, gw, E)).astype(np.float32)
    x.tofile(tmp_path / "x.bin")
    (tmp_path / "meta.txt").write_text(f"{gw} {gh} {E} {D}\n")
    exe = tmp_path / "test_neck"
    compile_program("test_neck.cpp", exe)
    run = subprocess.run([str(exe), str(tmp_path)], capture_output=True, text=True, timeout=120)
    assert run.returncode == 0, run.stdout + run.stderr
    refs = oracle.neck(x, layers)
    for i, ref in enumerate(refs):
        out = np.fromfile(tmp_path / f"out{i}.bin", dtype=np.float32).reshape(ref.shape)
        err = np.abs(out - ref).max() / np.abs(ref).max()
        assert err <= 2e-6, (i, err)
