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
