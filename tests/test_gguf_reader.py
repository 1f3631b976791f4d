"""GGUF reader of the host layer (sam.cpp_b200/host/gguf_reader.hpp), no GGML:
files written by gguf-py 0.19.0 (the version the reference CI pins) are read by
a small C++ program (tests/cpp/test_gguf_reader.cpp) and its listing compared
with gguf-py's own view of the file; malformed files must be rejected with the
reference reader's reasons (src/io/gguf_reader.hpp)."""
import subprocess

import numpy as np
import pytest

from conftest import PACKAGE, ROOT

gguf = pytest.importorskip("gguf")
CXX = "/usr/bin/g++"


@pytest.fixture(scope="module")
def dump(tmp_path_factory):
    exe = tmp_path_factory.mktemp("gguf") / "test_gguf_reader"
    subprocess.run([CXX, "-std=c++17", "-O2", "-Wall", "-Wextra", f"-I{PACKAGE / 'host'}",
                    str(ROOT / "tests" / "cpp" / "test_gguf_reader.cpp"), "-o", str(exe)], check=True)

    def run(path):
        r = subprocess.run([str(exe), str(path)], capture_output=True, text=True, timeout=60)
        return r.returncode, r.stdout
    return run


def fnv1a64(data: bytes) -> str:
    h = 1469598103934665603
    for b in data:
        h = ((h ^ b) * 1099511628211) & 0xFFFFFFFFFFFFFFFF
    return f"{h:016x}"


def write_checkpoint(path, oracle, alignment=None):
    rng = np.random.default_rng(4)
    w = gguf.GGUFWriter(str(path), "sam3")
    if alignment:
        w.add_custom_alignment(alignment)
    w.add_uint32("sam3.vit.depth", 32)
    w.add_string("general.name", "synthetic-sam3")
    w.add_array("sam3.vit.global_blocks", [7, 15, 23, 31])
    tensors = {}
    for name, qtype, n, k in (("vit.blocks.0.attn.qkv.weight", 12, 24, 512), ("vit.blocks.0.mlp.lin2.weight", 8, 8, 96),
                              ("vit.blocks.0.attn.proj.weight", 14, 8, 256), ("vit.blocks.0.mlp.lin1.weight", 13, 4, 256)):
        rows = oracle.quantize(qtype, rng.normal(0, 0.02, (n, k)).astype(np.float32)).reshape(n, -1)
        w.add_tensor(name, rows, raw_dtype=gguf.GGMLQuantizationType(qtype))
        tensors[name] = (qtype, [k, n], rows.tobytes())
    bias = rng.normal(0, 1, 24).astype(np.float32)
    w.add_tensor("vit.blocks.0.attn.qkv.bias", bias)
    tensors["vit.blocks.0.attn.qkv.bias"] = (0, [24], bias.tobytes())
    half = rng.normal(0, 1, (3, 16)).astype(np.float16)
    w.add_tensor("vit.pos_embed.f16", half)
    tensors["vit.pos_embed.f16"] = (1, [16, 3], half.tobytes())
    w.write_header_to_file()
    w.write_kv_data_to_file()
    w.write_tensors_to_file()
    w.close()
    return tensors


def parse(listing):
    tensors, keys = {}, {}
    for line in listing.splitlines():
        parts = line.split()
        if parts[0] == "tensor":
            bar = parts.index("|")
            tensors[parts[1]] = (int(parts[2]), [int(d) for d in parts[3:bar]], int(parts[bar + 1]),
                                 int(parts[bar + 2]), parts[bar + 3])
        elif parts[0] == "key":
            keys[parts[1]] = parts[2:]
    return tensors, keys


def test_reads_gguf_py_checkpoint(tmp_path, oracle, dump):
    path = tmp_path / "model.gguf"
    expected = write_checkpoint(path, oracle)
    rc, out = dump(path)
    assert rc == 0, out
    tensors, keys = parse(out)
    reference = gguf.GGUFReader(str(path))
    offsets = {t.name: int(t.data_offset) for t in reference.tensors}
    assert set(tensors) == set(expected)
    for name, (qtype, dims, data) in expected.items():
        got_type, got_dims, size, offset, digest = tensors[name]
        assert (got_type, got_dims, size) == (qtype, dims, len(data)), name
        assert offset == offsets[name], name
        assert digest == fnv1a64(data), name
    assert keys["sam3.vit.depth"] == ["4", "32"]
    assert keys["general.name"] == ["8", "synthetic-sam3"]
    assert keys["general.architecture"] == ["8", "sam3"]
    assert keys["sam3.vit.global_blocks"] == ["9", "5", "4"]


def corrupt(src, dst, fn):
    data = bytearray(src.read_bytes())
    fn(data)
    dst.write_bytes(bytes(data))


@pytest.mark.parametrize("case,reason", [
    ("magic", "expected GGUF"),
    ("version", "GGUF v3"),
    ("tensor_padding", "nonzero GGUF tensor padding"),
    ("truncated", "truncated"),
    ("trailing", "unexpected data after GGUF tensor blob"),
])
def test_rejects_malformed_files(tmp_path, oracle, dump, case, reason):
    good = tmp_path / "good.gguf"
    write_checkpoint(good, oracle)
    reference = gguf.GGUFReader(str(good))
    bias = next(t for t in reference.tensors if t.name == "vit.blocks.0.attn.qkv.weight")
    end_of_first = int(bias.data_offset) + int(bias.n_bytes)  # 24 rows x 288 B = 6912: no padding after it
    f16 = next(t for t in reference.tensors if t.name == "vit.pos_embed.f16")  # 96 bytes + 0 padding
    q80 = next(t for t in reference.tensors if t.name == "vit.blocks.0.mlp.lin2.weight")  # 8 x 102 = 816 B -> 16 pad
    edits = {
        "magic": lambda d: d.__setitem__(slice(0, 4), b"GGUX"),
        "version": lambda d: d.__setitem__(slice(4, 8), (2).to_bytes(4, "little")),
        "tensor_padding": lambda d: d.__setitem__(int(q80.data_offset) + int(q80.n_bytes) + 3, 0x7F),
        "truncated": lambda d: d.__delitem__(slice(len(d) - 40, len(d))),
        "trailing": lambda d: d.extend(b"\x00" * 32),
    }
    assert end_of_first > 0 and int(f16.n_bytes) == 96
    bad = tmp_path / f"{case}.gguf"
    corrupt(good, bad, edits[case])
    rc, out = dump(bad)
    assert rc == 1 and reason in out, out


def test_rejects_alignment_other_than_32(tmp_path, oracle, dump):
    path = tmp_path / "aligned64.gguf"
    write_checkpoint(path, oracle, alignment=64)
    rc, out = dump(path)
    assert rc == 1 and "32-byte alignment" in out, out
