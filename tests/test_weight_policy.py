"""Weight-precision policy of the host loader (sam.cpp_b200/host/weight_policy.hpp,
mirroring src/models/sam3/weights.hpp): which GGUF type every SAM 3 image
tensor must have under the schema-3 / schema-4 profiles and the SHA-256-bound
mixed (schema 5/6/7) policy, and the checkpoint-level checks a loader runs
before it uploads any weight.

Known answers come from the reference's own tests:
  - tests/runtime/ggml/test_quantization.cpp:106-167 (profiles, the 4736-wide
    fc2 Q8_0 fallback, vision-only versus full profiles, counts) and :170-230
    (module lists, per-module counts and parameters);
  - tests/runtime/ggml/test_mixed_quantization.cpp:40-46 (the canonical policy
    text), :288-300 (mixed counts), :318-340 (tensor overrides and the pinned
    policy identity c290f907...), :363-370 (the F16 policy).
The counts need the names and shapes of the 348 linear weights the policy can
quantize (src/models/sam3/tensors.hpp:108-432), restated in `inventory()`;
every other tensor of the 1133-tensor image registry is F32 under every
profile, so the reference's F32 count is 1133 - 348 = 785.
"""
import hashlib
import subprocess

import numpy as np
import pytest

from conftest import PACKAGE, ROOT

gguf = pytest.importorskip("gguf")
CXX = "/usr/bin/g++"
F32, F16, Q8_0, Q4_K, Q5_K, Q6_K = 0, 1, 8, 12, 13, 14
MODULE_CSV = "vision=q4_k,text=q8_0,fusion=q6_k,decoder=q5_k"
ENCODED = "sam3:image-mixed-linear-v1\nbase=q4_k\nvision=q4_k\ntext=q8_0\nfusion=q6_k\ndecoder=q5_k\n"
TENSOR_CSV = ("ddec.layers.0.linear1.weight=f32,fenc.layers.0.linear1.weight=q5_k,"
              "text.resizer.weight=q4_k,vit.blocks.0.attn.qkv.weight=q6_k")
TENSOR_IDENTITY = "c290f907480a3b3cadc5304989e2d4463ba0e8ca1e414a18bcf63bcfca17f471"
F16_MODULE_CSV = "vision=f16,text=q8_0,fusion=q6_k,decoder=q4_k"
F16_TENSOR_CSV = "text.resizer.weight=f16,vit.blocks.0.attn.qkv.weight=q5_k"
F16_ENCODED = ("sam3:image-mixed-f16-linear-v1\nbase=q4_k\nvision=f16\ntext=q8_0\nfusion=q6_k\ndecoder=q4_k\n"
               "tensor:text.resizer.weight=f16\ntensor:vit.blocks.0.attn.qkv.weight=q5_k\n")


@pytest.fixture(scope="module")
def policy(tmp_path_factory):
    exe = tmp_path_factory.mktemp("policy") / "test_weight_policy"
    subprocess.run([CXX, "-std=c++17", "-O2", "-Wall", "-Wextra", f"-I{PACKAGE / 'host'}",
                    str(ROOT / "tests" / "cpp" / "test_weight_policy.cpp"), "-o", str(exe)], check=True)

    def ask(lines):
        r = subprocess.run([str(exe)], input="\n".join(lines) + "\n", capture_output=True, text=True, timeout=120)
        assert r.returncode == 0, r.stderr
        return r.stdout.splitlines()
    return ask


def inventory():
    """(name, dimensions) of the linear weights the policy's whitelist names, GGML
    order (dimensions[0] = row width), by module (tensors.hpp:108-432).  A
    [256, 1] weight is stored by GGUF as rank 1."""
    D, FFN = 256, 2048
    mods = {"vision": [], "text": [("text.resizer.weight", [1024, 256])], "fusion": [], "decoder": []}
    for b in range(32):
        p = f"vit.blocks.{b}."
        mods["vision"] += [(p + "attn.qkv.weight", [1024, 3072]), (p + "attn.proj.weight", [1024, 1024]),
                           (p + "mlp.lin1.weight", [1024, 4736]), (p + "mlp.lin2.weight", [4736, 1024])]
    for b in range(24):
        p = f"text.blocks.{b}."
        mods["text"] += [(p + "attn.in_proj.weight", [1024, 3072]), (p + "attn.out_proj.weight", [1024, 1024]),
                         (p + "mlp.fc1.weight", [1024, 4096]), (p + "mlp.fc2.weight", [4096, 1024])]
    layer = {"sa.in_proj_weight": [D, 3 * D], "sa.out_proj.weight": [D, D], "ca.in_proj_weight": [D, 3 * D],
             "ca.out_proj.weight": [D, D], "linear1.weight": [D, FFN], "linear2.weight": [FFN, D]}
    for b in range(6):
        mods["fusion"] += [(f"fenc.layers.{b}.{s}", d) for s, d in layer.items()]
    dec = dict(layer)
    dec.update({"ca_text.in_proj_weight": [D, 3 * D], "ca_text.out_proj.weight": [D, D]})
    for b in range(6):
        mods["decoder"] += [(f"ddec.layers.{b}.{s}", d) for s, d in dec.items()]
    for b in range(3):
        mods["decoder"] += [(f"geom.layers.{b}.{s}", d) for s, d in layer.items()]
    for j in range(3):
        mods["decoder"] += [(f"ddec.bbox_embed.layers.{j}.weight", [D, 4 if j == 2 else D]),
                            (f"ddec.presence_token_head.layers.{j}.weight", [D] if j == 2 else [D, D]),
                            (f"seg.mask_predictor.mask_embed.layers.{j}.weight", [D, D])]
    mods["decoder"] += [("ddec.ref_point_head.layers.0.weight", [512, D]), ("ddec.ref_point_head.layers.1.weight", [D, D])]
    for axis in "xy":
        mods["decoder"] += [(f"ddec.boxRPB_embed_{axis}.layers.0.weight", [2, D]),
                            (f"ddec.boxRPB_embed_{axis}.layers.1.weight", [D, 8])]
    mods["decoder"] += [("scoring.prompt_proj.weight", [D, D]), ("scoring.hs_proj.weight", [D, D]),
                        ("scoring.prompt_mlp.layers.0.weight", [D, FFN]), ("scoring.prompt_mlp.layers.1.weight", [FFN, D]),
                        ("geom.points_direct_project.weight", [2, D]), ("geom.boxes_direct_project.weight", [4, D]),
                        ("geom.boxes_pos_enc_project.weight", [258, D]), ("geom.points_pool_project.weight", [D, D]),
                        ("geom.points_pos_enc_project.weight", [D, D]), ("geom.final_proj.weight", [D, D]),
                        ("seg.cross_attend_prompt.in_proj_weight", [D, 3 * D]),
                        ("seg.cross_attend_prompt.out_proj.weight", [D, D])]
    return mods


def _dims(d):
    return " ".join(str(v) for v in d)


def test_sha256_matches_hashlib(policy):
    texts = ["", "abc", "a" * 55, "a" * 56, "a" * 64, "a" * 119, ENCODED, F16_ENCODED]
    out = policy(["sha256 " + t.replace("\n", "\\n") for t in texts])
    assert out == [hashlib.sha256(t.encode()).hexdigest() for t in texts]


def test_policy_identity_known_answer():
    """The reference pins the schema-6 policy text's digest
    (test_mixed_quantization.cpp:320); the canonical text this header builds
    for that allocation must hash to it."""
    text = ("sam3:image-tensor-mixed-linear-v1\nbase=q4_k\nvision=q4_k\ntext=q8_0\nfusion=q6_k\ndecoder=q5_k\n"
            + "".join(f"tensor:{f}\n" for f in TENSOR_CSV.split(",")))
    assert hashlib.sha256(text.encode()).hexdigest() == TENSOR_IDENTITY


def test_profiles_and_fc2_fallback(policy):
    """test_quantization.cpp:115-165."""
    out = policy([
        "image image-vision-linear-q6_k-v1 vit.blocks.0.mlp.lin2.weight 4736 1024",
        "image image-linear-q4_k-v1 vit.blocks.31.mlp.lin2.weight 4736 1024",
        "image image-linear-q6_k-v1 vit.blocks.0.mlp.lin2.weight 4864 1024",
        "image image-linear-q6_k-v1 vit.blocks.0.attn.qkv.weight 4736 3072",
        "image image-linear-q6_k-v1 vit.blocks.0.attn.qkv.weight 1024 3072",
        "image image-linear-q5_k-v1 text.blocks.23.mlp.fc2.weight 1024 3072",
        "image image-linear-q8_0-v1 vit.blocks.0.attn.qkv.weight 1024 3072",
        "image image-linear-q8_0-v1 text.blocks.0.attn.in_proj.weight 1024 3072",
        "image image-vision-linear-q8_0-v1 text.blocks.0.attn.in_proj.weight 1024 3072",
        "image image-vision-linear-q6_k-v1 text.blocks.23.mlp.fc2.weight 1024 3072",
        "image image-linear-q4_k-v1 vit.blocks.32.attn.qkv.weight 1024 3072",
        "image image-linear-q4_k-v1 vit.blocks.0.mlp.lin2.bias 1024",
        "image image-linear-q8_0-v1 neck.det.0.conv_1x1.weight 256 256 1 1",
        "image q4_k vit.blocks.0.attn.qkv.weight 1024 3072",
    ])
    assert out[:2] == ["8", "8"] and out[2] == "14"
    assert out[3].startswith("ERROR") and "noncanonical row width" in out[3]
    assert out[4:10] == ["14", "13", "8", "8", "0", "0"]
    assert out[10:13] == ["0", "0", "0"]
    assert out[13].startswith("ERROR")


def test_module_lists(policy):
    """test_quantization.cpp:172-178."""
    out = policy(["modules vision,text,fusion,decoder", "modules vision", "modules text,vision",
                  "modules vision,vision", "modules vision,text,", "modules vision,cuda"])
    assert out[:2] == ["vision,text,fusion,decoder", "vision"]
    assert all(line.startswith("ERROR") for line in out[2:])


def _types(policy, prefix, names_dims):
    return [int(v) for v in policy([f"{prefix} {n} {_dims(d)}" for n, d in names_dims])]


def test_canonical_inventory_counts(policy):
    """Per-module counts and parameters of the schema-4 whitelist
    (test_quantization.cpp:206-229), the vision-only and full schema-3 counts
    (:141-160) and the K-quant fc2 fallbacks."""
    mods = inventory()
    everything = [t for m in ("vision", "text", "fusion", "decoder") for t in mods[m]]
    # 354 whitelisted names; 6 of them (row widths 2, 4, 258 and the rank-1
    # presence head) can never be quantized, which leaves the reference's 348.
    assert len(everything) == 354
    expected = {"vision": (128, 444596224), "text": (97, 302252032), "fusion": (36, 9437184),
                "decoder": (87, 18027520)}
    for module, (count, elements) in expected.items():
        types = _types(policy, f"modular image-full-linear-q8_0-v1 {module}", everything)
        chosen = [(n, d) for (n, d), t in zip(everything, types) if t != F32]
        assert len(chosen) == count and sum(int(np.prod(d)) for _, d in chosen) == elements, module
    full_q8 = _types(policy, "modular image-full-linear-q8_0-v1 vision,text,fusion,decoder", everything)
    full_q6 = _types(policy, "modular image-full-linear-q6_k-v1 vision,text,fusion,decoder", everything)
    assert sum(t != F32 for t in full_q8) == 348
    assert sum(int(np.prod(d)) for (n, d), t in zip(everything, full_q8) if t != F32) == 774312960
    assert sum(t != F32 for t in full_q6) == 348 and full_q6.count(Q8_0) == 32
    vision_q6 = _types(policy, "image image-vision-linear-q6_k-v1", everything)
    legacy_q6 = _types(policy, "image image-linear-q6_k-v1", everything)
    assert sum(t != F32 for t in vision_q6) == 128 and vision_q6.count(Q8_0) == 32
    assert sum(t != F32 for t in legacy_q6) == 224


def test_mixed_policy_counts_and_protection(policy):
    """test_mixed_quantization.cpp:288-300: vision Q4_K (fc2 Q8_0), text Q8_0,
    fusion Q6_K, decoder Q5_K; protected tensors stay F32."""
    sha = hashlib.sha256(ENCODED.encode()).hexdigest()
    prefix = f"mixed q4_k {MODULE_CSV} {sha} - -"
    everything = [t for m in ("vision", "text", "fusion", "decoder") for t in inventory()[m]]
    types = _types(policy, prefix, everything)
    counts = {t: types.count(t) for t in set(types)}
    # 6 whitelisted names can never be quantized (see the inventory test); with
    # the registry's 1133 tensors the F32 count is 1133 - 348 = 785, the reference's.
    assert counts == {Q4_K: 96, Q8_0: 129, Q6_K: 36, Q5_K: 87, F32: 6}
    out = policy([f"{prefix} geom.points_direct_project.weight 2 256", f"{prefix} text.token_embed.weight 256 2",
                  f"{prefix} ddec.presence_token_head.layers.2.weight 256",
                  f"mixed q4_k {MODULE_CSV} {'0' * 64} - - vit.blocks.0.attn.qkv.weight 1024 3072",
                  f"mixed q4_k vision=q4_k,text=q8_0,fusion=q6_k {sha} - - vit.blocks.0.attn.qkv.weight 1024 3072"])
    assert out[:3] == ["0", "0", "0"]
    assert "SHA-256" in out[3] and out[4].startswith("ERROR")


def test_tensor_overrides(policy):
    """test_mixed_quantization.cpp:318-340: exact-name overrides take
    precedence; malformed, duplicate, unsorted or ineligible ones are rejected."""
    prefix = f"mixed q4_k {MODULE_CSV} {TENSOR_IDENTITY} {TENSOR_CSV} -"
    out = policy([f"{prefix} vit.blocks.0.attn.qkv.weight 256 2", f"{prefix} text.resizer.weight 256 2",
                  f"{prefix} fenc.layers.0.linear1.weight 256 2", f"{prefix} ddec.layers.0.linear1.weight 256 2"])
    assert out == [str(Q6_K), str(Q4_K), str(Q5_K), str(F32)]
    invalid = ["vit.blocks.0.attn.qkv.weight=f16",
               "vit.blocks.0.attn.qkv.weight=q6_k,vit.blocks.0.attn.qkv.weight=f32",
               "vit.blocks.01.attn.qkv.weight=f32", "vit.blocks.32.attn.qkv.weight=f32", "text.token_embed.weight=f32",
               "vit.blocks.0.attn.qkv.weight=q6_k,text.resizer.weight=q4_k", "vit.blocks.*.attn.qkv.weight=f32"]
    out = policy([f"mixed q4_k {MODULE_CSV} {TENSOR_IDENTITY} {v} - vit.blocks.0.attn.qkv.weight 256 2"
                  for v in invalid])
    assert all(line.startswith("ERROR") for line in out), out


def test_f16_policy(policy):
    """test_mixed_quantization.cpp:363-370 (schema 7)."""
    sha = hashlib.sha256(F16_ENCODED.encode()).hexdigest()
    prefix = f"mixed q4_k {F16_MODULE_CSV} {sha} {F16_TENSOR_CSV} image-mixed-f16-linear-v1"
    out = policy([f"{prefix} vit.blocks.0.mlp.lin2.weight 4736 2", f"{prefix} vit.blocks.0.attn.qkv.weight 256 2",
                  f"{prefix} text.resizer.weight 256 2", f"{prefix} text.token_embed.weight 256 2",
                  f"mixed q4_k {F16_MODULE_CSV} {sha} {F16_TENSOR_CSV} - vit.blocks.0.attn.qkv.weight 256 2"])
    assert out[:4] == [str(F16), str(Q5_K), str(F16), str(F32)]
    assert out[4].startswith("ERROR")


def test_bench_formats_follow_the_policy(policy):
    """bench.py's config-3 weights (Q4_K linears, fc2 Q8_0) are what the
    vision-only Q4_K profile assigns to every ViT block."""
    import bench
    names = {"qkv": "attn.qkv.weight", "proj": "attn.proj.weight", "fc1": "mlp.lin1.weight", "fc2": "mlp.lin2.weight"}
    lines = [f"image image-vision-linear-q4_k-v1 vit.blocks.{b}.{names[n]} {k} {nn}"
             for b in (0, 31) for n, nn, k, *_ in bench.LINEARS]
    assert [int(v) for v in policy(lines)] == [qtype for _ in (0, 31) for _, _, _, qtype, *_ in bench.LINEARS]


# ---- checkpoint-level checks on gguf-py files ------------------------------------

SAM3_PARAMETERS = {
    "sam3.vision.image_size": 1008, "sam3.vision.patch_size": 14, "sam3.vision.embedding_length": 1024,
    "sam3.vision.block_count": 32, "sam3.vision.attention.head_count": 16, "sam3.vision.feed_forward_length": 4736,
    "sam3.vision.window_size": 24, "sam3.text.embedding_length": 1024, "sam3.text.attention.head_count": 16,
    "sam3.text.block_count": 24, "sam3.text.context_length": 32, "sam3.text.vocab_size": 49408,
    "sam3.text.output_length": 256, "sam3.neck.embedding_length": 256, "sam3.fusion.block_count": 6,
    "sam3.fusion.attention.head_count": 8, "sam3.fusion.feed_forward_length": 2048, "sam3.decoder.block_count": 6,
    "sam3.decoder.attention.head_count": 8, "sam3.decoder.feed_forward_length": 2048, "sam3.decoder.query_count": 200,
    "sam3.geometry.block_count": 3}
FIXTURE_TENSORS = ("vit.blocks.0.attn.qkv.weight", "text.resizer.weight", "fenc.layers.0.linear1.weight",
                   "ddec.layers.0.linear1.weight", "text.token_embed.weight", "vit.blocks.0.mlp.lin2.weight")


def write_mixed_fixture(path, oracle, change=None, wrong_type=False, types=None):
    """A schema-5 checkpoint (test_mixed_quantization.cpp:48-90): six tensors,
    each stored as the mixed policy assigns (or one deliberately not)."""
    meta = {"sam.schema_version": 5, "general.file_type": 14, "general.quantization_version": 2}
    strings = {"general.architecture": "sam3", "sam.task": "text_image", "sam.storage_profile": "image-mixed-linear-v1",
               "sam.quantization.base_precision": "q4_k", "sam.quantization.module_precisions": MODULE_CSV,
               "sam.quantization.policy_sha256": hashlib.sha256(ENCODED.encode()).hexdigest()}
    if change:
        change(meta, strings)
    w = gguf.GGUFWriter(str(path), "sam3")
    w.kv_data[0].pop("general.architecture", None)
    for key, value in meta.items():
        w.add_uint32(key, value)
    for key, value in strings.items():
        w.add_string(key, value)
    for key, value in SAM3_PARAMETERS.items():
        w.add_uint32(key, value)
    w.add_key_value("sam3.vision.global_attention_blocks", [7, 15, 23, 31], gguf.GGUFValueType.ARRAY,
                    sub_type=gguf.GGUFValueType.UINT32)
    rng = np.random.default_rng(1)
    for name in FIXTURE_TENSORS:
        width = 4736 if "lin2" in name else 256
        qtype = types[name]
        if wrong_type and name == "vit.blocks.0.attn.qkv.weight":
            qtype = Q8_0
        values = rng.normal(0, 0.02, (2, width)).astype(np.float32)
        if qtype == F32:
            w.add_tensor(name, values)
        else:
            w.add_tensor(name, oracle.quantize(qtype, values).reshape(2, -1), raw_dtype=gguf.GGMLQuantizationType(qtype))
    w.write_header_to_file()
    w.write_kv_data_to_file()
    w.write_tensors_to_file()
    w.close()


EXPECTED_FIXTURE_TYPES = {"vit.blocks.0.attn.qkv.weight": Q4_K, "text.resizer.weight": Q8_0,
                          "fenc.layers.0.linear1.weight": Q6_K, "ddec.layers.0.linear1.weight": Q5_K,
                          "text.token_embed.weight": F32, "vit.blocks.0.mlp.lin2.weight": Q8_0}


def test_inspect_mixed_checkpoint(policy, oracle, tmp_path):
    path = tmp_path / "mixed.gguf"
    write_mixed_fixture(path, oracle, types=EXPECTED_FIXTURE_TYPES)
    out = policy([f"inspect {path} 6", f"inspect {path} 1133"])
    assert out[0] == "5 mixed vision,text,fusion,decoder"
    listed = dict(line.split() for line in out[1:7])
    assert {k: int(v) for k, v in listed.items()} == EXPECTED_FIXTURE_TYPES and out[7] == "END"
    assert "tensor count" in out[8]


@pytest.mark.parametrize("what,change,wrong_type", [
    ("stored type differs from the policy", None, True),
    ("digest of another allocation", lambda m, s: s.update({"sam.quantization.policy_sha256": "0" * 64}), False),
    ("schema 6 without tensor overrides", lambda m, s: m.update({"sam.schema_version": 6}), False),
    ("module list beside module formats", lambda m, s: s.update({"sam.quantization.modules": "vision"}), False),
    ("file type of another base precision", lambda m, s: m.update({"general.file_type": 7}), False),
    ("quantization version 1", lambda m, s: m.update({"general.quantization_version": 1}), False),
    ("video task", lambda m, s: s.update({"sam.task": "text_video"}), False),
])
def test_inspect_rejects(policy, oracle, tmp_path, what, change, wrong_type):
    path = tmp_path / "bad.gguf"
    write_mixed_fixture(path, oracle, change=change, wrong_type=wrong_type, types=EXPECTED_FIXTURE_TYPES)
    out = policy([f"inspect {path} 6"])
    assert out[0].startswith("ERROR"), (what, out)
