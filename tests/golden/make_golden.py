"""Generate the golden fixtures the oracle and the GPU kernels are pinned to.

Run in the development container (it needs gguf-py 0.19.0 and, for the
staging checks, the SAM.cpp reference tree):

    python tests/golden/make_golden.py [--reference /path/to/SAM.cpp]

Sources of truth:
  * gguf-py 0.19.0 (`gguf.quants`), the package the reference CI pins
    (.github/workflows/quick-checks.yml:22) and whose Q8_0 quantizer the
    reference converter calls (tools/convert/sam3_gguf.py:319-324):
    Q8_0 quantize bytes and Q8_0/Q4_K/Q5_K/Q6_K dequantized values.
  * The reference's own independent verifiers, imported from the reference
    tree: tools/validation/verify_q8_rhs_staging.py (check_blocks) and
    tools/validation/verify_q8_mmq_rhs_staging.py (check_blocks).  The Q8_1 and
    MMQ-D4 bytes stored here are the oracle's, accepted by those verifiers with
    zero errors and zero tie allowances.
The fixtures are small .npz files; tests read them on any machine.
"""
from __future__ import annotations

import argparse
import os
import importlib.util
import json
import sys
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
ROOT = HERE.parent.parent
sys.path.insert(0, str(ROOT))
from oracle import oracle as o  # noqa: E402


def load_module(path: Path, name: str):
    spec = importlib.util.spec_from_file_location(name, path)
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


def weight_matrix(rng, n, k):
    w = rng.normal(0.0, 0.02, (n, k)).astype(np.float32)
    mask = rng.random(w.shape) < 0.01
    w[mask] *= 8
    return w


def random_kquant_blocks(rng, qtype, count):
    """Arbitrary code bytes with finite, moderate f16 scales (any valid block)."""
    bb = o.lib().oracle_block_bytes(qtype)
    blocks = rng.integers(0, 256, (count, bb), dtype=np.uint8)
    scale = rng.uniform(1e-4, 2e-2, (count, 2)).astype(np.float16).view(np.uint8).reshape(count, 4)
    if qtype == o.Q6_K:
        blocks[:, 208:210] = scale[:, :2]
    else:
        blocks[:, 0:4] = scale
    return blocks.reshape(-1)


def activation_matrix(rng, rows, k):
    x = rng.normal(0.0, 1.0, (rows, k)).astype(np.float32)
    x[0, :] = 0.0                                   # all-zero blocks
    x[1, :32] = np.float32(1.0)                     # constant block
    x[1, 32:64] = np.linspace(-127, 127, 32, dtype=np.float32)  # exact .5 ties after scaling
    x[2, :32] *= np.float32(1e-20)                  # tiny magnitudes
    x[3, :32] *= np.float32(5000.0)                 # large magnitudes (f16 scale still finite)
    x[4, 5] = np.float32(-7.0)                      # negative extreme
    return x


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", type=Path, default=os.environ.get("SAM_REFERENCE_TREE"),
                    help="root of the SAM.cpp source tree (or set SAM_REFERENCE_TREE)")
    args = ap.parse_args()
    if args.reference is None:
        ap.error("--reference (or SAM_REFERENCE_TREE) must name the SAM.cpp source tree")
    args.reference = Path(args.reference)
    import gguf
    from gguf import GGMLQuantizationType as T

    o.build()
    rng = np.random.default_rng(20261201)
    manifest = {"gguf_version": getattr(gguf, "__version__", "0.19.0"), "fixtures": {}}

    # Q8_0 quantizer bytes (gguf-py is the reference converter's quantizer).
    w = weight_matrix(rng, 24, 512)
    w[0, :32] = 0.0
    w[1, :32] = np.linspace(-1, 1, 32, dtype=np.float32)
    q8 = gguf.quants.quantize(w, T.Q8_0)
    np.savez_compressed(HERE / "q8_0_quantize.npz", source=w, blocks=np.asarray(q8).reshape(-1))
    manifest["fixtures"]["q8_0_quantize"] = {"rows": 24, "k": 512}

    # Dequantization for every format: our packer's blocks and arbitrary blocks.
    for qtype, gt in [(o.Q8_0, T.Q8_0), (o.Q4_K, T.Q4_K), (o.Q5_K, T.Q5_K), (o.Q6_K, T.Q6_K)]:
        name = o.TYPE_NAMES[qtype]
        n, k = 16, 512
        packed = o.quantize(qtype, weight_matrix(rng, n, k))
        if qtype != o.Q8_0:
            packed = np.concatenate([packed, random_kquant_blocks(rng, qtype, 8)])
        bb = o.lib().oracle_block_bytes(qtype)
        be = o.lib().oracle_block_elements(qtype)
        values = gguf.quants.dequantize(packed.reshape(-1, bb), gt).reshape(-1).astype(np.float32)
        assert values.size == packed.size // bb * be
        np.savez_compressed(HERE / f"dequant_{name.lower()}.npz", blocks=packed, values=values)
        manifest["fixtures"][f"dequant_{name.lower()}"] = {"blocks": int(packed.size // bb)}

    # Q8_1 (MMVQ) and MMQ-D4 staging, validated by the reference verifiers.
    x = activation_matrix(rng, 65, 160)
    q8_1 = o.quantize_q8_1(x)
    d4 = o.quantize_mmq_d4(x)
    verdicts = {}
    vdir = args.reference / "tools" / "validation"
    if (vdir / "verify_q8_rhs_staging.py").exists():
        mmvq = load_module(vdir / "verify_q8_rhs_staging.py", "ref_verify_q8_rhs")
        mmq = load_module(vdir / "verify_q8_mmq_rhs_staging.py", "ref_verify_q8_mmq")
        verdicts["q8_1"] = mmvq.check_blocks(x.reshape(-1, 32), q8_1.reshape(-1, 36))
        padded = np.zeros((x.shape[0], 512), dtype=np.float32)
        padded[:, :160] = x
        blocks = d4.reshape(4, x.shape[0], 144)
        per = [mmq.check_blocks(padded[:, 128 * b:128 * (b + 1)], blocks[b]) for b in range(4)]
        verdicts["mmq_d4"] = {key: int(sum(p[key] for p in per)) for key in per[0]}
        for kind, v in verdicts.items():
            errors = sum(v[key] for key in v if key.endswith("errors"))
            allowances = sum(v[key] for key in v if "allowances" in key)
            if errors or allowances:
                raise SystemExit(f"{kind} staging rejected by the reference verifier: {v}")
    else:
        print("reference verifiers not found; staging fixtures are not pinned", file=sys.stderr)
    np.savez_compressed(HERE / "q8_staging.npz", source=x, q8_1=q8_1, mmq_d4=d4)
    manifest["fixtures"]["q8_staging"] = {"rows": 65, "k": 160, "reference_verdicts": verdicts}

    (HERE / "manifest.json").write_text(json.dumps(manifest, indent=2, default=int) + "\n")
    print(json.dumps(manifest, indent=2, default=int))


if __name__ == "__main__":
    main()
