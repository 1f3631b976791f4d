"""bench.py's reference arm on the CPU: the JSON line the driver reads.

The restated CPU backbone is replaced by a stub (a fixed two seconds per
image), so nothing heavy runs; what is checked is the line itself: impl,
metric and unit as the GPU arm's, value = 1000 / ms_per_step (a step is one
image), the same workload config as the GPU arm, and the e2e and
cpu_baseline objects the contract asks for."""
import argparse
import contextlib
import io
import json
import sys
from pathlib import Path

ROOT = Path(__file__).resolve().parents[1]
sys.path.insert(0, str(ROOT))

import bench  # noqa: E402


class StubBackbone:
    threads = 3

    def __init__(self, oracle_module):
        self.calls = 0

    def step(self):
        self.calls += 1
        return 2.0

    def describe(self):
        return "stub sample"


def run_line(monkeypatch, world=1, rank=0, steps=2, warmup=3):
    monkeypatch.setattr(bench, "CpuBackbone", StubBackbone)
    args = argparse.Namespace(steps=steps, warmup=warmup)
    out = io.StringIO()
    with contextlib.redirect_stdout(out):
        bench.run_reference(args, world, rank)
    lines = [l for l in out.getvalue().splitlines() if l.strip()]
    return [json.loads(l) for l in lines]


def test_reference_line_keys_and_value(monkeypatch):
    (line,) = run_line(monkeypatch)
    assert line["impl"] == "reference"
    assert line["metric"] == bench.METRIC
    assert line["unit"] == "images/s" and line["higher_is_better"] is True
    assert line["value"] == 0.5
    assert abs(line["value"] - 1000.0 / line["ms_per_step"]) < 1e-12
    assert line["steps"] == 2 and line["warmup"] == 3
    assert line["config"] == bench.workload_config(1)
    e2e = line["e2e"]
    assert e2e["value"] == line["value"] and e2e["unit"] == line["unit"]
    assert e2e["h2d_bytes_per_step"] == 0 and e2e["d2h_bytes_per_step"] == 0
    cpu = line["cpu_baseline"]
    assert cpu["value"] == line["value"] and cpu["kind"] == "port" and cpu["cores"] == 3
    assert cpu["sample"] == "stub sample"


def test_reference_line_only_on_rank_zero(monkeypatch):
    assert run_line(monkeypatch, world=2, rank=1) == []
    (line,) = run_line(monkeypatch, world=2, rank=0)
    assert line["n_gpus"] == 2 and line["config"] == bench.workload_config(2)
