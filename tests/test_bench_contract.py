"""bench.py's output contract, on the CPU: the reference arm (the reference's own
torch DiT on the host cores, from the offline install in baseline/_ref, or the
oracle port when that is missing) prints one JSON line with every key the
contract names, on the default config (5); the GPU comparison arm says it is
unavailable without a GPU; a non-zero rank of the reference arm exits quietly."""

from __future__ import annotations

import json
import os
import subprocess
import sys
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parents[1]


def _run(args, env_extra=None, timeout=600):
    env = dict(os.environ)
    env.update(env_extra or {})
    return subprocess.run([sys.executable, str(ROOT / "bench.py"), *args], capture_output=True, text=True,
                          timeout=timeout, cwd=ROOT, env=env)


def _last_json(stdout: str) -> dict:
    lines = [l for l in stdout.splitlines() if l.startswith("{")]
    assert len(lines) == 1, stdout
    return json.loads(lines[0])


def test_reference_arm_prints_the_contract_line():
    r = _run(["--impl", "reference", "--steps", "1", "--warmup", "3"])
    assert r.returncode == 0, r.stderr[-2000:]
    line = _last_json(r.stdout)
    for k in ("metric", "value", "unit", "n_gpus", "steps", "warmup", "ms_per_step", "higher_is_better",
              "scaling", "vs_baseline", "dtype", "data", "config", "cpu_baseline", "e2e"):
        assert k in line, k
    assert line["impl"] == "reference"
    assert line["metric"] == "DiT estimator mel-frames/s (per NFE)" and line["unit"] == "mel-frames/s"
    assert line["value"] > 0 and line["steps"] == 1 and line["warmup"] == 3 and line["higher_is_better"] is True
    assert "workload" in line["config"] and line["config"]["workload"].startswith("config5")
    assert line["config"]["packed_rows"] == 96000
    cb = line["cpu_baseline"]
    assert cb["kind"] in ("port", "reference") and cb["cores"] >= 1 and cb["value"] == line["value"] and cb["sample"]
    if (ROOT / "baseline" / "_ref" / "faster_cosyvoice").is_dir():
        assert cb["kind"] == "reference", cb
    assert line["e2e"] == {"value": line["value"], "unit": "mel-frames/s", "h2d_bytes_per_step": 0,
                           "d2h_bytes_per_step": 0}


def test_reference_arm_other_ranks_do_nothing():
    r = _run(["--impl", "reference", "--steps", "1", "--warmup", "3"],
             {"RANK": "1", "WORLD_SIZE": "2", "LOCAL_RANK": "1"})
    assert r.returncode == 0, r.stderr[-2000:]
    assert not [l for l in r.stdout.splitlines() if l.startswith("{")]


@pytest.mark.skipif(__import__("torch").cuda.is_available(), reason="checks the no-GPU answer")
def test_gpu_comparison_arm_unavailable_without_gpu():
    r = _run(["--impl", "reference-gpu", "--config", "2"])
    assert r.returncode == 0, r.stderr[-2000:]
    line = _last_json(r.stdout)
    assert line["impl"] == "reference-gpu" and "unavailable" in line


def test_vocoder_reference_arm_prints_a_line():
    r = _run(["--vocoder", "--config", "2", "--impl", "reference", "--steps", "1", "--warmup", "3"])
    assert r.returncode == 0, r.stderr[-2000:]
    line = _last_json(r.stdout)
    assert line["impl"] == "reference" and line["metric"] == "vocoder mel-frames/s (HiFT decode)"
    assert line["value"] > 0 and line["cpu_baseline"]["value"] == line["value"] and line["cpu_baseline"]["sample"]
    assert line["config"]["finalize"] is True and line["config"]["requests"] == 8
    assert 1 <= line["config"]["measured_requests"] <= 8 and line["config"]["measured_mel_frames"] > 0
