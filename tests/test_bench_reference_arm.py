"""The benchmark's reference arm on CPU: `bench.py --impl reference` times the
CPU restatement of the path on the host cores and prints the same JSON line as
the GPU arm, with `impl: reference`; ranks other than 0 print nothing. Each
timed step is one whole unit of the workload (one image through all 32 blocks,
or one full operator call), so ms_per_step is a time that was measured."""
import json
import os
import subprocess
import sys

from conftest import ROOT

BENCH = os.path.join(ROOT, "bench.py")


def _run(extra_env, *args):
    env = dict(os.environ, **extra_env)
    return subprocess.run([sys.executable, BENCH, "--impl", "reference", *args],
                          capture_output=True, text=True, timeout=600, env=env, cwd=ROOT)


def test_reference_arm_prints_one_json_line_with_the_contract_keys():
    r = _run({"WORLD_SIZE": "1", "RANK": "0", "LOCAL_RANK": "0"}, "--steps", "1", "--warmup", "0")
    assert r.returncode == 0, r.stderr
    lines = [ln for ln in r.stdout.splitlines() if ln.strip()]
    assert len(lines) == 1
    d = json.loads(lines[0])
    assert d["impl"] == "reference"
    assert d["unit"] == "images/s" and d["higher_is_better"] is True
    assert d["metric"].startswith("encoder images/s at 1008^2")
    assert d["value"] > 0 and d["n_gpus"] == 1 and d["steps"] == 1 and d["warmup"] == 0
    assert d["config"]["images"] == 64 and d["data"] == "synthetic"
    cb = d["cpu_baseline"]
    assert cb["kind"] == "port" and cb["cores"] >= 1 and cb["value"] == d["value"]
    assert "1008^2" in cb["sample"]
    assert d["e2e"] == {"value": d["value"], "unit": "images/s", "h2d_bytes_per_step": 0,
                        "d2h_bytes_per_step": 0}
    # one measured image per step
    assert abs(d["ms_per_step"] - 1e3 / d["value"]) < 1e-6 * d["ms_per_step"]
    assert "timed whole" in cb["sample"]


def test_reference_arm_single_operator_config():
    r = _run({"WORLD_SIZE": "1", "RANK": "0", "LOCAL_RANK": "0"}, "--config", "c0",
             "--steps", "2", "--warmup", "1")
    assert r.returncode == 0, r.stderr
    d = json.loads([ln for ln in r.stdout.splitlines() if ln.strip()][0])
    assert d["unit"] == "TFLOP/s" and d["metric"].startswith("c0 palettized QKV projection")
    gflop = 2 * 5184 * 3072 * 1024 / 1e9
    assert abs(d["config"]["algorithmic_gflop_per_call"] - gflop) < 1e-6
    # value is the measured call's FLOP rate
    assert abs(d["value"] - gflop / d["ms_per_step"]) < 1e-6 * d["value"]


def test_reference_arm_other_ranks_exit_quietly():
    r = _run({"WORLD_SIZE": "2", "RANK": "1", "LOCAL_RANK": "1"}, "--steps", "1", "--warmup", "0")
    assert r.returncode == 0, r.stderr
    assert r.stdout.strip() == ""
