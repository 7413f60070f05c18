"""The benchmark's reference arm on CPU: `bench.py --impl reference` times the
CPU restatement of the path on the host cores and prints the same JSON line as
the GPU arm, with `impl: reference`; ranks other than 0 print nothing."""
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
    # 64 images at the measured per-image rate
    assert abs(d["ms_per_step"] - 64e3 / d["value"]) < 1e-6 * d["ms_per_step"]


def test_reference_arm_other_ranks_exit_quietly():
    r = _run({"WORLD_SIZE": "2", "RANK": "1", "LOCAL_RANK": "1"}, "--steps", "1", "--warmup", "0")
    assert r.returncode == 0, r.stderr
    assert r.stdout.strip() == ""
