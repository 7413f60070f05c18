"""Host-side helpers of bench.py on CPU: the algorithmic FLOP counts behind
`roofline.achieved`, the peak and traffic files behind `roofline.peak` and
`roofline.traffic`, and the parsing of nvidia-smi clock samples."""
import json
import os
import sys

from conftest import ROOT

sys.path.insert(0, ROOT)
import bench  # noqa: E402


def test_encoder_flops_per_image_match_the_workload():
    f = bench.encoder_flops_per_image()
    # 16 blocks at 5184 tokens + 16 at 2592: linear 130.46 + 65.23 GFLOP per
    # block pair, attention 110.08 + 27.52; patch embedding 5184 x 1024 x 588 x 2
    assert abs(f["gemm"] / 1e9 - 3131.0) < 0.5
    assert abs(f["attention"] / 1e9 - 2201.5) < 0.5
    assert abs(f["patch"] / 1e9 - 6.24) < 0.01


def test_peaks_measured_file_or_stated_fallback(tmp_path, monkeypatch):
    monkeypatch.setattr(bench, "ROOT", str(tmp_path))
    p = bench.load_peaks()
    assert p["source"] == "fallback"
    assert (p["bf16_tflops"], p["bf16_tflops_sustained"], p["hbm_gbs"]) == (1590.0, 1400.0, 6650.0)
    (tmp_path / "MEASURED_PEAKS.json").write_text(json.dumps(
        {"bf16_tflops": 1662.1, "bf16_tflops_sustained": 1380.9, "hbm_gbs": 6547.8}))
    p = bench.load_peaks()
    assert p["source"] == "measured" and p["bf16_tflops_sustained"] == 1380.9


def test_committed_traffic_summary_gives_the_mean_per_launch():
    t = bench.load_traffic()
    assert t is not None
    per = [s["dram_read_bytes"] + s["dram_write_bytes"] for s in t["shapes"].values()]
    assert len(per) == 8  # the eight encoder GEMM shapes (pre / post prune)
    assert abs(t["bytes_per_launch_weighted"] - sum(per) / len(per)) < 1.0
    assert 5.0e8 < t["bytes_per_launch_weighted"] < 6.0e8


class _DoneProc:
    def terminate(self):
        pass

    def wait(self, timeout=None):
        return 0


def _sampler_with(rows, uuid):
    s = bench.ClockSampler(uuid)
    s.file.write("".join(", ".join(r) + "\n" for r in rows))
    s.proc = _DoneProc()
    return s


def test_clock_samples_median_under_load_and_reasons():
    mine, other = "GPU-aaaa", "GPU-bbbb"
    row = lambda u, sm, cap="Not Active", th="Not Active": [  # noqa: E731
        "0", u, str(sm), "1965", "900.0", "0x0", "Not Active", "Not Active", th, cap]
    rows = [row(mine, 300), row(mine, 1770, cap="Active"), row(mine, 1755),
            row(mine, 1780, cap="Active"), row(other, 900, th="Active")]
    s = _sampler_with(rows, mine)
    r = s.stop()
    # median of the upper half of this GPU's samples (idle start excluded);
    # the other GPU's thermal reason is not this run's
    assert r["sm_mhz"] == 1775.0 and r["sm_max_mhz"] == 1965.0
    assert r["reasons"] == ["sw_power_cap"] and r["samples"] == 4
    assert not os.path.exists(s.file.name)  # the sample file is removed


def test_clock_sampler_without_nvidia_smi_reports_nothing():
    s = bench.ClockSampler(None)
    s.proc = None
    assert s.stop() is None
    assert not os.path.exists(s.file.name)
