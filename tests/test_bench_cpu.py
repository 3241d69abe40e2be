"""bench.py host logic on CPU: the clock-record summary the timing rules depend on, and the
reference arm's JSON line (the driver parses both)."""
import json
import os
import subprocess
import sys
from pathlib import Path

REPO = Path(__file__).resolve().parents[1]
sys.path.insert(0, str(REPO))

CONTRACT_KEYS = ("metric", "value", "unit", "n_gpus", "steps", "warmup", "ms_per_step", "higher_is_better",
                 "scaling", "vs_baseline", "dtype", "data", "config")


def _sampler(lines):
    import bench
    cs = bench.ClockSampler("GPU-00000000-0000-0000-0000-000000000000")
    cs.lines = list(lines)
    return cs.summary()


def test_clock_summary_median_max_and_power_cap():
    s = _sampler([
        "1965, 1965, 400.1, 0x0000000000000000, Not Active, Not Active, Not Active, Not Active",
        "1620, 1965, 998.0, 0x0000000000000004, Not Active, Not Active, Not Active, Active",
        "1580, 1965, 1001.2, 0x0000000000000004, Not Active, Not Active, Not Active, Active",
        "[N/A], [N/A]",  # a line nvidia-smi could not fill is skipped
    ])
    assert s["sm_mhz"] == 1620.0 and s["sm_max_mhz"] == 1965.0
    assert s["reasons"] == ["sw_power_cap"] and s["samples"] == 3


def test_clock_summary_reports_every_slowdown_reason():
    s = _sampler([
        "1200, 1965, 700.0, 0x0000000000000048, Active, Active, Not Active, Not Active",
        "1300, 1965, 700.0, 0x0000000000000020, Not Active, Not Active, Active, Not Active",
    ])
    assert s["reasons"] == ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown"]


def test_clock_summary_without_samples():
    assert _sampler([]) == {"sm_mhz": None, "sm_max_mhz": None, "reasons": [], "samples": 0,
                            "gpu": "GPU-00000000-0000-0000-0000-000000000000"}


class _Props:
    def __init__(self, uuid):
        self.uuid = uuid


def test_clock_sampler_names_the_gpu_by_uuid_not_by_cuda_ordinal(monkeypatch):
    """Under CUDA_VISIBLE_DEVICES=3 the process's CUDA device 0 is the node's GPU 3;
    nvidia-smi numbers GPUs node-wide, so the sampler must select by UUID."""
    import bench
    monkeypatch.setenv("CUDA_VISIBLE_DEVICES", "3")
    sel = bench.nvidia_smi_selector(_Props("6f1d2a3b-1111-2222-3333-444455556666"))
    assert sel == "GPU-6f1d2a3b-1111-2222-3333-444455556666"
    assert bench.nvidia_smi_selector(_Props("GPU-abc")) == "GPU-abc"  # already prefixed
    cs = bench.ClockSampler(sel)
    assert cs.gpu == sel and cs.summary()["gpu"] == sel
    import pytest
    with pytest.raises(ValueError):
        bench.nvidia_smi_selector(_Props(""))


def _reference_arm(extra_env=None):
    env = dict(os.environ)
    env.update(extra_env or {})
    return subprocess.run([sys.executable, str(REPO / "bench.py"), "--impl", "reference", "--m", "64", "--n", "48",
                           "--k", "40", "--steps", "2", "--warmup", "1"], capture_output=True, text=True,
                          timeout=600, cwd=REPO, env=env)


def test_reference_arm_prints_the_contract_line():
    out = _reference_arm()
    assert out.returncode == 0, out.stderr
    line = json.loads(out.stdout.strip().splitlines()[-1])
    for key in CONTRACT_KEYS + ("impl", "cpu_baseline", "e2e"):
        assert key in line, key
    assert line["impl"] == "reference" and line["steps"] == 2 and line["warmup"] == 1
    assert line["value"] > 0 and line["cpu_baseline"]["value"] == line["value"]
    assert line["cpu_baseline"]["kind"] == "port" and line["cpu_baseline"]["cores"] >= 1
    assert line["e2e"] == {"value": line["value"], "unit": line["unit"], "h2d_bytes_per_step": 0,
                           "d2h_bytes_per_step": 0}


def test_reference_arm_runs_on_rank_zero_only():
    out = _reference_arm({"RANK": "1"})
    assert out.returncode == 0, out.stderr
    assert out.stdout.strip() == ""


def test_roofline_peak_is_the_unscaled_burst_peak_with_the_clock_scaled_figure_beside_it():
    import bench
    pk = {"bf16_tflops": 1642.6, "bf16_tflops_sustained": 1377.5, "sm_max_mhz": 1965.0}
    peak, note = bench.tensor_roofline_peak(pk, "measured", {"sm_mhz": 1965.0, "sm_max_mhz": 1965.0})
    assert abs(peak - 1642.6 / 6) < 1e-9 and "maximum clock" in note
    peak, note = bench.tensor_roofline_peak(pk, "measured", {"sm_mhz": 1572.0, "sm_max_mhz": 1965.0})
    assert abs(peak - 1642.6 / 6) < 1e-9 and "not scaled" in note and "0.800" in note
    assert abs(bench.clock_scaled_peak(pk, {"sm_mhz": 1572.0, "sm_max_mhz": 1965.0}) - 1642.6 / 6 * 0.8) < 1e-9
    peak, _ = bench.tensor_roofline_peak(pk, "measured", {"sm_mhz": None, "sm_max_mhz": None})
    assert abs(peak - 1642.6 / 6) < 1e-9
