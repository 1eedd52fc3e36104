"""The parts of ``bench.py`` that run without a GPU: the clock sampler's summary of nvidia-smi
samples (NVML thread or nvidia-smi CSV; median SM clock, throttle reasons that invalidate a run) and the reference arm's
``unavailable`` line for tensor-parallel runs."""
import json
import os
import subprocess
import sys

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path.insert(0, ROOT)

import bench  # noqa: E402


def test_clock_summary_takes_the_median_and_collects_active_reasons(tmp_path):
    s = bench.ClockSampler([0])
    s.path = str(tmp_path / "clocks.csv")
    rows = [
        "0, 1965, 1965, 700.5, 0x0, Not Active, Not Active, Not Active, Not Active",
        "0, 1800, 1965, 990.1, 0x4, Not Active, Not Active, Not Active, Active",
        "0, 1890, 1965, 985.0, 0x4, Not Active, Not Active, Not Active, Active",
        "garbage line",
    ]
    (tmp_path / "clocks.csv").write_text("\n".join(rows) + "\n")
    s._read_csv()
    out = s.summary()
    assert out["sm_mhz"] == 1890 and out["sm_max_mhz"] == 1965 and out["samples"] == 3
    assert out["reasons"] == ["sw_power_cap"] and out["power_w_max"] == 990.1


def test_clock_summary_without_samples_says_so(tmp_path):
    s = bench.ClockSampler([0])
    s.path = str(tmp_path / "missing.csv")
    s._read_csv()
    assert s.summary() == {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unsampled"]}


class _FakeNvml:
    """The read-only NVML calls the sampler makes, with fixed answers."""
    NVML_CLOCK_SM = 1
    nvmlClocksEventReasonHwSlowdown = 0x8
    nvmlClocksEventReasonHwThermalSlowdown = 0x40
    nvmlClocksEventReasonSwThermalSlowdown = 0x20
    nvmlClocksEventReasonSwPowerCap = 0x4

    def __init__(self):
        self.calls = 0

    def nvmlDeviceGetCurrentClocksEventReasons(self, h):
        self.calls += 1
        return 0x4 if self.calls % 2 else 0x0

    def nvmlDeviceGetClockInfo(self, h, kind):
        return 1965 if self.calls % 2 else 1800

    def nvmlDeviceGetMaxClockInfo(self, h, kind):
        return 1965

    def nvmlDeviceGetPowerUsage(self, h):
        return 995_000

    def nvmlShutdown(self):
        pass


def test_clock_sampler_nvml_thread_samples_inside_a_short_window(monkeypatch):
    import time
    fake = _FakeNvml()
    monkeypatch.setattr(bench.ClockSampler, "_nvml_handles", lambda self: (fake, ["h0"]))
    with bench.ClockSampler([0], interval_s=0.005) as s:
        time.sleep(0.05)
    out = s.summary()
    assert out["source"] == "nvml" and out["samples"] >= 3
    assert out["sm_max_mhz"] == 1965 and out["power_w_max"] == 995.0 and out["reasons"] == ["sw_power_cap"]


def test_visible_indices_follow_cuda_visible_devices(monkeypatch):
    monkeypatch.setenv("CUDA_VISIBLE_DEVICES", "3,5,6")
    assert bench.visible_indices(2) == [3, 5]
    monkeypatch.delenv("CUDA_VISIBLE_DEVICES")
    assert bench.visible_indices(4) == [0, 1, 2, 3]


def test_reference_arm_at_tp2_prints_its_unavailable_line():
    proc = subprocess.run([sys.executable, "bench.py", "--impl", "reference", "--gpus", "2"], cwd=ROOT,
                          capture_output=True, text=True, timeout=300)
    assert proc.returncode == 0, proc.stderr[-2000:]
    line = json.loads(proc.stdout.strip().splitlines()[-1])
    assert line["impl"] == "reference" and "unavailable" in line


def test_window_latency_uses_finished_requests_only():
    recs = [
        {"arrival_time": 0.0, "first_token_time": 0.1, "finish_time": 1.1, "output_tokens": 11},   # tpot 0.1
        {"arrival_time": 0.0, "first_token_time": 0.3, "finish_time": 0.5, "output_tokens": 3},    # tpot 0.1
        {"arrival_time": 0.5, "first_token_time": 0.6, "finish_time": None, "output_tokens": 4},   # unfinished
    ]
    lat = bench.window_latency(recs)
    assert lat["requests"] == 2
    assert abs(lat["ttft_p50_ms"] - 200.0) < 1e-6 and abs(lat["ttft_p99_ms"] - 298.0) < 1e-6
    assert abs(lat["tpot_p99_ms"] - 100.0) < 1e-6
    assert bench.window_latency([])["tpot_p99_ms"] is None
