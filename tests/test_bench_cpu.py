"""bench.py's host-side pieces that need no GPU: the clock-sample window, the job's GPU indices and the reference arm."""

from __future__ import annotations

import datetime

import bench


def _line(when: float, index: int, mhz: float, power_cap: bool = False, thermal: bool = False) -> str:
    stamp = datetime.datetime.fromtimestamp(when).strftime("%Y/%m/%d %H:%M:%S.%f")[:-3]
    active = "Active" if power_cap else "Not Active"
    hot = "Active" if thermal else "Not Active"
    return f"{stamp}, {index}, {mhz}, 1965, 900.00, 0x0000000000000000, Not Active, {hot}, Not Active, {active}"


def test_only_samples_inside_the_timed_region_count() -> None:
    t0 = 1_000_000.0
    lines = [_line(t0 - 1.0, 0, 300.0, thermal=True),      # idle, before the region
             _line(t0 + 0.1, 0, 1800.0, power_cap=True),
             _line(t0 + 0.2, 0, 1900.0),
             _line(t0 + 0.3, 0, 1850.0),
             _line(t0 + 2.0, 0, 400.0)]                    # after the region
    summary = bench.Clocks.summarize(lines, t0, t0 + 0.35, 1)
    assert summary["samples"] == 3 and summary["in_timed_region"]
    assert summary["sm_mhz"] == 1850.0 and summary["sm_max_mhz"] == 1965.0
    assert summary["reasons"] == ["sw_power_cap"]


def test_a_region_shorter_than_the_interval_takes_the_next_sample_of_each_gpu() -> None:
    t0 = 2_000_000.0
    lines = [_line(t0 + 0.5, 0, 1700.0), _line(t0 + 0.5, 1, 1750.0), _line(t0 + 0.6, 0, 1000.0)]
    summary = bench.Clocks.summarize(lines, t0, t0 + 0.01, 2)
    assert summary["samples"] == 2 and not summary["in_timed_region"]
    assert summary["sm_mhz"] == 1725.0 and summary["gpus"] == 2


def test_no_samples_gives_no_clock_record() -> None:
    assert bench.Clocks.summarize([], 0.0, 1.0, 1) is None
    assert bench.Clocks.summarize(["garbage"], 0.0, 1.0, 1) is None


def test_job_gpus_follow_the_visible_devices(monkeypatch) -> None:
    monkeypatch.delenv("CUDA_VISIBLE_DEVICES", raising=False)
    assert bench._job_gpu_indices(4) == [0, 1, 2, 3]
    monkeypatch.setenv("CUDA_VISIBLE_DEVICES", "4,5,6,7")
    assert bench._job_gpu_indices(2) == [4, 5]


def _reference_arm(extra_env: dict | None = None):
    import json
    import os
    import subprocess
    import sys
    env = dict(os.environ, **(extra_env or {}))
    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    done = subprocess.run([sys.executable, os.path.join(root, "bench.py"), "--impl", "reference", "--steps", "1",
                           "--warmup", "1", "--cpu-prompt", "16", "--cpu-decode", "1", "--prompt", "16",
                           "--decode", "4"],
                          capture_output=True, text=True, timeout=600, env=env, cwd=root)
    assert done.returncode == 0, done.stderr[-2000:]
    lines = [line for line in done.stdout.splitlines() if line.startswith("{")]
    return [json.loads(line) for line in lines]


def test_reference_arm_prints_one_contract_line() -> None:
    """The reference arm (the reference's host path, timed on the host cores) needs no GPU: one JSON line with the
    workload's metric, its own CPU-baseline record and an end-to-end record with no host-device traffic."""
    lines = _reference_arm({"RANK": "0"})
    assert len(lines) == 1
    line = lines[0]
    # both arms print the same metric: the headline the native arm reports
    assert line["impl"] == "reference" and line["metric"] == bench.METRIC and line["unit"] == "tok/s"
    assert line["higher_is_better"] is True and line["steps"] == 1 and line["value"] > 0
    baseline = line["cpu_baseline"]
    assert baseline["kind"] == "port" and baseline["cores"] >= 1 and baseline["value"] == line["value"]
    assert "16-token prefill" in baseline["sample"] and "extrapolated per sequence" in baseline["sample"]
    assert baseline["host_cpus"] >= 1 and baseline["cpu_model"] and baseline["blas_threads"] >= 1
    assert baseline["literal_full_recompute_s_per_token"] > 0
    assert line["e2e"] == {"value": line["value"], "unit": "tok/s", "h2d_bytes_per_step": 0,
                           "d2h_bytes_per_step": 0}


def test_reference_arm_runs_on_rank_zero_only() -> None:
    assert _reference_arm({"RANK": "1", "WORLD_SIZE": "2"}) == []
