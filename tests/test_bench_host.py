"""bench.py's reference arm runs on the host CPU: one JSON line with the keys the benchmark contract names."""
import json
import os
import subprocess
import sys

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def test_reference_arm_prints_one_contract_line():
    res = subprocess.run([sys.executable, "bench.py", "--impl", "reference", "--steps", "1", "--warmup", "3",
                          "--cpu-rows", "16"], cwd=ROOT, capture_output=True, text=True, timeout=600)
    assert res.returncode == 0, res.stderr[-2000:]
    lines = [l for l in res.stdout.splitlines() if l.startswith("{")]
    assert len(lines) == 1, res.stdout
    d = json.loads(lines[0])
    for key in ("metric", "value", "unit", "n_gpus", "steps", "warmup", "ms_per_step", "higher_is_better", "scaling",
                "vs_baseline", "dtype", "data", "config", "cpu_baseline", "e2e"):
        assert key in d, key
    assert d["impl"] == "reference" and d["metric"] == "W4A8 linear INT8-TOPS" and d["unit"] == "TOPS"
    assert d["config"]["workload"] == "w4a8_linear" and d["config"]["cpu_rows_per_step"] == 16
    assert d["value"] > 0 and d["steps"] == 1 and d["warmup"] == 3 and d["higher_is_better"] is True
    cb = d["cpu_baseline"]
    assert cb["kind"] == "port" and cb["cores"] >= 1 and cb["value"] == d["value"] and "16 of 4096 tokens" in cb["sample"]
    assert d["e2e"] == {"value": d["value"], "unit": "TOPS", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}


def test_clock_sampler_reports_median_clock_and_throttle_reasons(monkeypatch):
    """The timed region's clock record, from a fake NVML: median SM clock, the maximum, and every throttle reason
    seen in any sample (the bench only reads clocks; it sets nothing)."""
    import importlib
    import time
    import types
    sys.path.insert(0, ROOT)
    fake = types.SimpleNamespace(
        NVML_CLOCK_SM=1,
        nvmlClocksEventReasonSwPowerCap=0x4, nvmlClocksEventReasonHwSlowdown=0x8,
        nvmlClocksEventReasonHwThermalSlowdown=0x40, nvmlClocksEventReasonSwThermalSlowdown=0x20,
        nvmlClocksEventReasonHwPowerBrakeSlowdown=0x80)
    clocks = iter([1965, 1800, 1700] + [1965] * 10_000)
    reasons = iter([0x0, 0x4, 0x0] + [0x0] * 10_000)
    fake.nvmlInit = lambda: None
    fake.nvmlDeviceGetHandleByIndex = lambda i: ("gpu", i)
    fake.nvmlDeviceGetMaxClockInfo = lambda h, kind: 1965
    fake.nvmlDeviceGetClockInfo = lambda h, kind: next(clocks)
    fake.nvmlDeviceGetCurrentClocksEventReasons = lambda h: next(reasons)
    monkeypatch.setitem(sys.modules, "pynvml", fake)
    bench = importlib.import_module("bench")
    with bench.ClockSampler(0) as clk:
        time.sleep(0.05)
    s = clk.summary()
    assert s["sm_max_mhz"] == 1965 and s["samples"] >= 3
    assert s["reasons"] == ["sw_power_cap"]
    assert s["sm_mhz"] in (1800, 1965)


def test_clock_sampler_without_nvml_says_unavailable(monkeypatch):
    import importlib
    sys.path.insert(0, ROOT)
    monkeypatch.setitem(sys.modules, "pynvml", None)          # import fails
    bench = importlib.import_module("bench")
    with bench.ClockSampler(0) as clk:
        pass
    assert clk.summary() == {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unavailable"]}


def test_reference_arm_under_torchrun_prints_once_from_rank_0():
    """Launched like the driver's N>1 runs (torchrun, two ranks): rank 0 alone runs and prints; both exit 0."""
    import socket
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        port = s.getsockname()[1]
    res = subprocess.run([sys.executable, "-m", "torch.distributed.run", "--nnodes=1", "--nproc-per-node", "2",
                          "--master-addr", "127.0.0.1", "--master-port", str(port), "bench.py", "--impl", "reference",
                          "--gpus", "2", "--steps", "1", "--warmup", "3", "--cpu-rows", "16"],
                         cwd=ROOT, capture_output=True, text=True, timeout=600)
    assert res.returncode == 0, res.stderr[-2000:]
    lines = [l for l in res.stdout.splitlines() if l.startswith("{")]
    assert len(lines) == 1
    d = json.loads(lines[0])
    assert d["impl"] == "reference" and d["n_gpus"] == 2 and d["cpu_baseline"]["cores"] == (os.cpu_count() or 1)
