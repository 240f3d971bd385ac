"""bench.py on the host: the reference arm's JSON line carries the bench
contract's keys (under torchrun only rank 0 prints), and the clock sampler maps
NVML's clock-event reasons to the names the line reports."""

import json
import os
import subprocess
import sys

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _run(extra_env=None, *args):
    env = dict(os.environ)
    env.update(extra_env or {})
    return subprocess.run([sys.executable, os.path.join(ROOT, "bench.py"), "--impl", "reference", *args],
                          cwd=ROOT, env=env, capture_output=True, text=True, timeout=300)


def test_reference_arm_prints_one_contract_line():
    r = _run(None, "--steps", "2", "--warmup", "1")
    assert r.returncode == 0, r.stderr
    lines = [ln for ln in r.stdout.splitlines() if ln.strip()]
    assert len(lines) == 1
    j = json.loads(lines[0])
    for key in ("metric", "value", "unit", "n_gpus", "steps", "warmup", "ms_per_step", "higher_is_better",
                "scaling", "vs_baseline", "dtype", "data", "config", "cpu_baseline", "e2e"):
        assert key in j, key
    assert j["impl"] == "reference" and j["value"] > 0 and j["higher_is_better"] is True
    assert j["steps"] == 2 and j["warmup"] == 3           # warm-up is raised to the contract's minimum
    assert j["config"]["workload"].startswith("chunk_ttt_write_isolated")
    cb = j["cpu_baseline"]
    assert cb["kind"] in ("reference", "port") and cb["cores"] >= 1 and cb["value"] == j["value"] and cb["sample"]
    assert j["e2e"] == {"value": j["value"], "unit": j["unit"], "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}


def test_reference_arm_other_ranks_exit_quietly():
    r = _run({"RANK": "1", "LOCAL_RANK": "1", "WORLD_SIZE": "2"}, "--steps", "1")
    assert r.returncode == 0, r.stderr
    assert r.stdout.strip() == ""


def test_clock_sampler_reads_nvml_reasons(monkeypatch):
    """The sampler maps NVML clock-event reason bits to the contract's names (a fake NVML here)."""
    import types
    sys.path.insert(0, ROOT)
    import bench

    clocks = iter([1800.0, 1790.0, 1810.0] + [1800.0] * 1000)
    fake = types.ModuleType("pynvml")
    fake.NVML_CLOCK_SM = 1
    fake.nvmlInit = lambda: None
    fake.nvmlShutdown = lambda: None
    fake.nvmlDeviceGetHandleByPciBusId = lambda bus: (_ for _ in ()).throw(RuntimeError("no bus id"))
    fake.nvmlDeviceGetHandleByIndex = lambda i: ("gpu", i)
    fake.nvmlDeviceGetMaxClockInfo = lambda h, c: 1965
    fake.nvmlDeviceGetClockInfo = lambda h, c: next(clocks)
    fake.nvmlDeviceGetCurrentClocksEventReasons = lambda h: 0x4 | 0x1   # sw_power_cap + GPU idle
    monkeypatch.setitem(sys.modules, "pynvml", fake)
    s = bench.ClockSampler(0)
    s.start()
    out = s.stop()
    assert out["sm_max_mhz"] == 1965.0 and out["samples"] >= 2 and 1790.0 <= out["sm_mhz"] <= 1810.0
    assert out["reasons"] == ["sw_power_cap"] and out["source"].startswith("NVML")
