"""bench.py on CPU: the reference arm (the CPU oracle on the host's cores) prints the contract
line, and the clock sampler reads NVML (a read-only stand-in here) or nvidia-smi lines and
sets nothing."""
import json
import os
import subprocess
import sys

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def test_reference_arm_prints_one_json_line():
    r = subprocess.run([sys.executable, os.path.join(ROOT, "bench.py"), "--impl", "reference",
                        "--steps", "1", "--warmup", "0"], capture_output=True, text=True,
                       timeout=600, cwd=ROOT)
    assert r.returncode == 0, r.stderr[-2000:]
    lines = [ln for ln in r.stdout.splitlines() if ln.startswith("{")]
    assert len(lines) == 1
    d = json.loads(lines[0])
    assert d["impl"] == "reference" and d["unit"] == "tokens/s" and d["value"] > 0
    assert d["cpu_baseline"]["kind"] == "port" and d["cpu_baseline"]["cores"] >= 1
    assert d["e2e"]["h2d_bytes_per_step"] == 0


class _FakeNVML:
    """Read-only NVML stand-in: records every NVML function bench.py calls."""
    NVML_CLOCK_SM = 1
    nvmlClocksEventReasonHwSlowdown = 1 << 3
    nvmlClocksEventReasonHwThermalSlowdown = 1 << 6
    nvmlClocksEventReasonSwThermalSlowdown = 1 << 5
    nvmlClocksEventReasonSwPowerCap = 1 << 2

    def __init__(self, clocks, reasons):
        self.clocks, self.reasons, self.n, self.used = clocks, reasons, 0, []

    def __getattribute__(self, name):
        if name.startswith("nvml") and not name.startswith("nvmlClocksEventReason"):
            object.__getattribute__(self, "used").append(name)
        return object.__getattribute__(self, name)

    def nvmlInit(self):
        pass

    def nvmlShutdown(self):
        pass

    def nvmlDeviceGetHandleByPciBusId(self, bus):
        return "gpu"

    def nvmlDeviceGetHandleByIndex(self, index):
        return "gpu"

    def nvmlDeviceGetMaxClockInfo(self, handle, kind):
        return 1965

    def nvmlDeviceGetClockInfo(self, handle, kind):
        self.n += 1
        return self.clocks[self.n % len(self.clocks)]

    def nvmlDeviceGetCurrentClocksEventReasons(self, handle):
        return self.reasons


def test_clock_sampler_only_reads_nvml(monkeypatch):
    import time
    sys.path.insert(0, ROOT)
    import bench
    fake = _FakeNVML([1600.0, 1635.0, 1700.0], _FakeNVML.nvmlClocksEventReasonSwPowerCap)
    monkeypatch.setitem(sys.modules, "pynvml", fake)
    with bench.ClockSampler(0) as c:
        time.sleep(0.1)
    s = c.summary()
    assert s["source"] == "nvml" and s["samples"] >= 2, s
    assert s["sm_mhz"] in (1600.0, 1635.0, 1700.0) and s["sm_max_mhz"] == 1965.0
    assert s["reasons"] == ["sw_power_cap"]
    reads = {"nvmlInit", "nvmlShutdown", "nvmlDeviceGetHandleByPciBusId",
             "nvmlDeviceGetHandleByIndex", "nvmlDeviceGetMaxClockInfo", "nvmlDeviceGetClockInfo",
             "nvmlDeviceGetCurrentClocksEventReasons"}
    assert set(fake.used) <= reads, set(fake.used) - reads


def test_clock_summary_parses_nvidia_smi_lines():
    sys.path.insert(0, ROOT)
    import bench
    c = bench.ClockSampler(0)
    c.lines = ["0, 1635, 1965, 951.20, 0x0000000000000004, Not Active, Not Active, Not Active, Active",
               "0, 1650, 1965, 960.00, 0x0000000000000000, Not Active, Not Active, Not Active, Not Active",
               "garbage"]
    s = c.summary()
    assert s == {"sm_mhz": 1642.5, "sm_max_mhz": 1965.0, "reasons": ["sw_power_cap"],
                 "samples": 2, "source": "nvidia-smi"}
