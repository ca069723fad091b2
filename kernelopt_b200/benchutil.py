"""Measurement helpers shared by bench.py: clock sampling through NVML (read-only), CUDA-event timing of
individual kernel launches, launch counting and GPU peak figures."""
from __future__ import annotations

import json
import statistics
import threading
import time
from pathlib import Path

import torch

ROOT = Path(__file__).resolve().parent.parent

# Throttle reasons that invalidate a measurement, and the benign power cap (NVML bit masks).
_REASONS = {0x1: "gpu_idle", 0x2: "applications_clocks_setting", 0x4: "sw_power_cap", 0x8: "hw_slowdown",
            0x20: "sw_thermal_slowdown", 0x40: "hw_thermal_slowdown", 0x80: "hw_power_brake_slowdown",
            0x100: "display_clock_setting"}


class ClockSampler:
    """Samples SM clock, power and clock-event reasons of one GPU every `period` s in a thread (NVML reads only)."""

    def __init__(self, device: torch.device, period: float = 0.1):
        self.period = period
        self.samples: list[tuple[float, float, int]] = []
        self._stop = threading.Event()
        self._thread = None
        self.handle = None
        self.max_mhz = None
        try:
            import pynvml
            pynvml.nvmlInit()
            bus = getattr(torch.cuda.get_device_properties(device), "pci_bus_id", None)
            if bus is not None:
                dom = getattr(torch.cuda.get_device_properties(device), "pci_domain_id", 0)
                dev_id = getattr(torch.cuda.get_device_properties(device), "pci_device_id", 0)
                self.handle = pynvml.nvmlDeviceGetHandleByPciBusId(f"{dom:08x}:{bus:02x}:{dev_id:02x}.0")
            else:
                self.handle = pynvml.nvmlDeviceGetHandleByIndex(device.index or 0)
            self.max_mhz = pynvml.nvmlDeviceGetMaxClockInfo(self.handle, pynvml.NVML_CLOCK_SM)
            self._nvml = pynvml
        except Exception:  # no NVML: clocks are reported as unavailable
            self.handle = None

    def _run(self):
        nv = self._nvml
        while not self._stop.is_set():
            try:
                sm = nv.nvmlDeviceGetClockInfo(self.handle, nv.NVML_CLOCK_SM)
                pw = nv.nvmlDeviceGetPowerUsage(self.handle) / 1000.0
                rs = nv.nvmlDeviceGetCurrentClocksEventReasons(self.handle)
                self.samples.append((float(sm), pw, int(rs)))
            except Exception:
                pass
            self._stop.wait(self.period)

    def __enter__(self):
        if self.handle is not None:
            self._thread = threading.Thread(target=self._run, daemon=True)
            self._thread.start()
        return self

    def __exit__(self, *exc):
        self._stop.set()
        if self._thread:
            self._thread.join()

    def summary(self) -> dict:
        if not self.samples:
            return {"sm_mhz": None, "sm_max_mhz": self.max_mhz, "reasons": ["unavailable (no NVML samples)"]}
        mask = 0
        for _, _, r in self.samples:
            mask |= r
        reasons = [name for bit, name in _REASONS.items() if mask & bit and name != "gpu_idle"]
        return {"sm_mhz": statistics.median(s[0] for s in self.samples), "sm_max_mhz": self.max_mhz,
                "power_w_max": max(s[1] for s in self.samples), "samples": len(self.samples), "reasons": reasons}


def measured_peaks() -> dict:
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        return {"hbm_gbs": d["hbm_gbs"], "bf16_tflops": d["bf16_tflops"],
                "bf16_tflops_sustained": d.get("bf16_tflops_sustained", d["bf16_tflops"]), "source": "measured"}
    return {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0, "source": "fallback"}


class EventTimer:
    """Accumulates CUDA-event durations of wrapped calls, on the stream each call is launched on."""

    def __init__(self):
        self.pairs: list[tuple[torch.cuda.Event, torch.cuda.Event, float]] = []

    def wrap(self, fn, work_of):
        def timed(*args, **kw):
            s = torch.cuda.current_stream()
            e0 = torch.cuda.Event(enable_timing=True)
            e1 = torch.cuda.Event(enable_timing=True)
            e0.record(s)
            out = fn(*args, **kw)
            e1.record(s)
            self.pairs.append((e0, e1, work_of(*args, **kw)))
            return out
        return timed

    def total(self) -> tuple[float, float, int]:
        """(seconds, work units, launches) after synchronisation."""
        torch.cuda.synchronize()
        secs = sum(a.elapsed_time(b) for a, b, _ in self.pairs) / 1e3
        return secs, sum(w for _, _, w in self.pairs), len(self.pairs)


def hold_stream(seconds: float = 0.05, stream=None) -> None:
    """Keeps `stream` busy for about `seconds` with a spin kernel, so that the host enqueues the launches that
    follow before the GPU reaches them: CUDA events around each of those launches then time the GPU's work
    alone, not the host's Python and launch overhead that would otherwise sit between the two events."""
    s = stream or torch.cuda.current_stream()
    with torch.cuda.stream(s):
        torch.cuda._sleep(int(seconds * 2.0e9))  # cycles; B200 SM clocks run at about 2 GHz or below


class Stopwatch:
    def __enter__(self):
        self.t0 = time.perf_counter()
        return self

    def __exit__(self, *exc):
        self.s = time.perf_counter() - self.t0
