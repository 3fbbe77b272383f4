"""Read-only GPU clock / throttle-reason sampling during a timed region (NVML).

Only queries are issued; no clock, power or mode setting is ever changed.
"""
from __future__ import annotations

import statistics
import threading
import time

REASON_BITS = {
    0x1: "gpu_idle",
    0x2: "applications_clocks_setting",
    0x4: "sw_power_cap",
    0x8: "hw_slowdown",
    0x10: "sync_boost",
    0x20: "sw_thermal_slowdown",
    0x40: "hw_thermal_slowdown",
    0x80: "hw_power_brake_slowdown",
    0x100: "display_clock_setting",
}
BAD_REASONS = {"hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown"}


def decode_reasons(mask: int) -> list[str]:
    return [name for bit, name in REASON_BITS.items() if mask & bit]


class ClockSampler:
    """Samples SM clock and throttle reasons of one GPU every `period` seconds."""

    def __init__(self, device_index: int, period: float = 0.2):
        self.index = device_index
        self.period = period
        self.samples: list[tuple[int, int]] = []
        self.max_mhz = None
        self._stop = threading.Event()
        self._thread = None
        self._nvml = None
        try:
            import pynvml

            pynvml.nvmlInit()
            self._nvml = pynvml
            self._h = pynvml.nvmlDeviceGetHandleByIndex(device_index)
            self.max_mhz = pynvml.nvmlDeviceGetMaxClockInfo(self._h, pynvml.NVML_CLOCK_SM)
        except Exception:  # no NVML (CPU box): sampling is a no-op
            self._nvml = None

    def _sample(self):
        nv = self._nvml
        try:
            mhz = nv.nvmlDeviceGetClockInfo(self._h, nv.NVML_CLOCK_SM)
            try:
                mask = nv.nvmlDeviceGetCurrentClocksEventReasons(self._h)
            except AttributeError:
                mask = nv.nvmlDeviceGetCurrentClocksThrottleReasons(self._h)
            self.samples.append((int(mhz), int(mask)))
        except Exception:
            pass

    def _run(self):
        while not self._stop.is_set():
            self._sample()
            time.sleep(self.period)

    def __enter__(self):
        if self._nvml is not None:
            self._sample()
            self._thread = threading.Thread(target=self._run, daemon=True)
            self._thread.start()
        return self

    def __exit__(self, *exc):
        self._stop.set()
        if self._thread is not None:
            self._thread.join(timeout=2)
        if self._nvml is not None:
            self._sample()

    def summary(self) -> dict:
        if not self.samples:
            return {"sm_mhz": None, "sm_max_mhz": self.max_mhz, "reasons": [], "samples": 0}
        mhz = [m for m, _ in self.samples]
        mask = 0
        for _, r in self.samples:
            mask |= r
        reasons = [r for r in decode_reasons(mask) if r != "gpu_idle"]
        return {"sm_mhz": statistics.median(mhz), "sm_max_mhz": self.max_mhz, "reasons": reasons,
                "samples": len(self.samples)}
