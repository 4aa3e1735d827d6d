"""Clock and throttle sampling during a timed region (NVML, read-only).

Reads SM clocks and clock-event reasons from a background thread; never
changes any GPU setting.
"""

from __future__ import annotations

import statistics
import threading
import time

_REASONS = {
    "gpu_idle": 0x1,
    "applications_clocks_setting": 0x2,
    "sw_power_cap": 0x4,
    "hw_slowdown": 0x8,
    "sync_boost": 0x10,
    "sw_thermal_slowdown": 0x20,
    "hw_thermal_slowdown": 0x40,
    "hw_power_brake_slowdown": 0x80,
    "display_clock_setting": 0x100,
}


class ClockSampler:
    def __init__(self, device_index: int, period_s: float = 0.005):
        self.device_index = device_index
        self.period_s = period_s
        self.samples: list[tuple[int, int]] = []
        self._stop = threading.Event()
        self._thread = None
        self.max_mhz = None
        self.error = None

    def __enter__(self):
        try:
            import pynvml

            pynvml.nvmlInit()
            self._nv = pynvml
            self._h = pynvml.nvmlDeviceGetHandleByIndex(self.device_index)
            self.max_mhz = pynvml.nvmlDeviceGetMaxClockInfo(self._h, pynvml.NVML_CLOCK_SM)
        except Exception as exc:  # pragma: no cover - depends on the box
            self.error = f"nvml unavailable: {exc}"
            return self
        self._thread = threading.Thread(target=self._run, daemon=True)
        self._thread.start()
        return self

    def _run(self):
        nv, h = self._nv, self._h
        while not self._stop.is_set():
            try:
                mhz = nv.nvmlDeviceGetClockInfo(h, nv.NVML_CLOCK_SM)
                reasons = nv.nvmlDeviceGetCurrentClocksEventReasons(h)
                self.samples.append((mhz, reasons))
            except Exception as exc:  # pragma: no cover
                self.error = str(exc)
                return
            time.sleep(self.period_s)

    def __exit__(self, *exc):
        self._stop.set()
        if self._thread is not None:
            self._thread.join(timeout=2)
        return False

    def summary(self) -> dict:
        if not self.samples:
            return {"sm_mhz": None, "sm_max_mhz": self.max_mhz, "reasons": [], "samples": 0,
                    "note": self.error or "no samples in the timed region"}
        mhz = [s[0] for s in self.samples]
        mask = 0
        for _, r in self.samples:
            mask |= r
        reasons = [name for name, bit in _REASONS.items() if mask & bit and name != "gpu_idle"]
        return {"sm_mhz": statistics.median(mhz), "sm_max_mhz": self.max_mhz, "reasons": reasons,
                "samples": len(mhz)}
