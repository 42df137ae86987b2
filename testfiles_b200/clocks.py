"""SM clock and throttle-reason sampling during a timed region (NVML reads
only; no GPU setting is ever changed).

``with ClockSampler(device_index) as s: ...`` polls the SM clock and the
active clock-event reasons every 20 ms on a background thread;
``s.summary()`` gives the median SM clock over busy samples, the maximum SM
clock and every reason seen (idle excluded).  Without NVML the summary says
so (``sm_mhz: None``).
"""

from __future__ import annotations

import os
import statistics
import threading

REASON_BITS = {
    0x1: "gpu_idle", 0x2: "applications_clocks_setting", 0x4: "sw_power_cap", 0x8: "hw_slowdown",
    0x10: "sync_boost", 0x20: "sw_thermal_slowdown", 0x40: "hw_thermal_slowdown",
    0x80: "hw_power_brake_slowdown", 0x100: "display_clock_setting",
}


class ClockSampler:
    def __init__(self, device_index: int, period_s: float = 0.02):
        self.samples: list[tuple[int, int]] = []
        self.max_mhz = None
        self._stop = threading.Event()
        self._thread = None
        try:
            import pynvml

            pynvml.nvmlInit()
            visible = os.environ.get("CUDA_VISIBLE_DEVICES")
            index = int(visible.split(",")[device_index]) if visible else device_index
            self._nvml = pynvml
            self._handle = pynvml.nvmlDeviceGetHandleByIndex(index)
            self.max_mhz = pynvml.nvmlDeviceGetMaxClockInfo(self._handle, pynvml.NVML_CLOCK_SM)
        except Exception:  # noqa: BLE001 - clocks are reported as unavailable
            self._nvml = None
        self.period = period_s

    def _run(self):
        nv = self._nvml
        while not self._stop.is_set():
            try:
                mhz = nv.nvmlDeviceGetClockInfo(self._handle, nv.NVML_CLOCK_SM)
                reasons = nv.nvmlDeviceGetCurrentClocksEventReasons(self._handle)
                self.samples.append((mhz, reasons))
            except Exception:  # noqa: BLE001
                pass
            self._stop.wait(self.period)

    def __enter__(self):
        if self._nvml is not None:
            self._thread = threading.Thread(target=self._run, daemon=True)
            self._thread.start()
        return self

    def __exit__(self, *exc):
        self._stop.set()
        if self._thread is not None:
            self._thread.join()

    def summary(self) -> dict:
        if self._nvml is None or not self.samples:
            return {"sm_mhz": None, "sm_max_mhz": self.max_mhz, "reasons": [], "samples": 0}
        busy = [s for s in self.samples if not s[1] & 0x1] or self.samples
        reasons = 0
        for _, r in busy:
            reasons |= r
        return {
            "sm_mhz": statistics.median(m for m, _ in busy),
            "sm_max_mhz": self.max_mhz,
            "reasons": [name for bit, name in REASON_BITS.items() if reasons & bit and bit != 0x1],
            "samples": len(busy),
        }
