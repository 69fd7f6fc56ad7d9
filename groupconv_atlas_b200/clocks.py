"""Read-only sampling of the GPU's SM clock, power and clock-event reasons
through NVML while a timed region runs (the record that says whether a
measurement was throttled).  Nothing here changes a GPU setting."""
from __future__ import annotations

import os
import statistics
import threading
import time


class ClockSampler:
    """Samples SM clock, power and clock-event reasons through NVML (read only)."""
    REASONS = {
        'hw_slowdown': 'nvmlClocksEventReasonHwSlowdown',
        'hw_thermal_slowdown': 'nvmlClocksEventReasonHwThermalSlowdown',
        'sw_thermal_slowdown': 'nvmlClocksEventReasonSwThermalSlowdown',
        'sw_power_cap': 'nvmlClocksEventReasonSwPowerCap',
        'hw_power_brake_slowdown': 'nvmlClocksEventReasonHwPowerBrakeSlowdown',
    }

    def __init__(self, device_index, period=0.005):
        self.period = period
        self.samples = []
        self._stop = threading.Event()
        self._thread = None
        try:
            import pynvml
            pynvml.nvmlInit()
            self.nvml = pynvml
            # NVML enumerates physical GPUs; map through CUDA_VISIBLE_DEVICES if set.
            visible = os.environ.get('CUDA_VISIBLE_DEVICES')
            index = device_index
            if visible:
                ids = [v.strip() for v in visible.split(',') if v.strip()]
                if device_index < len(ids) and ids[device_index].isdigit():
                    index = int(ids[device_index])
            self.handle = pynvml.nvmlDeviceGetHandleByIndex(index)
            self.max_mhz = pynvml.nvmlDeviceGetMaxClockInfo(self.handle, pynvml.NVML_CLOCK_SM)
        except Exception as exc:  # no NVML: report why instead of clocks
            self.nvml = None
            self.error = str(exc)

    def _run(self):
        n = self.nvml
        while not self._stop.is_set():
            try:
                sm = n.nvmlDeviceGetClockInfo(self.handle, n.NVML_CLOCK_SM)
                reasons = n.nvmlDeviceGetCurrentClocksEventReasons(self.handle)
                power = n.nvmlDeviceGetPowerUsage(self.handle) / 1000.0
                self.samples.append((sm, reasons, power))
            except Exception:
                pass
            time.sleep(self.period)

    def __enter__(self):
        if self.nvml is not None:
            self._thread = threading.Thread(target=self._run, daemon=True)
            self._thread.start()
        return self

    def __exit__(self, *exc):
        self._stop.set()
        if self._thread is not None:
            self._thread.join()

    def summary(self):
        if self.nvml is None:
            return {'sm_mhz': None, 'sm_max_mhz': None, 'reasons': [], 'error': self.error}
        if not self.samples:
            return {'sm_mhz': None, 'sm_max_mhz': self.max_mhz, 'reasons': [], 'samples': 0}
        active = set()
        for _, mask, _ in self.samples:
            for name, const in self.REASONS.items():
                if mask & getattr(self.nvml, const):
                    active.add(name)
        return {'sm_mhz': statistics.median(s[0] for s in self.samples), 'sm_max_mhz': self.max_mhz,
                'reasons': sorted(active), 'samples': len(self.samples),
                'power_w_max': max(s[2] for s in self.samples)}
