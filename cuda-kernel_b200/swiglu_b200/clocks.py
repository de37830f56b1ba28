"""Read-only GPU clock sampling during a timed region (NVML, else nvidia-smi).

Samples SM clock, max SM clock, power and the active clock-event (throttle)
reasons every ``interval_s`` on a background thread. Nothing is ever set.
"""
from __future__ import annotations

import statistics
import subprocess
import threading
import time

# nvmlClocksEventReason* bit values (nvml.h)
_REASONS = {
    0x1: "gpu_idle", 0x2: "applications_clocks_setting", 0x4: "sw_power_cap", 0x8: "hw_slowdown",
    0x10: "sync_boost", 0x20: "sw_thermal_slowdown", 0x40: "hw_thermal_slowdown",
    0x80: "hw_power_brake_slowdown", 0x100: "display_clock_setting",
}
REJECT = {"hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown"}


class ClockSampler:
    def __init__(self, device_index: int = 0, interval_s: float = 0.01):
        self.index = device_index
        self.interval = interval_s
        self.samples: list[dict] = []
        self._stop = threading.Event()
        self._thread = None
        self._nvml = None
        self._handle = None
        try:
            import pynvml
            pynvml.nvmlInit()
            self._nvml = pynvml
            self._handle = pynvml.nvmlDeviceGetHandleByIndex(self._physical_index(device_index))
        except Exception:
            self._nvml = None

    @staticmethod
    def _physical_index(i: int) -> int:
        import os
        vis = os.environ.get("CUDA_VISIBLE_DEVICES")
        if vis:
            parts = [p.strip() for p in vis.split(",") if p.strip()]
            if i < len(parts) and parts[i].isdigit():
                return int(parts[i])
        return i

    def _sample_nvml(self) -> dict:
        n, h = self._nvml, self._handle
        sm = n.nvmlDeviceGetClockInfo(h, n.NVML_CLOCK_SM)
        try:
            mask = n.nvmlDeviceGetCurrentClocksEventReasons(h)
        except AttributeError:
            mask = n.nvmlDeviceGetCurrentClocksThrottleReasons(h)
        try:
            power = n.nvmlDeviceGetPowerUsage(h) / 1000.0
        except Exception:
            power = None
        return {"t": time.time(), "sm_mhz": sm, "mask": int(mask), "power_w": power}

    def _run(self):
        while not self._stop.is_set():
            try:
                self.samples.append(self._sample_nvml())
            except Exception:
                pass
            self._stop.wait(self.interval)

    def start(self):
        if self._nvml is not None:
            self._thread = threading.Thread(target=self._run, daemon=True)
            self._thread.start()
        return self

    def stop(self, window: tuple[float, float] | None = None,
             fallback_window: tuple[float, float] | None = None) -> dict:
        """Stop sampling; summarise the samples inside `window` (host times bracketing the
        timed region). When it caught fewer than three, add those of `fallback_window`
        (an untimed soak of the same work right after it)."""
        if self._thread is not None:
            self._stop.set()
            self._thread.join(timeout=5)
        if window is not None and self._nvml is not None:
            inside = [s for s in self.samples if window[0] <= s["t"] <= window[1]]
            if len(inside) >= 3 or fallback_window is None:
                out = self.summary(inside or self.samples)
                out["window"] = "timed region" if inside else "whole run"
                return out
            soak = [s for s in self.samples if fallback_window[0] <= s["t"] <= fallback_window[1]]
            out = self.summary(inside + soak)
            out["window"] = f"timed region ({len(inside)} samples) + untimed soak of the same graphs ({len(soak)})"
            return out
        return self.summary()

    def max_mhz(self):
        if self._nvml is None:
            return None
        try:
            return self._nvml.nvmlDeviceGetMaxClockInfo(self._handle, self._nvml.NVML_CLOCK_SM)
        except Exception:
            return None

    def summary(self, samples: list[dict] | None = None) -> dict:
        if self._nvml is None:
            return _smi_snapshot(self.index)
        samples = self.samples if samples is None else samples
        loaded = [s for s in samples if not (s["mask"] & 0x1)] or samples
        reasons = sorted({name for s in loaded for bit, name in _REASONS.items() if s["mask"] & bit} - {"gpu_idle"})
        return {
            "sm_mhz": statistics.median(s["sm_mhz"] for s in loaded) if loaded else None,
            "sm_max_mhz": self.max_mhz(),
            "reasons": reasons,
            "samples": len(samples),
            "samples_under_load": len(loaded),
            "power_w_max": max((s["power_w"] for s in loaded if s["power_w"] is not None), default=None),
            "source": "nvml",
            "rejected": bool(set(reasons) & REJECT),
        }


def _smi_snapshot(index: int) -> dict:
    try:
        out = subprocess.run(
            ["nvidia-smi", f"--id={index}", "--query-gpu=clocks.sm,clocks.max.sm,clocks_event_reasons.active",
             "--format=csv,noheader,nounits"], capture_output=True, text=True, timeout=20).stdout.strip()
        sm, smax, mask = [v.strip() for v in out.split(",")]
        m = int(mask, 16)
        reasons = sorted(name for bit, name in _REASONS.items() if m & bit and name != "gpu_idle")
        return {"sm_mhz": float(sm), "sm_max_mhz": float(smax), "reasons": reasons, "samples": 1,
                "source": "nvidia-smi", "rejected": bool(set(reasons) & REJECT)}
    except Exception as exc:  # no GPU tools: report absence, never invent clocks
        return {"sm_mhz": None, "sm_max_mhz": None, "reasons": [], "samples": 0, "source": f"unavailable: {exc}"}
