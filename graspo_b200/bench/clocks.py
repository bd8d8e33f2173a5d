"""Sample GPU clocks and throttle reasons while a measurement runs.

Runs ``nvidia-smi --query-gpu=... -lms 200`` in the background and reports
the median SM clock under load, the maximum SM clock and every clock-event
reason seen active.  Reading clocks changes nothing on the GPU.
"""

from __future__ import annotations

import subprocess
import threading

FIELDS = ("index", "clocks.sm", "clocks.max.sm", "power.draw", "utilization.gpu",
          "clocks_event_reasons.hw_slowdown", "clocks_event_reasons.hw_thermal_slowdown",
          "clocks_event_reasons.sw_thermal_slowdown", "clocks_event_reasons.sw_power_cap")
REASONS = ("hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap")


class ClockSampler:
    def __init__(self, gpu_index: int | None = None, period_ms: int = 200) -> None:
        self.gpu_index = gpu_index
        self.period_ms = period_ms
        self.rows: list[list[str]] = []
        self._proc = None
        self._thread = None

    def __enter__(self) -> "ClockSampler":
        cmd = ["nvidia-smi", f"--query-gpu={','.join(FIELDS)}", "--format=csv,noheader,nounits",
               f"-lms={self.period_ms}"]
        if self.gpu_index is not None:
            cmd.insert(1, f"--id={self.gpu_index}")
        try:
            self._proc = subprocess.Popen(cmd, stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except OSError:
            self._proc = None
            return self
        self._thread = threading.Thread(target=self._read, daemon=True)
        self._thread.start()
        return self

    def _read(self) -> None:
        for line in self._proc.stdout:
            parts = [p.strip() for p in line.split(",")]
            if len(parts) == len(FIELDS):
                self.rows.append(parts)

    def __exit__(self, *exc) -> None:
        if self._proc is not None:
            self._proc.terminate()
            try:
                self._proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self._proc.kill()
        if self._thread is not None:
            self._thread.join(timeout=5)

    def summary(self) -> dict:
        if not self.rows:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": [], "samples": 0}

        def num(x):
            try:
                return float(x)
            except ValueError:
                return None

        loaded = [r for r in self.rows if (num(r[4]) or 0) >= 50] or self.rows
        clocks = sorted(v for v in (num(r[1]) for r in loaded) if v is not None)
        reasons = sorted({REASONS[i] for r in self.rows for i, f in enumerate(r[5:9]) if "Active" in f and "Not" not in f})
        return {
            "sm_mhz": clocks[len(clocks) // 2] if clocks else None,
            "sm_max_mhz": max((num(r[2]) or 0) for r in self.rows),
            "reasons": reasons,
            "samples": len(self.rows),
            "samples_under_load": len(loaded),
            "power_w_max": max((num(r[3]) or 0) for r in self.rows),
        }
