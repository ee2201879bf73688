"""Sample GPU clocks and throttle reasons with nvidia-smi during a timed region."""
from __future__ import annotations

import statistics
import subprocess
import tempfile

FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
          "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
          "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")
REASON_COLS = {5: "hw_slowdown", 6: "hw_thermal_slowdown", 7: "sw_thermal_slowdown",
               8: "sw_power_cap"}


class ClockSampler:
    """Runs `nvidia-smi -lms` in the background; `stop()` returns the summary dict."""

    def __init__(self, gpus: list[int], period_ms: int = 100):
        self.gpus = gpus
        self.period_ms = period_ms
        self.proc = None
        self.out = None

    def start(self) -> "ClockSampler":
        self.out = tempfile.TemporaryFile(mode="w+")
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", "-i", ",".join(map(str, self.gpus)), f"--query-gpu={FIELDS}",
                 "--format=csv,noheader,nounits", "-lms", str(self.period_ms)],
                stdout=self.out, stderr=subprocess.DEVNULL)
        except OSError:
            self.proc = None
        return self

    def stop(self) -> dict:
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": [], "samples": 0,
                    "note": "nvidia-smi unavailable"}
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
        self.out.seek(0)
        return summarize(self.out.read())


def summarize(text: str) -> dict:
    sm, sm_max, power, reasons = [], [], [], set()
    n = 0
    for line in text.splitlines():
        cols = [c.strip() for c in line.split(",")]
        if len(cols) < 9:
            continue
        try:
            sm.append(float(cols[1]))
            sm_max.append(float(cols[2]))
            power.append(float(cols[3]))
        except ValueError:
            continue
        n += 1
        for i, name in REASON_COLS.items():
            if cols[i].lower().startswith("active"):
                reasons.add(name)
    if not sm:
        return {"sm_mhz": None, "sm_max_mhz": None, "reasons": sorted(reasons), "samples": 0}
    # "Under load": samples drawing at least half the peak power seen.
    pmax = max(power) if power else 0
    loaded = [s for s, p in zip(sm, power) if p >= 0.5 * pmax] or sm
    return {"sm_mhz": statistics.median(loaded), "sm_max_mhz": max(sm_max),
            "reasons": sorted(reasons), "samples": n, "power_w_max": pmax}
