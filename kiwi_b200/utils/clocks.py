"""GPU clock / throttle sampling during a timed region (nvidia-smi, read only)."""
import os
import shutil
import statistics
import subprocess
import tempfile

REASONS = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
QUERY = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.hw_slowdown,"
         "clocks_event_reasons.hw_thermal_slowdown,clocks_event_reasons.sw_thermal_slowdown,"
         "clocks_event_reasons.sw_power_cap")


class ClockSampler:
    """Samples SM clock and throttle reasons every `period_ms` while active.
    ``summary()`` gives the median SM MHz under load, the max clock and the
    reasons seen active (never changes any GPU setting)."""

    def __init__(self, device_index=0, period_ms=200):
        self.device_index = device_index
        self.period_ms = period_ms
        self.proc = None
        self.path = None

    def __enter__(self):
        if shutil.which("nvidia-smi") is None:
            return self
        fd, self.path = tempfile.mkstemp(prefix="kiwi_clocks_", suffix=".csv")
        os.close(fd)
        self._f = open(self.path, "w")
        self.proc = subprocess.Popen(
            ["nvidia-smi", f"--query-gpu={QUERY}", "--format=csv,noheader,nounits", "-i", str(self.device_index),
             "-lms", str(self.period_ms)], stdout=self._f, stderr=subprocess.DEVNULL)
        return self

    def __exit__(self, *exc):
        if self.proc is not None:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()
            self._f.close()
        return False

    def summary(self):
        if not self.path or not os.path.exists(self.path):
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": [], "samples": 0}
        sm, mx, seen = [], [], set()
        with open(self.path) as f:
            for line in f:
                p = [s.strip() for s in line.split(",")]
                if len(p) < 8:
                    continue
                try:
                    sm.append(float(p[1]))
                    mx.append(float(p[2]))
                except ValueError:
                    continue
                for name, v in zip(REASONS, p[4:8]):
                    if v.lower() == "active":
                        seen.add(name)
        os.unlink(self.path)
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": max(mx) if mx else None,
                "reasons": sorted(seen), "samples": len(sm)}
