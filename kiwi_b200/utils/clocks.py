"""GPU clock / throttle sampling during a timed region (nvidia-smi, read only).

A reader thread timestamps every nvidia-smi sample on arrival; ``mark_start`` /
``mark_end`` bracket the timed region and ``summary()`` reports the samples
inside it (or, if the region was shorter than the sampling period, the samples
nearest to it)."""
import shutil
import statistics
import subprocess
import threading
import time

REASONS = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
QUERY = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.hw_slowdown,"
         "clocks_event_reasons.hw_thermal_slowdown,clocks_event_reasons.sw_thermal_slowdown,"
         "clocks_event_reasons.sw_power_cap")


class ClockSampler:
    """Samples SM clocks, power and throttle reasons with nvidia-smi (read
    only) in a background process while the ``with`` block runs; ``summary()``
    reports the samples between ``mark_start()`` and ``mark_end()``."""
    def __init__(self, device_index=0, period_ms=50):
        self.device_index = device_index
        self.period_ms = period_ms
        self.proc = None
        self.samples = []   # (arrival time, sm, max, power, reasons)
        self.t0 = self.t1 = None

    def __enter__(self):
        if shutil.which("nvidia-smi") is None:
            return self
        self.proc = subprocess.Popen(
            ["nvidia-smi", f"--query-gpu={QUERY}", "--format=csv,noheader,nounits", "-i", str(self.device_index),
             "-lms", str(self.period_ms)], stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        self.thread = threading.Thread(target=self._read, daemon=True)
        self.thread.start()
        return self

    def _read(self):
        for line in self.proc.stdout:
            p = [s.strip() for s in line.split(",")]
            if len(p) < 8:
                continue
            try:
                sm, mx = float(p[1]), float(p[2])
                pw = float(p[3]) if p[3] not in ("[N/A]", "N/A") else None
            except ValueError:
                continue
            reasons = {n for n, v in zip(REASONS, p[4:8]) if v.lower() == "active"}
            self.samples.append((time.time(), sm, mx, pw, reasons))

    def wait_first_sample(self, timeout_s=5.0):
        end = time.time() + timeout_s
        while self.proc is not None and not self.samples and time.time() < end:
            time.sleep(0.01)

    def mark_start(self):
        self.t0 = time.time()

    def mark_end(self):
        self.t1 = time.time()

    def __exit__(self, *exc):
        if self.proc is not None:
            time.sleep(2 * self.period_ms / 1000)
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()
            self.thread.join(timeout=2)
        return False

    def summary(self):
        if not self.samples:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": [], "samples": 0}
        t0 = self.t0 if self.t0 is not None else self.samples[0][0]
        t1 = self.t1 if self.t1 is not None else self.samples[-1][0]
        inside = [s for s in self.samples if t0 <= s[0] <= t1 + self.period_ms / 1000]
        if not inside:  # region shorter than the period: nearest samples after the start
            inside = sorted(self.samples, key=lambda s: abs(s[0] - t0))[:2]
        seen = set().union(*(s[4] for s in inside))
        return {"sm_mhz": statistics.median(s[1] for s in inside), "sm_max_mhz": max(s[2] for s in inside),
                "reasons": sorted(seen), "samples": len(inside),
                "power_w_max": max((s[3] for s in inside if s[3] is not None), default=None)}
