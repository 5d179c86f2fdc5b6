"""Samples SM clocks and throttle reasons with ``nvidia-smi`` while a timed region runs.

Read-only: this never changes any GPU setting. The sampler is a child process of ours and is
stopped by its own PID.
"""
from __future__ import annotations

import csv
import io
import os
import statistics
import subprocess
import tempfile
from typing import Optional

FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
          "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
          "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")
REASONS = ("hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap")


def _device_selector(device_index: int) -> Optional[str]:
    try:
        import torch
        u = str(torch.cuda.get_device_properties(device_index).uuid)
        return u if u.startswith("GPU-") else "GPU-" + u
    except Exception:
        return None


class ClockSampler:
    def __init__(self, device_index: int = 0, period_ms: int = 200):
        self.sel = _device_selector(device_index)
        self.period = period_ms
        self.proc = None
        self.path = None
        self.result = None

    def __enter__(self):
        fd, self.path = tempfile.mkstemp(prefix="hk_clocks_", suffix=".csv")
        os.close(fd)
        cmd = ["nvidia-smi", f"--query-gpu={FIELDS}", "--format=csv,noheader,nounits", f"-lms", str(self.period)]
        if self.sel:
            cmd += ["-i", self.sel]
        try:
            self.proc = subprocess.Popen(cmd, stdout=open(self.path, "w"), stderr=subprocess.DEVNULL)
        except FileNotFoundError:
            self.proc = None
            return self
        # nvidia-smi takes a while to start: wait for its first sample so that even a short timed
        # region is covered by at least one reading taken under load.
        import time
        t_end = time.time() + 5.0
        while time.time() < t_end and self.proc.poll() is None:
            if os.path.getsize(self.path) > 0:
                break
            time.sleep(0.01)
        return self

    def __exit__(self, *exc):
        if self.proc is not None:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()
        self.result = self.parse()
        try:
            os.unlink(self.path)
        except OSError:
            pass
        return False

    def parse(self) -> dict:
        if not self.path or not os.path.exists(self.path):
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unsampled"]}
        rows = list(csv.reader(io.StringIO(open(self.path).read())))
        sm, smax, power, reasons = [], None, [], set()
        for r in rows:
            if len(r) < 9:
                continue
            r = [c.strip() for c in r]
            try:
                sm.append(float(r[1]))
                smax = float(r[2])
                power.append(float(r[3]))
            except ValueError:
                continue
            for name, val in zip(REASONS, r[5:9]):
                if val.lower() == "active":
                    reasons.add(name)
        if not sm:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unsampled"]}
        return {"sm_mhz": statistics.median(sm), "sm_max_mhz": smax, "reasons": sorted(reasons),
                "samples": len(sm), "power_w_max": max(power) if power else None}
