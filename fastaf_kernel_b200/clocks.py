"""Sample SM clocks and throttle reasons with nvidia-smi during a timed region.

Read-only: it queries clocks and never changes any GPU setting.
"""

from __future__ import annotations

import csv
import io
import os
import shutil
import statistics
import subprocess
import tempfile
from typing import Optional

QUERY = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
         "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
         "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")
_REASONS = ("hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap")


def _device_selector(device_index: int) -> Optional[str]:
    try:
        import torch
        uuid = str(torch.cuda.get_device_properties(device_index).uuid)
        return uuid if uuid.startswith("GPU-") else "GPU-" + uuid
    except Exception:
        return None


class ClockSampler:
    """Context manager: ``with ClockSampler(dev) as cs: ...; cs.summary()``."""

    def __init__(self, device_index: int = 0, period_ms: int = 200):
        self.device_index = device_index
        self.period_ms = period_ms
        self.proc = None
        self.path = None
        self._summary = None

    def __enter__(self):
        exe = shutil.which("nvidia-smi")
        if exe is None:
            return self
        fd, self.path = tempfile.mkstemp(prefix="gdn_clocks_", suffix=".csv")
        os.close(fd)
        cmd = [exe, f"--query-gpu={QUERY}", "--format=csv,noheader,nounits",
               f"-lms={self.period_ms}"]
        sel = _device_selector(self.device_index)
        if sel:
            cmd.append(f"--id={sel}")
        self._fh = open(self.path, "w")
        self.proc = subprocess.Popen(cmd, stdout=self._fh, stderr=subprocess.DEVNULL)
        return self

    def __exit__(self, *exc):
        if self.proc is not None:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()
            self._fh.close()
            self._summary = self._parse()
            try:
                os.unlink(self.path)
            except OSError:
                pass
        return False

    def _parse(self):
        rows = []
        with open(self.path) as f:
            for r in csv.reader(io.StringIO(f.read())):
                if len(r) < 9:
                    continue
                try:
                    rows.append([x.strip() for x in r])
                except ValueError:
                    continue
        if not rows:
            return None
        sm = [float(r[1]) for r in rows if r[1].replace(".", "").isdigit()]
        mx = [float(r[2]) for r in rows if r[2].replace(".", "").isdigit()]
        reasons = set()
        for r in rows:
            for name, val in zip(_REASONS, r[5:9]):
                if val.lower() == "active":
                    reasons.add(name)
        return {"sm_mhz": statistics.median(sm) if sm else None,
                "sm_max_mhz": max(mx) if mx else None,
                "reasons": sorted(reasons), "samples": len(rows)}

    def summary(self):
        return self._summary or {"sm_mhz": None, "sm_max_mhz": None, "reasons": [],
                                 "samples": 0, "note": "nvidia-smi unavailable"}
