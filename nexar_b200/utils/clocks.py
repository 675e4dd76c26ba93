"""Sample GPU clocks and throttle reasons with nvidia-smi while a region runs.

Read-only: queries `nvidia-smi --query-gpu=...`; never changes any setting.
"""
from __future__ import annotations

import statistics
import subprocess
import threading
import time
from typing import List, Optional

_FIELDS = ("uuid,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.hw_slowdown,"
           "clocks_event_reasons.hw_thermal_slowdown,clocks_event_reasons.sw_thermal_slowdown,"
           "clocks_event_reasons.sw_power_cap")
_REASONS = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]


class ClockSampler:
    def __init__(self, uuids: Optional[List[str]] = None, period_ms: int = 200):
        self.uuids = set(u.lower() for u in uuids) if uuids else None
        self.period = period_ms / 1000.0
        self.samples = []  # (sm_mhz, max_mhz, power, [reasons])
        self._stop = threading.Event()
        self._thr = None
        self.available = True

    def _poll_once(self):
        try:
            out = subprocess.run(["nvidia-smi", f"--query-gpu={_FIELDS}", "--format=csv,noheader,nounits"],
                                 capture_output=True, text=True, timeout=5)
        except Exception:
            self.available = False
            return
        if out.returncode != 0:
            self.available = False
            return
        for line in out.stdout.strip().splitlines():
            parts = [p.strip() for p in line.split(",")]
            if len(parts) < 8:
                continue
            uuid = parts[0].lower()
            if self.uuids and not any(uuid.endswith(u.replace("gpu-", "")) or u in uuid for u in self.uuids):
                continue
            try:
                sm = float(parts[1])
                mx = float(parts[2])
                pw = float(parts[3]) if parts[3] not in ("[N/A]", "N/A") else float("nan")
            except ValueError:
                continue
            reasons = [r for r, v in zip(_REASONS, parts[4:8]) if v.lower() == "active"]
            self.samples.append((sm, mx, pw, reasons))

    def _run(self):
        while not self._stop.is_set():
            self._poll_once()
            if not self.available:
                return
            self._stop.wait(self.period)

    def __enter__(self):
        self._thr = threading.Thread(target=self._run, daemon=True)
        self._thr.start()
        return self

    def __exit__(self, *exc):
        self._stop.set()
        if self._thr is not None:
            self._thr.join(timeout=10)

    def summary(self) -> dict:
        if not self.samples:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": [], "samples": 0,
                    "note": "nvidia-smi unavailable" if not self.available else "no samples"}
        sms = [s[0] for s in self.samples]
        reasons = sorted({r for s in self.samples for r in s[3]})
        pw = [s[2] for s in self.samples if s[2] == s[2]]
        return {"sm_mhz": statistics.median(sms), "sm_max_mhz": max(s[1] for s in self.samples),
                "reasons": reasons, "samples": len(self.samples),
                "power_w_max": max(pw) if pw else None}


def device_uuids(devices) -> List[str]:
    import torch
    out = []
    for d in devices:
        try:
            u = str(torch.cuda.get_device_properties(d).uuid)
            out.append(u if u.startswith("GPU-") else "GPU-" + u)
        except Exception:
            pass
    return out
