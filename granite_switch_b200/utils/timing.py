"""Device timing helpers and an nvidia-smi clock sampler for benchmark runs."""
from __future__ import annotations

import csv
import io
import os
import shutil
import statistics
import subprocess

import torch


class ClockSampler:
    """Samples SM clocks and throttle reasons with ``nvidia-smi -lms`` while active.

    Read-only: it queries the clocks and never changes a GPU setting.
    """

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, index: int = 0, period_ms: int = 200):
        self.index, self.period = index, period_ms
        self.proc = None

    def __enter__(self):
        if shutil.which("nvidia-smi") is None:
            return self
        self.proc = subprocess.Popen(
            ["nvidia-smi", f"--id={self.index}", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
             f"-lms", str(self.period)], stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        return self

    def __exit__(self, *exc):
        self.text = ""
        if self.proc is not None:
            self.proc.terminate()
            try:
                self.text, _ = self.proc.communicate(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()
                self.text, _ = self.proc.communicate()
        return False

    def summary(self) -> dict:
        rows = []
        for r in csv.reader(io.StringIO(getattr(self, "text", "") or "")):
            if len(r) < 9:
                continue
            try:
                rows.append([x.strip() for x in r])
            except Exception:
                continue
        if not rows:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unsampled"]}
        sm = [float(r[1]) for r in rows if r[1].replace(".", "").isdigit()]
        mx = [float(r[2]) for r in rows if r[2].replace(".", "").isdigit()]
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = set()
        for r in rows:
            for i, n in enumerate(names):
                if r[5 + i].lower().startswith("active"):
                    reasons.add(n)
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": max(mx) if mx else None,
                "reasons": sorted(reasons), "samples": len(rows)}


def max_over_ranks(value: float, group=None) -> float:
    if not torch.distributed.is_initialized():
        return value
    t = torch.tensor([value], dtype=torch.float64, device="cuda")
    torch.distributed.all_reduce(t, op=torch.distributed.ReduceOp.MAX, group=group)
    return float(t.item())


def local_rank() -> int:
    return int(os.environ.get("LOCAL_RANK", "0"))
