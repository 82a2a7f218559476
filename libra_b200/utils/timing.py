"""Device timing and clock sampling helpers.

* ``DeviceTimer``: CUDA-event timing on the launching stream with a
  synchronize on both sides; ``max_over_ranks`` reduces a duration with MAX so
  multi-GPU numbers are the slowest rank's.
* ``ClockSampler``: samples ``nvidia-smi`` SM clocks, power and throttle reasons
  in a background process while a timed region runs (read-only queries).
"""

from __future__ import annotations

import statistics
import subprocess
import tempfile
import time
from typing import Dict, List, Optional

import torch
import torch.distributed as dist


class DeviceTimer:
    def __init__(self, device: torch.device):
        self.device = device
        self.cuda = device.type == "cuda"

    def __enter__(self):
        if self.cuda:
            torch.cuda.synchronize(self.device)
            self.start = torch.cuda.Event(enable_timing=True)
            self.end = torch.cuda.Event(enable_timing=True)
            self.start.record()
        else:
            self.t0 = time.perf_counter()
        return self

    def __exit__(self, *exc):
        if self.cuda:
            self.end.record()
            torch.cuda.synchronize(self.device)
            self.ms = self.start.elapsed_time(self.end)
        else:
            self.ms = (time.perf_counter() - self.t0) * 1e3
        return False


def max_over_ranks(value: float, device: torch.device) -> float:
    if not (dist.is_available() and dist.is_initialized()) or dist.get_world_size() == 1:
        return float(value)
    t = torch.tensor([float(value)], dtype=torch.float64, device=device)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def sum_over_ranks(value: float, device: torch.device) -> float:
    if not (dist.is_available() and dist.is_initialized()) or dist.get_world_size() == 1:
        return float(value)
    t = torch.tensor([float(value)], dtype=torch.float64, device=device)
    dist.all_reduce(t, op=dist.ReduceOp.SUM)
    return float(t.item())


_QUERY = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
          "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
          "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")


class ClockSampler:
    """Background ``nvidia-smi`` sampler (200 ms period) for one GPU index."""

    def __init__(self, gpu_index: int = 0, period_ms: int = 200):
        self.gpu_index = gpu_index
        self.period_ms = period_ms
        self.proc = None
        self.file = None

    def start(self) -> "ClockSampler":
        try:
            self.file = tempfile.NamedTemporaryFile("w+", suffix=".csv", delete=False)
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--id={self.gpu_index}", f"--query-gpu={_QUERY}", "--format=csv,noheader,nounits",
                 f"-lms={self.period_ms}"], stdout=self.file, stderr=subprocess.DEVNULL)
        except (OSError, FileNotFoundError):
            self.proc = None
        return self

    def stop(self) -> Dict[str, object]:
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"], "samples": 0}
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
        self.file.flush()
        self.file.seek(0)
        rows = [r.strip().split(",") for r in self.file.read().splitlines() if r.strip()]
        return summarize_clock_rows(rows)


def summarize_clock_rows(rows: List[List[str]]) -> Dict[str, object]:
    sm, smax, power = [], [], []
    reasons = set()
    names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
    for r in rows:
        if len(r) < 9:
            continue
        try:
            sm.append(float(r[1]))
            smax.append(float(r[2]))
            power.append(float(r[3]))
        except ValueError:
            continue
        for name, flag in zip(names, r[5:9]):
            if flag.strip().lower() in ("active", "1"):
                reasons.add(name)
    if not sm:
        return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["no samples"], "samples": 0}
    loaded = [s for s, p in zip(sm, power) if p > 0.5 * max(power)] or sm
    return {"sm_mhz": statistics.median(loaded), "sm_max_mhz": max(smax), "reasons": sorted(reasons),
            "samples": len(sm), "power_w_max": max(power)}
