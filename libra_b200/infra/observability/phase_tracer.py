"""Per-rank phase spans as append-only JSONL (schema ``libra.phase_trace.v1``).

Record layout is the reference's (``infra/observability/phase_tracer.py``):
``phase_start`` / ``phase_span`` (start_ns, end_ns, duration_s, details) /
``phase_unfinished`` events tagged with rank and world size, so existing trace
tooling keeps working.  B200 addition: ``device_span`` records carry the
CUDA-event duration of a region measured on the device (``DeviceSpan``), and
``to_chrome`` converts a set of rank files to Chrome/Perfetto "X" events.
"""

from __future__ import annotations

import glob
import json
import os
import threading
import time
from pathlib import Path
from typing import Any, Dict, List, Optional, Tuple

SCHEMA = "libra.phase_trace.v1"


class PhaseTracer:
    def __init__(self, path, *, rank: int, world_size: int):
        self.path = Path(path)
        self.path.parent.mkdir(parents=True, exist_ok=True)
        self.rank, self.world_size = int(rank), int(world_size)
        self._open: Dict[Tuple[int, str], Tuple[int, dict]] = {}
        self._lock = threading.Lock()

    def _emit(self, rec: Dict[str, Any]) -> None:
        line = json.dumps({"schema": SCHEMA, "rank": self.rank, "world_size": self.world_size, **rec},
                          sort_keys=True, default=str)
        with self.path.open("a", encoding="utf-8") as fh:
            fh.write(line + "\n")

    def start(self, step: int, phase: str, details: Optional[dict] = None) -> None:
        now = time.time_ns()
        with self._lock:
            self._open[(int(step), str(phase))] = (now, dict(details or {}))
            self._emit({"event": "phase_start", "step": int(step), "phase": str(phase), "ts_ns": now,
                        "details": dict(details or {})})

    def end(self, step: int, phase: str, details: Optional[dict] = None) -> None:
        now = time.time_ns()
        with self._lock:
            t0, merged = self._open.pop((int(step), str(phase)), (now, {}))
            merged = dict(merged, **(details or {}))
            self._emit({"event": "phase_span", "step": int(step), "phase": str(phase), "start_ns": t0,
                        "end_ns": now, "duration_s": (now - t0) / 1e9, "details": merged})

    def device_span(self, step: int, phase: str, device_ms: float, details: Optional[dict] = None) -> None:
        now = time.time_ns()
        with self._lock:
            self._emit({"event": "device_span", "step": int(step), "phase": str(phase),
                        "start_ns": now - int(device_ms * 1e6), "end_ns": now, "duration_s": device_ms / 1e3,
                        "details": dict(details or {})})

    def close(self) -> None:
        now = time.time_ns()
        with self._lock:
            for (step, phase), (t0, d) in list(self._open.items()):
                self._emit({"event": "phase_unfinished", "step": step, "phase": phase, "start_ns": t0, "end_ns": now,
                            "duration_s": (now - t0) / 1e9, "details": d})
            self._open.clear()


class DeviceSpan:
    """Context manager recording CUDA-event time of a region into a tracer."""

    def __init__(self, tracer: Optional[PhaseTracer], step: int, phase: str, device=None):
        self.tracer, self.step, self.phase, self.device = tracer, step, phase, device

    def __enter__(self):
        import torch

        self.cuda = torch.cuda.is_available() and self.tracer is not None
        if self.cuda:
            self.a, self.b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            self.a.record()
        return self

    def __exit__(self, *exc):
        if self.cuda:
            import torch

            self.b.record()
            self.b.synchronize()
            self.tracer.device_span(self.step, self.phase, self.a.elapsed_time(self.b))
        return False


def to_chrome(paths: List[str]) -> List[Dict[str, Any]]:
    events = []
    for path in paths:
        with open(path, encoding="utf-8") as fh:
            for line in fh:
                r = json.loads(line)
                if r.get("event") not in ("phase_span", "phase_unfinished", "device_span"):
                    continue
                phase = str(r.get("phase", "unknown"))
                events.append({"name": phase, "cat": "libra.device" if r["event"] == "device_span" else "libra.phase",
                               "ph": "X", "ts": int(r["start_ns"]) / 1e3,
                               "dur": max(0.0, (int(r["end_ns"]) - int(r["start_ns"])) / 1e3),
                               "pid": f"rank-{int(r.get('rank', 0))}",
                               "tid": f"gpu:{phase}" if r["event"] == "device_span" else phase,
                               "args": {"step": r.get("step"), **dict(r.get("details") or {})}})
    events.sort(key=lambda e: (e["ts"], str(e["pid"])))
    return events


def main(argv=None) -> None:
    import argparse

    ap = argparse.ArgumentParser(description="Convert phase-trace JSONL files to a Chrome trace")
    ap.add_argument("--input-glob", required=True)
    ap.add_argument("--output", required=True)
    a = ap.parse_args(argv)
    paths = sorted(glob.glob(a.input_glob))
    if not paths:
        raise SystemExit(f"no files match {a.input_glob}")
    out = Path(a.output)
    out.parent.mkdir(parents=True, exist_ok=True)
    out.write_text(json.dumps({"traceEvents": to_chrome(paths), "displayTimeUnit": "ms"}), encoding="utf-8")
    print(f"wrote {out} from {len(paths)} file(s)")


if __name__ == "__main__":
    main()
