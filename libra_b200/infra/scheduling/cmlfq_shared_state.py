"""Cross-process C-MLFQ load counters (reference ``infra/scheduling/cmlfq_shared_state.py``).

Each process owns one ``rank_<R>.json`` snapshot in a shared directory (atomic
rename on every change plus a heartbeat thread); readers sum the counters of
all snapshots whose heartbeat is younger than the TTL, so counters left by a
dead process stop counting after the TTL.
"""

from __future__ import annotations

import atexit
import json
import os
import socket
import threading
import time
from collections import Counter
from pathlib import Path
from typing import Dict


class SharedCMLFQLoadState:
    def __init__(self, directory: str, ttl_s: float = 60.0, heartbeat_interval_s: float = 10.0, writer_id: str = ""):
        self.directory = Path(directory)
        self.directory.mkdir(parents=True, exist_ok=True)
        self.writer_id = writer_id or f"rank_{os.environ.get('RANK', '0')}"
        self.heartbeat_interval_s = max(1.0, heartbeat_interval_s)
        self.ttl_s = max(2.0 * heartbeat_interval_s, ttl_s)
        self._path = self.directory / f"{self.writer_id}.json"
        self._counts: Counter = Counter()
        self._lock = threading.Lock()
        self._stop = threading.Event()
        self._write()
        self._thread = threading.Thread(target=self._beat, daemon=True, name=f"cmlfq-heartbeat-{self.writer_id}")
        self._thread.start()
        atexit.register(self.close)

    def increment(self, instance_id: str) -> None:
        with self._lock:
            self._counts[instance_id] += 1
            self._write_locked()

    def decrement(self, instance_id: str) -> None:
        with self._lock:
            self._counts[instance_id] = max(0, self._counts[instance_id] - 1)
            self._write_locked()

    def aggregate(self) -> Dict[str, int]:
        now = time.time()
        total: Counter = Counter()
        for p in self.directory.glob("rank_*.json"):
            try:
                snap = json.loads(p.read_text(encoding="utf-8"))
                if now - float(snap.get("updated_at", 0.0)) > self.ttl_s:
                    continue
                for inst, n in snap.get("counts", {}).items():
                    total[str(inst)] += max(0, int(n))
            except (OSError, ValueError, TypeError):
                continue
        return dict(total)

    def close(self) -> None:
        if self._stop.is_set():
            return
        self._stop.set()
        with self._lock:
            self._counts.clear()
            self._write_locked()

    def _beat(self) -> None:
        while not self._stop.wait(self.heartbeat_interval_s):
            self._write()

    def _write(self) -> None:
        with self._lock:
            self._write_locked()

    def _write_locked(self) -> None:
        snap = {"writer_id": self.writer_id, "rank": int(os.environ.get("RANK", "0")), "pid": os.getpid(),
                "hostname": socket.gethostname(), "updated_at": time.time(), "counts": dict(self._counts)}
        tmp = self._path.with_name(f".{self._path.name}.{os.getpid()}.{threading.get_ident()}.tmp")
        tmp.write_text(json.dumps(snap, sort_keys=True), encoding="utf-8")
        os.replace(tmp, self._path)
