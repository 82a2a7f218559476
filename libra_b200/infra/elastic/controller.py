"""Elastic hybrid worker controller (launch/stop requests from a task directory).

Role of the reference's ``scripts/elastic_hybrid_controller.py:40-133``: training
ranks drop ``.launch_<worker>.json`` (``{"command": ..., "env": {...}}``) and
``.stop_<worker>.json`` files into the shared task directory; the controller
claims each request by renaming it, starts or stops exactly the worker it
recorded, and answers with ``.launch_<worker>.started`` (pid) or
``.launch_<worker>.error``.  On a single box the worker is a local process
group started through ``ProcessLauncher``; the reference reaches remote hosts
over SSH instead.

    python -m libra_b200.infra.elastic.controller --task-dir logs/elastic_training_tasks
"""

from __future__ import annotations

import argparse
import json
import os
import signal
import time
from pathlib import Path
from typing import Dict, Optional

from libra_b200.infra.elastic.runtime_executor import ProcessLauncher, write_json_atomic


class Controller:
    def __init__(self, task_dir: str, launcher: Optional[ProcessLauncher] = None, stop_timeout_s: float = 30.0):
        self.task_dir = Path(task_dir)
        self.task_dir.mkdir(parents=True, exist_ok=True)
        self.launcher = launcher or ProcessLauncher()
        self.stop_timeout_s = stop_timeout_s
        self.workers: Dict[str, object] = {}
        self.stopped = False

    def poll_once(self) -> bool:
        handled = self._stops()
        return self._launches() or handled

    def _launches(self) -> bool:
        handled = False
        for req in sorted(self.task_dir.glob(".launch_*.json")):
            wid = req.stem[len(".launch_"):]
            claimed = req.with_suffix(".running")
            try:
                req.replace(claimed)
            except OSError:
                continue
            handled = True
            try:
                spec = json.loads(claimed.read_text(encoding="utf-8"))
                env = {**os.environ, **{str(k): str(v) for k, v in (spec.get("env") or {}).items()}}
                proc = self.launcher.start(str(spec["command"]), env, str(self.task_dir / f"{wid}.controller.log"))
                self.workers[wid] = proc
                write_json_atomic(self.task_dir / f".launch_{wid}.started", {"worker_id": wid, "pid": proc.pid})
            except Exception as exc:  # noqa: BLE001 - reported to the requester
                write_json_atomic(self.task_dir / f".launch_{wid}.error", {"worker_id": wid, "error": str(exc)})
            finally:
                claimed.unlink(missing_ok=True)
        return handled

    def _stops(self) -> bool:
        handled = False
        for req in sorted(self.task_dir.glob(".stop_*.json")):
            wid = req.stem[len(".stop_"):]
            req.unlink(missing_ok=True)
            handled = True
            proc = self.workers.pop(wid, None)
            if proc is not None:
                self.launcher.stop(proc, self.stop_timeout_s)
        return handled

    def stop_all(self) -> None:
        for wid in list(self.workers):
            self.launcher.stop(self.workers.pop(wid), self.stop_timeout_s)

    def run(self, poll_interval: float = 0.5) -> None:
        def _stop(*_):
            self.stopped = True

        signal.signal(signal.SIGTERM, _stop)
        signal.signal(signal.SIGINT, _stop)
        while not self.stopped:
            if not self.poll_once():
                time.sleep(poll_interval)
        self.stop_all()


def request_launch(task_dir: str, worker_id: str, command: str, env: Optional[Dict[str, str]] = None) -> Path:
    path = Path(task_dir) / f".launch_{worker_id}.json"
    write_json_atomic(path, {"worker_id": worker_id, "command": command, "env": env or {}})
    return path


def request_stop(task_dir: str, worker_id: str) -> Path:
    path = Path(task_dir) / f".stop_{worker_id}.json"
    write_json_atomic(path, {"worker_id": worker_id})
    return path


def main(argv=None) -> None:
    ap = argparse.ArgumentParser(description="libra_b200 elastic hybrid worker controller")
    ap.add_argument("--task-dir", required=True)
    ap.add_argument("--poll-interval", type=float, default=0.5)
    a = ap.parse_args(argv)
    Controller(a.task_dir).run(a.poll_interval)


if __name__ == "__main__":
    main()
