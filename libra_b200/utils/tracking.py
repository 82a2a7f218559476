"""Experiment tracking (reference: wandb calls in trainer/async_rl_trainer.py:1748-1812).

``Tracker.create(config)`` returns a wandb-backed tracker when ``wandb`` is
importable and enabled (``config.wandb_project`` or ``WANDB_PROJECT``),
otherwise a JSONL tracker writing ``<log_dir>/metrics.jsonl``.  Only rank 0
logs.
"""

from __future__ import annotations

import json
import os
import time
from typing import Any, Dict, Optional


class JsonlTracker:
    def __init__(self, path: str, run_config: Optional[Dict[str, Any]] = None):
        os.makedirs(os.path.dirname(os.path.abspath(path)), exist_ok=True)
        self.path = path
        self._fh = open(path, "a", encoding="utf-8")
        if run_config is not None:
            self._write({"event": "config", "time": time.time(), "config": run_config})

    def _write(self, rec: Dict[str, Any]) -> None:
        self._fh.write(json.dumps(rec, default=str) + "\n")
        self._fh.flush()

    def log(self, metrics: Dict[str, Any], step: int) -> None:
        self._write({"event": "metrics", "step": int(step), "time": time.time(),
                     **{k: v for k, v in metrics.items() if isinstance(v, (int, float, str, bool))}})

    def finish(self) -> None:
        if not self._fh.closed:
            self._fh.close()


class WandbTracker:
    def __init__(self, project: str, name: str = "", run_config: Optional[Dict[str, Any]] = None):
        import wandb

        self._wandb = wandb
        self.run = wandb.init(project=project, name=name or None, config=run_config or {})

    def log(self, metrics: Dict[str, Any], step: int) -> None:
        self._wandb.log({k: v for k, v in metrics.items() if isinstance(v, (int, float))}, step=int(step))

    def finish(self) -> None:
        self.run.finish()


class NullTracker:
    def log(self, metrics, step) -> None:
        pass

    def finish(self) -> None:
        pass


class Tracker:
    @staticmethod
    def create(config, rank: int = 0):
        if rank != 0:
            return NullTracker()
        project = getattr(config, "wandb_project", "") or os.environ.get("WANDB_PROJECT", "")
        run_cfg = config.to_dict() if hasattr(config, "to_dict") else None
        if project and os.environ.get("WANDB_MODE", "") != "disabled":
            try:
                return WandbTracker(project, getattr(config, "experiment_name", ""), run_cfg)
            except Exception:  # noqa: BLE001 - wandb missing or offline: fall back to a local file
                pass
        return JsonlTracker(os.path.join(getattr(config, "log_dir", "./logs"), "metrics.jsonl"), run_cfg)
