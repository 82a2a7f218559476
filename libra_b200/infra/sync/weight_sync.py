"""Trainer -> rollout weight synchronisation front end.

Modes (config ``weight_sync_mode`` / ``rollout_weight_sync_mode``; reference
``infra/sync/weight_sync.py``, ``trainer/async_rl_trainer.py:1132-1560``):

* **disk** - the trainer writes a versioned checkpoint (HF safetensors export +
  manifest) and every HTTP rollout instance reloads it in place
  (``POST /reload_weights``) or is restarted by its supervisor
  (``reload_request.json`` -> ``ack_<instance>_<version>.json``).
* **peer** (the B200 replacement of the reference's NCCL broadcast) - the
  trainer exports its flat bf16 parameter buffer as a CUDA IPC handle; each
  rollout instance maps it and pulls the slices it needs over NVLink
  (``peer_weight_sync``), resharding for its TP degree on the way.
* in-process engines - a device-to-device copy (``LLMEngine.update_weights``).
"""

from __future__ import annotations

import json
import os
import time
import urllib.request
from concurrent.futures import ThreadPoolExecutor
from pathlib import Path
from typing import Any, Dict, Iterable, List, Optional


def _post(url: str, payload: dict, timeout: float) -> dict:
    req = urllib.request.Request(url, data=json.dumps(payload).encode(), headers={"Content-Type": "application/json"},
                                 method="POST")
    with urllib.request.urlopen(req, timeout=timeout + 10) as r:
        if r.status != 200:
            raise RuntimeError(f"{url} returned HTTP {r.status}")
        return json.loads(r.read().decode())


def _http_clients(rollout_engine) -> List[Any]:
    engines = getattr(rollout_engine, "engines", None) or [rollout_engine]
    return [e for e in engines if hasattr(e, "base_url")]


def reload_http_instances(rollout_engine, checkpoint_path: str, version: int, timeout: float = 1200.0,
                          strategy: str = "parallel", route: str = "/reload_weights",
                          extra: Optional[dict] = None) -> Dict[str, dict]:
    clients = _http_clients(rollout_engine)
    payload = {"checkpoint_path": checkpoint_path, "version": int(version), "timeout_seconds": timeout,
               **(extra or {})}
    if not clients:
        return {}
    if strategy == "serial":
        return {c.base_url: _post(c.base_url + route, payload, timeout) for c in clients}
    with ThreadPoolExecutor(max_workers=len(clients)) as pool:
        futs = {c.base_url: pool.submit(_post, c.base_url + route, payload, timeout) for c in clients}
        return {k: f.result() for k, f in futs.items()}


# ------------------------------------------------------------------ sentinel protocol
def write_json_atomic(path: Path, obj: Any) -> None:
    path.parent.mkdir(parents=True, exist_ok=True)
    tmp = path.with_name(f".{path.name}.{os.getpid()}.{time.time_ns()}.tmp")
    tmp.write_text(json.dumps(obj, indent=2, default=str), encoding="utf-8")
    os.replace(tmp, path)


def request_reload(control_dir: str, version: int, checkpoint_path: str, method: str = "restart",
                   strategy: str = "parallel", request_id: str = "", extra: Optional[dict] = None) -> dict:
    """Ask supervisors to reload; returns the request record."""
    req = {"request_id": request_id or f"r{version}-{time.time_ns()}", "version": int(version),
           "checkpoint_path": checkpoint_path, "method": method, "strategy": strategy, "created_at": time.time(),
           **(extra or {})}
    write_json_atomic(Path(control_dir) / "reload_request.json", req)
    return req


def wait_for_acks(control_dir: str, request: dict, instance_ids: Iterable[str], timeout: float = 1200.0,
                  poll_s: float = 0.05) -> Dict[str, dict]:
    """Wait for ``ack_<instance>_<version>.json`` of every instance; raise on an error sentinel or timeout."""
    root = Path(control_dir)
    want = list(instance_ids)
    deadline = time.monotonic() + timeout
    acks: Dict[str, dict] = {}
    while len(acks) < len(want):
        for iid in want:
            if iid in acks:
                continue
            err = root / f"reload_error_{iid}_{request['version']}.json"
            if err.exists():
                raise RuntimeError(f"instance {iid} failed to reload v{request['version']}: {err.read_text()}")
            ack = root / f"ack_{iid}_{request['version']}.json"
            if ack.exists():
                rec = json.loads(ack.read_text())
                if rec.get("request_id") == request["request_id"]:
                    acks[iid] = rec
        if len(acks) < len(want):
            if time.monotonic() > deadline:
                missing = sorted(set(want) - set(acks))
                raise TimeoutError(f"reload v{request['version']}: no ack from {missing} within {timeout}s")
            time.sleep(poll_s)
    return acks


class DiskWeightSync:
    def __init__(self, sync_path: str):
        self.sync_path = sync_path
        self.current_version = 0
        os.makedirs(sync_path, exist_ok=True)

    def save_weights(self, engine, version: int) -> str:
        from libra_b200.engine.checkpointing import DistributedCheckpointManager

        vdir = DistributedCheckpointManager(self.sync_path).save(engine, version, export_for_rollout=True,
                                                                 include_optimizer=False, export_only=True)
        self.current_version = int(version)
        return str(vdir)

    def load_weights(self, params: Dict[str, Any], version: Optional[int] = None) -> int:
        from libra_b200.engine.checkpointing import latest_version, load_params_into

        v = latest_version(self.sync_path) if version is None else version
        if v is None:
            return self.current_version
        load_params_into(params, os.path.join(self.sync_path, f"v{v}"))
        self.current_version = int(v)
        return self.current_version


class WeightSyncFactory:
    @staticmethod
    def create_sync(mode: str, sync_path: str = "./logs/async_rl_weights", **kw):
        if mode == "disk":
            return DiskWeightSync(sync_path)
        if mode in ("peer", "nccl"):
            from libra_b200.infra.sync.peer_weight_sync import PeerWeightSync

            return PeerWeightSync(**kw)
        raise ValueError(f"unknown weight sync mode {mode!r}")
