"""Tensor-parallel rollout buckets as real multi-process servers.

A heterogeneous rollout pool mixes instances of different TP degrees (the
reference's ``engine/heterogeneous_engine.py:207-309`` starts one vLLM server
per bucket with ``--tensor-parallel-size``).  A TP-k bucket here is k server
processes, one per GPU of the bucket (``python -m libra_b200.engine.server
--tp k`` under ``torch.distributed.run``): TP rank 0 schedules, samples and
serves HTTP, the others replay its steps, and every row-parallel linear of a
step is reduced over NVLink peer memory fused with the residual add and the
next RMSNorm.  The trainer talks to the bucket through the HTTP client and
syncs weights into it with ``/reload_weights_peer`` (each server rank pulls
its own TP slice straight from the trainer's flat buffer over NVLink) or from
a checkpoint directory (``/reload_weights``).

``TPServerGroup`` owns the launched processes: one process group (its own
session), stopped by that group id only.
"""

from __future__ import annotations

import json
import os
import signal
import socket
import subprocess
import sys
import time
import urllib.request
from typing import List, Optional, Sequence


def free_port() -> int:
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


class TPServerGroup:
    def __init__(self, model: str, tp: int, gpus: Sequence[int], port: int = 0, *, checkpoint: str = "",
                 kv_memory_fraction: float = 0.5, max_batch_tokens: int = 8192, device: str = "cuda",
                 log_path: str = "", startup_timeout: float = 600.0, extra_env: Optional[dict] = None):
        if tp < 1:
            raise ValueError("tp must be >= 1")
        if device == "cuda" and len(gpus) < tp:
            raise ValueError(f"a TP-{tp} bucket needs {tp} GPUs, got {list(gpus)}")
        self.model, self.tp, self.gpus = model, int(tp), [int(g) for g in gpus][:tp]
        self.host, self.port = "127.0.0.1", int(port) or free_port()
        env = dict(os.environ)
        for k in ("RANK", "LOCAL_RANK", "WORLD_SIZE", "LOCAL_WORLD_SIZE", "MASTER_ADDR", "MASTER_PORT",
                  "GROUP_RANK", "ROLE_RANK", "ROLE_WORLD_SIZE", "TORCHELASTIC_RUN_ID"):
            env.pop(k, None)  # the bucket is its own torch.distributed job
        if device == "cuda":
            env["CUDA_VISIBLE_DEVICES"] = ",".join(str(g) for g in self.gpus)
        env.update(extra_env or {})
        here = os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
        env["PYTHONPATH"] = here + os.pathsep + env.get("PYTHONPATH", "")
        server = ["-m", "libra_b200.engine.server", "--model", model, "--port", str(self.port), "--tp", str(self.tp),
                  "--kv-memory-fraction", str(kv_memory_fraction), "--max-batch-tokens", str(max_batch_tokens),
                  "--device", "cuda:0" if device == "cuda" else "cpu"]
        if checkpoint:
            server += ["--checkpoint", checkpoint]
        if self.tp > 1:
            cmd = [sys.executable, "-m", "torch.distributed.run", "--nnodes=1", f"--nproc-per-node={self.tp}",
                   "--master-addr", "127.0.0.1", "--master-port", str(free_port())] + server
        else:
            cmd = [sys.executable] + server
        self._log = open(log_path, "w") if log_path else subprocess.DEVNULL
        self.proc = subprocess.Popen(cmd, env=env, stdout=self._log, stderr=subprocess.STDOUT,
                                     start_new_session=True)
        self._wait_healthy(startup_timeout)

    @property
    def base_url(self) -> str:
        return f"http://{self.host}:{self.port}"

    def _wait_healthy(self, timeout: float) -> None:
        deadline = time.monotonic() + timeout
        while time.monotonic() < deadline:
            if self.proc.poll() is not None:
                raise RuntimeError(f"TP-{self.tp} server group exited with code {self.proc.returncode}")
            try:
                with urllib.request.urlopen(self.base_url + "/health", timeout=2) as r:
                    if r.status == 200:
                        return
            except OSError:
                pass
            time.sleep(0.5)
        self.close()
        raise TimeoutError(f"TP-{self.tp} server group did not become healthy within {timeout:.0f}s")

    def client(self, model_path: str = "", instance_id: str = ""):
        from libra_b200.engine.rollout_engine import HTTPRolloutEngine

        return HTTPRolloutEngine(self.host, self.port, model_path or self.model,
                                 instance_id=instance_id or f"tp{self.tp}-{self.host}:{self.port}")

    def post(self, route: str, body: dict, timeout: float = 600.0) -> dict:
        req = urllib.request.Request(self.base_url + route, data=json.dumps(body).encode(), method="POST",
                                     headers={"Content-Type": "application/json"})
        with urllib.request.urlopen(req, timeout=timeout) as r:
            data = r.read()
        return json.loads(data) if data else {}

    def reload_peer(self, request: dict, timeout: float = 600.0) -> dict:
        """Weight sync over NVLink: ``request`` is ``peer_weight_sync.publish(engine)``."""
        return self.post("/reload_weights_peer", request, timeout)

    def reload_disk(self, checkpoint_path: str, version: int, timeout: float = 600.0) -> dict:
        return self.post("/reload_weights", {"checkpoint_path": checkpoint_path, "version": int(version)}, timeout)

    def close(self, timeout: float = 30.0) -> None:
        if self.proc.poll() is None:
            try:
                os.killpg(self.proc.pid, signal.SIGTERM)  # the group this object started, nothing else
                self.proc.wait(timeout=timeout)
            except (ProcessLookupError, subprocess.TimeoutExpired):
                try:
                    os.killpg(self.proc.pid, signal.SIGKILL)
                except ProcessLookupError:
                    pass
        if self._log not in (None, subprocess.DEVNULL):
            self._log.close()
            self._log = None
