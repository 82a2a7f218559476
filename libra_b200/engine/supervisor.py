"""Restartable rollout-server supervisor (reference ``scripts/restartable_vllm_server.py``).

Runs one rollout server command in its own session and restarts it when it
exits unexpectedly (bounded retries with backoff) or when a reload sentinel
file appears (the disk weight-sync path that restarts instead of hot-reloading:
the trainer writes ``<sentinel>`` with the new checkpoint path, the supervisor
restarts the server on it and writes ``<sentinel>.ack``).

    python -m libra_b200.engine.supervisor --sentinel /tmp/reload.json -- \\
        python -m libra_b200.engine.server --model qwen3-4b --port 8000
"""

from __future__ import annotations

import argparse
import json
import os
import shlex
import signal
import time
from typing import List, Optional


class Supervisor:
    def __init__(self, command: List[str], sentinel: str = "", max_restarts: int = 5, backoff_s: float = 2.0,
                 poll_s: float = 0.5, stop_timeout_s: float = 30.0, launcher=None):
        from libra_b200.infra.elastic.runtime_executor import ProcessLauncher

        self.command, self.sentinel = list(command), sentinel
        self.max_restarts, self.backoff_s, self.poll_s, self.stop_timeout_s = max_restarts, backoff_s, poll_s, stop_timeout_s
        self.launcher = launcher or ProcessLauncher()
        self.proc = None
        self.restarts = 0
        self.stopped = False
        self.checkpoint = ""

    def _cmd(self) -> str:
        cmd = list(self.command)
        if self.checkpoint:
            if "--checkpoint" in cmd:
                cmd[cmd.index("--checkpoint") + 1] = self.checkpoint
            else:
                cmd += ["--checkpoint", self.checkpoint]
        return " ".join(shlex.quote(c) for c in cmd)

    def start(self) -> None:
        self.proc = self.launcher.start(self._cmd(), dict(os.environ))

    def stop(self) -> None:
        if self.proc is not None:
            self.launcher.stop(self.proc, self.stop_timeout_s)
            self.proc = None

    def _reload_request(self) -> Optional[dict]:
        if not self.sentinel or not os.path.exists(self.sentinel):
            return None
        try:
            with open(self.sentinel, encoding="utf-8") as f:
                req = json.load(f)
        except (OSError, ValueError):
            return None
        os.remove(self.sentinel)
        return req

    def poll_once(self) -> str:
        """One supervision step; returns what happened."""
        req = self._reload_request()
        if req is not None:
            self.stop()
            self.checkpoint = str(req.get("checkpoint_path", self.checkpoint))
            self.start()
            with open(self.sentinel + ".ack", "w", encoding="utf-8") as f:
                json.dump({"version": req.get("version"), "pid": self.proc.pid, "time": time.time()}, f)
            return "reloaded"
        if self.proc is not None and self.proc.poll() is not None:
            if self.restarts >= self.max_restarts:
                self.stopped = True
                return "gave_up"
            self.restarts += 1
            time.sleep(self.backoff_s * self.restarts)
            self.start()
            return "restarted"
        return "running"

    def run(self) -> int:
        def _term(*_):
            self.stopped = True

        signal.signal(signal.SIGTERM, _term)
        signal.signal(signal.SIGINT, _term)
        self.start()
        while not self.stopped:
            if self.poll_once() == "gave_up":
                break
            time.sleep(self.poll_s)
        self.stop()
        return 0 if self.restarts < self.max_restarts else 1


def main(argv=None) -> int:
    ap = argparse.ArgumentParser(description="restart a rollout server on crash or reload request")
    ap.add_argument("--sentinel", default="")
    ap.add_argument("--max-restarts", type=int, default=5)
    ap.add_argument("command", nargs=argparse.REMAINDER)
    a = ap.parse_args(argv)
    cmd = a.command[1:] if a.command[:1] == ["--"] else a.command
    return Supervisor(cmd, a.sentinel, a.max_restarts).run()


if __name__ == "__main__":
    raise SystemExit(main())
