"""Single-box launcher: rollout servers on the rollout GPUs, trainer via torchrun.

The reference starts a Ray cluster with a train actor and rollout actors
(``launcher/ray_launcher.py:8-142``).  One B200 box needs no cluster manager:
this launcher plans the GPU split from the config (the planner's
``heterogeneous_rollout.instances`` when present), starts one rollout server per
instance in its own session (HTTP rollout backend), waits for their health
checks, then runs the trainer under ``torch.distributed.run`` on the training
GPUs.  ``rollout_backend: native`` configs skip the servers (the trainer owns
in-process engines).  ``--dry-run`` prints the commands.

    python -m libra_b200.launcher.box_launcher --config cfg.yaml [--dry-run]
"""

from __future__ import annotations

import argparse
import os
import shlex
import sys
import time
from typing import Dict, List

from libra_b200.launcher.cluster import build_rollout_launch_commands, compute_gpu_allocation


class BoxLauncher:
    def __init__(self, config, config_path: str, train_entry: str = "examples/train.py", python: str = ""):
        self.config, self.config_path, self.train_entry = config, config_path, train_entry
        self.python = python or sys.executable
        self.procs: List = []

    def rollout_commands(self) -> List[Dict[str, object]]:
        c, h = self.config, self.config.heterogeneous_rollout
        model = os.path.basename(str(c.model_path or "qwen3-4b")).lower()
        ckpt = c.model_path if c.model_path and os.path.isdir(c.model_path) else ""
        if h.instances:
            cmds = []
            for i, inst in enumerate(h.instances):
                alloc = compute_gpu_allocation(["127.0.0.1"], max(8, max(inst.gpus) + 1), 0, 0)[0]
                alloc.rollout_gpu_ids = list(inst.gpus)
                port = int(inst.port or int(h.vllm_base_port) + i)
                cmds += build_rollout_launch_commands([alloc], model, ckpt, base_port=port, tp_list=[int(inst.tp)],
                                                      kv_memory_fraction=h.gpu_memory_utilization, python=self.python)
            return cmds
        alloc = compute_gpu_allocation(["127.0.0.1"], 8, int(c.train_gpus), int(c.rollout_gpus))
        return build_rollout_launch_commands(alloc, model, ckpt, tp_size=int(getattr(c, "vllm_tp_size", 1) or 1),
                                             base_port=int(h.vllm_base_port), python=self.python,
                                             kv_memory_fraction=h.gpu_memory_utilization)

    def train_command(self) -> str:
        dev = ",".join(str(g) for g in range(int(self.config.train_gpus)))
        return (f"CUDA_VISIBLE_DEVICES={dev} {shlex.quote(self.python)} -m torch.distributed.run --standalone "
                f"--local-addr 127.0.0.1 --nproc-per-node {int(self.config.train_gpus)} {self.train_entry} "
                f"--config {shlex.quote(self.config_path)}")

    def launch(self, dry_run: bool = False, ready_timeout_s: float = 600.0) -> int:
        from libra_b200.infra.elastic.runtime_executor import ProcessLauncher

        native = str(getattr(self.config, "rollout_backend", "")).lower() in ("native", "local")
        cmds = [] if native else self.rollout_commands()
        train = self.train_command()
        if dry_run:
            for c in cmds:
                print(c["command"])
            print(train)
            return 0
        pl = ProcessLauncher()
        env = dict(os.environ)
        try:
            for c in cmds:
                self.procs.append(pl.start(str(c["command"]), env))
            for c in cmds:
                pl.wait_ready("127.0.0.1", int(c["port"]), ready_timeout_s)
            trainer = pl.start(train, env)
            self.procs.append(trainer)
            return trainer.wait()
        finally:
            for p in self.procs:
                pl.stop(p, 30.0)


def main(argv=None) -> int:
    from libra_b200.config import AsyncRLConfig

    ap = argparse.ArgumentParser(description="libra_b200 single-box launcher")
    ap.add_argument("--config", required=True)
    ap.add_argument("--train-entry", default="examples/train.py")
    ap.add_argument("--dry-run", action="store_true")
    a = ap.parse_args(argv)
    cfg = AsyncRLConfig.from_file(a.config)
    return BoxLauncher(cfg, a.config, a.train_entry).launch(dry_run=a.dry_run)


if __name__ == "__main__":
    raise SystemExit(main())
