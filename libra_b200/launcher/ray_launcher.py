"""Ray launcher for multi-node runs (reference ``launcher/ray_launcher.py``).

Ray is optional: on one box use ``box_launcher``.  With Ray installed, a
``TrainActor`` per training GPU runs the trainer entry point and a
``RolloutWorker`` per rollout instance runs our rollout server; the actors are
plain process wrappers so the training code is the same as under torchrun.
"""

from __future__ import annotations

import importlib.util
import os
import sys


def ray_available() -> bool:
    return importlib.util.find_spec("ray") is not None


class RayAsyncLauncher:
    def __init__(self, config, config_path: str = "", train_entry: str = "examples/train.py"):
        if not ray_available():
            raise ImportError("ray is not installed; use libra_b200.launcher.box_launcher on a single box")
        self.config, self.config_path, self.train_entry = config, config_path, train_entry

    def launch(self):
        import ray

        from libra_b200.launcher.box_launcher import BoxLauncher

        ray.init(address=os.environ.get("RAY_ADDRESS", "auto"), ignore_reinit_error=True)
        box = BoxLauncher(self.config, self.config_path, self.train_entry)

        @ray.remote(num_gpus=0)
        def run(cmd: str) -> int:
            import subprocess

            return subprocess.call(cmd, shell=True)

        rollout = [run.remote(str(c["command"])) for c in box.rollout_commands()]
        trainer = run.remote(box.train_command())
        rc = ray.get(trainer)
        for r in rollout:
            ray.cancel(r, force=True)
        return rc


def launch_ray_cluster(config, config_path: str = ""):
    return RayAsyncLauncher(config, config_path).launch()
