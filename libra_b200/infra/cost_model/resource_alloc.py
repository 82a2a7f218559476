"""Legacy heuristic allocators kept for API parity (reference
``infra/cost_model/resource_alloc.py``); the Global Resource Planner is the
path the trainer uses.  ``TrajectoryAwareAllocator`` sizes rollout batch and
concurrency from the recent trajectory-length distribution;
``CostModelAllocator`` delegates to the two-level optimizer.
"""

from __future__ import annotations

import statistics
from dataclasses import dataclass
from typing import List, Optional

from libra_b200.infra.cost_model.model import CostModel, RequestInfo
from libra_b200.infra.cost_model.optimizer import TwoLevelNestedOptimizer


@dataclass
class ResourceConfig:
    max_concurrent_requests: int = 32
    batch_size: int = 32
    gpu_allocation: int = 4
    target_rollout_time: float = 30.0


class TrajectoryAwareAllocator:
    def __init__(self, base_batch_size: int = 32, base_concurrency: int = 32, target_rollout_time: float = 30.0,
                 tokens_per_second_per_gpu: float = 5000.0, window: int = 1000, update_interval: int = 10):
        self.base_batch_size, self.base_concurrency = base_batch_size, base_concurrency
        self.target_rollout_time = target_rollout_time
        self.tps = tokens_per_second_per_gpu
        self.window, self.update_interval = window, update_interval
        self.lengths: List[float] = []

    def update_trajectory_lengths(self, lengths: List[float]) -> None:
        self.lengths = (self.lengths + [float(x) for x in lengths])[-self.window:]

    def _p90(self) -> float:
        if not self.lengths:
            return 1024.0
        s = sorted(self.lengths)
        return s[min(len(s) - 1, int(0.9 * (len(s) - 1)))]

    def allocate_resources(self, num_gpus: int = 4) -> ResourceConfig:
        mean = statistics.fmean(self.lengths) if self.lengths else 1024.0
        tail = self._p90() / max(mean, 1.0)
        budget = self.tps * num_gpus * self.target_rollout_time
        conc = max(1, int(min(4 * self.base_concurrency, budget / max(mean, 1.0) / max(tail, 1.0))))
        batch = max(1, int(min(self.base_batch_size * 2, conc)))
        return ResourceConfig(conc, batch, num_gpus, self.target_rollout_time)

    def estimate_train_time(self) -> float:
        mean = statistics.fmean(self.lengths) if self.lengths else 1024.0
        return self.base_batch_size * mean / max(self.tps, 1.0)

    def should_update_config(self, step: int) -> bool:
        return step > 0 and step % self.update_interval == 0

    def get_statistics(self) -> dict:
        return {"n": len(self.lengths), "mean": statistics.fmean(self.lengths) if self.lengths else 0.0,
                "p90": self._p90() if self.lengths else 0.0}


class SimpleTrajectoryAllocator(TrajectoryAwareAllocator):
    def allocate_resources(self, num_gpus: int = 4) -> ResourceConfig:
        return ResourceConfig(self.base_concurrency, self.base_batch_size, num_gpus, self.target_rollout_time)


class CostModelAllocator:
    def __init__(self, cost_model: Optional[CostModel] = None, calibrator=None):
        self.cost_model = cost_model or CostModel()
        self.calibrator = calibrator
        self.optimizer = TwoLevelNestedOptimizer(self.cost_model)
        self.last_result = None

    def allocate_resources(self, n_total_gpus: int, requests: List[RequestInfo], batch_size: int = 32):
        self.last_result = self.optimizer.optimize(n_total_gpus, requests, B_global=batch_size)
        return self.last_result

    def update_calibration(self, epoch_data) -> dict:
        if self.calibrator is None:
            return {}
        self.calibrator.update(epoch_data)
        return self.calibrator.get_statistics()

    def get_optimization_report(self) -> dict:
        r = self.last_result
        if r is None:
            return {}
        return {"t_train": r.t_train, "t_rollout": r.t_rollout, "t_global": r.t_global,
                "train": vars(r.train_config) if r.train_config else None,
                "rollout": r.rollout_config.tp_list if r.rollout_config else None}
