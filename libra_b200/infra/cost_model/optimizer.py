"""Two-level nested search over (train parallelism) x (rollout TP multiset).

Outer level: every (tp, pp, dp, b_micro) that fits the GPU budget, the
granularity and min-GPU rules, divides the global batch into whole GRPO groups
per DP replica, and does not OOM; candidates whose training time alone already
exceeds the best global time are skipped.  Inner level: integer partitions of
the remaining GPUs into allowed TP sizes (or a fixed per-node pattern),
optionally only heterogeneous ones; the best rollout makespan is kept.
Objective: minimise max(T_train, T_rollout) (reference
``infra/cost_model/optimizer.py``).  On one 8-GPU box the partition space is
tiny, so the inner search is exhaustive.
"""

from __future__ import annotations

import logging
import time
from dataclasses import dataclass, field
from typing import List, Optional

from libra_b200.infra.cost_model.model import RequestInfo, RolloutClusterConfig, TrainParallelConfig

log = logging.getLogger(__name__)
MAX_PARTITIONS = 500


@dataclass
class OptimizationResult:
    train_config: Optional[TrainParallelConfig] = None
    rollout_config: Optional[RolloutClusterConfig] = None
    t_train: float = float("inf")
    t_rollout: float = float("inf")
    t_global: float = float("inf")
    n_configs_explored: int = 0
    n_configs_pruned_oom: int = 0
    n_configs_pruned_early_stop: int = 0
    optimization_time_ms: float = 0.0
    all_evaluated: List[dict] = field(default_factory=list)

    def summary(self) -> str:
        lines = ["Two-level nested optimizer result"]
        if self.train_config is not None:
            t = self.train_config
            lines.append(f"Training: TP={t.tp} PP={t.pp} DP={t.dp} b_micro={t.b_micro} ({t.n_gpus} GPUs)")
        if self.rollout_config is not None:
            lines.append(f"Rollout: {self.rollout_config.tp_list} ({self.rollout_config.n_gpus} GPUs)")
        lines.append(f"T_train={self.t_train:.4f}s T_rollout={self.t_rollout:.4f}s T_global={self.t_global:.4f}s")
        lines.append(f"explored={self.n_configs_explored} oom={self.n_configs_pruned_oom} "
                     f"early_stop={self.n_configs_pruned_early_stop} time={self.optimization_time_ms:.2f}ms")
        return "\n".join(lines)


def _powers_of_two(limit: int) -> List[int]:
    out, v = [], 1
    while v <= limit:
        out.append(v)
        v *= 2
    return out


def generate_training_configs(n_total_gpus: int, max_tp: int = 8, max_pp: int = 8,
                              allowed_tp: Optional[List[int]] = None, allowed_pp: Optional[List[int]] = None,
                              micro_batch_sizes: Optional[List[int]] = None) -> List[TrainParallelConfig]:
    tps = [t for t in (allowed_tp or _powers_of_two(max_tp)) if t <= n_total_gpus]
    pps = [p for p in (allowed_pp or _powers_of_two(max_pp)) if p <= n_total_gpus]
    mbs = micro_batch_sizes or [1, 2, 4, 8]
    return [TrainParallelConfig(tp=tp, pp=pp, dp=dp, b_micro=b)
            for tp in tps for pp in pps if tp * pp <= n_total_gpus
            for dp in range(1, n_total_gpus // (tp * pp) + 1) for b in mbs]


def generate_rollout_configs(n_gpus: int, allowed_tp_sizes: Optional[List[int]] = None,
                             max_instances: int = 32) -> List[RolloutClusterConfig]:
    """Non-increasing partitions of ``n_gpus`` into allowed TP sizes."""
    if n_gpus <= 0:
        return []
    sizes = sorted((t for t in (allowed_tp_sizes or [1, 2, 4, 8]) if t <= n_gpus), reverse=True)
    out: List[RolloutClusterConfig] = []

    def rec(left: int, cap: int, acc: List[int]) -> None:
        if len(out) >= MAX_PARTITIONS:
            return
        if left == 0:
            out.append(RolloutClusterConfig(list(acc)))
            return
        if len(acc) >= max_instances:
            return
        for t in sizes:
            if t <= left and t <= cap:
                acc.append(t)
                rec(left - t, t, acc)
                acc.pop()

    rec(n_gpus, max(sizes) if sizes else 0, [])
    return out


class TwoLevelNestedOptimizer:
    def __init__(self, cost_model, allowed_rollout_tp: Optional[List[int]] = None, max_rollout_instances: int = 32,
                 require_heterogeneous_rollout_tp: bool = False, verbose: bool = False):
        self.cost_model = cost_model
        self.allowed_rollout_tp = allowed_rollout_tp or [1, 2, 4, 8]
        self.max_rollout_instances = max_rollout_instances
        self.require_heterogeneous_rollout_tp = require_heterogeneous_rollout_tp
        self.verbose = verbose

    def _rollout_candidates(self, n: int, pattern: Optional[List[int]]) -> List[RolloutClusterConfig]:
        if pattern:
            per = sum(pattern)
            cands = [RolloutClusterConfig(list(pattern) * (n // per))] if per and n % per == 0 else []
        else:
            cands = generate_rollout_configs(n, self.allowed_rollout_tp, self.max_rollout_instances)
        if self.require_heterogeneous_rollout_tp:
            cands = [c for c in cands if len(set(c.tp_list)) > 1]
        return cands

    def _best_rollout(self, cands: List[RolloutClusterConfig], requests: List[RequestInfo]):
        best, best_t, best_d = None, float("inf"), {}
        for rc in cands:
            t, d = self.cost_model.evaluate_rollout(rc, requests)
            if t < best_t:
                best, best_t, best_d = rc, t, d
        return best, best_t, best_d

    def optimize(self, n_total_gpus: int, requests: List[RequestInfo], B_global: int = 32,
                 allowed_train_tp: Optional[List[int]] = None, allowed_train_pp: Optional[List[int]] = None,
                 micro_batch_sizes: Optional[List[int]] = None, fixed_train_gpus: int = 0,
                 allocation_granularity_gpus: int = 1, min_train_gpus: int = 1, min_rollout_gpus: int = 1,
                 rollout_node_tp_pattern: Optional[List[int]] = None, train_cp_size: int = 1,
                 dp_batch_group_size: int = 1) -> OptimizationResult:
        t0 = time.perf_counter()
        L = int(sum(r.total_length for r in requests) / len(requests)) if requests else 1024
        res = OptimizationResult()
        gran = max(1, int(allocation_granularity_gpus))
        configs = generate_training_configs(n_total_gpus, allowed_tp=allowed_train_tp, allowed_pp=allowed_train_pp,
                                            micro_batch_sizes=micro_batch_sizes)
        for c in configs:
            c.cp = max(1, int(train_cp_size))
        configs = [c for c in configs if c.n_gpus >= max(1, min_train_gpus) and c.n_gpus % gran == 0
                   and n_total_gpus - c.n_gpus >= max(1, min_rollout_gpus)
                   and (fixed_train_gpus <= 0 or c.n_gpus == fixed_train_gpus)]
        pattern = [int(t) for t in (rollout_node_tp_pattern or [])]
        rollout_cache = {}
        for tc in configs:
            res.n_configs_explored += 1
            if B_global % max(1, tc.dp * tc.b_micro) or (B_global // tc.dp) % max(1, int(dp_batch_group_size)):
                continue
            if self.cost_model.check_train_oom(tc, B_global, L):
                res.n_configs_pruned_oom += 1
                continue
            t_train, _ = self.cost_model.evaluate_training(tc, B_global, L)
            if t_train >= res.t_global:
                res.n_configs_pruned_early_stop += 1
                continue
            n_roll = n_total_gpus - tc.n_gpus
            if n_roll not in rollout_cache:
                rollout_cache[n_roll] = self._best_rollout(self._rollout_candidates(n_roll, pattern), requests)
            rc, t_roll, _ = rollout_cache[n_roll]
            if rc is None:
                continue
            tg = max(t_train, t_roll)
            if self.verbose:
                res.all_evaluated.append({"train": {"tp": tc.tp, "pp": tc.pp, "cp": tc.cp, "dp": tc.dp,
                                                    "b_micro": tc.b_micro}, "rollout": rc.tp_list,
                                          "t_train": t_train, "t_rollout": t_roll, "t_global": tg})
            if tg < res.t_global:
                res.train_config, res.rollout_config = tc, rc
                res.t_train, res.t_rollout, res.t_global = t_train, t_roll, tg
        res.optimization_time_ms = (time.perf_counter() - t0) * 1e3
        if self.verbose:
            log.info(res.summary())
        return res

    def optimize_rollout_only(self, n_rollout_gpus: int, requests: List[RequestInfo]):
        return self._best_rollout(self._rollout_candidates(n_rollout_gpus, None), requests)
