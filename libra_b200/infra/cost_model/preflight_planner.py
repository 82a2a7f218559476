"""Startup (preflight) planning: one planner pass with the gates forced open.

Before the trainer starts, the planner runs once on a length profile with
interval/warm-up/history gates open and, for ``initial_allocation_strategy ==
"grp"``, no reconfiguration cost or fixed train split; the chosen plan is
written into the config and ``initial_allocation_applied`` is set.  The
trainer refuses to start under the ``grp`` strategy without it (reference
``infra/cost_model/preflight_planner.py``, ``trainer/async_rl_trainer.py:217-228``).
"""

from __future__ import annotations

import copy
import json
from contextlib import contextmanager
from dataclasses import dataclass, field
from pathlib import Path
from typing import Any, Dict, Iterable, List, Optional

from libra_b200.config import AsyncRLConfig
from libra_b200.infra.cost_model.global_resource_planner import (GlobalResourcePlan, GlobalResourcePlanner,
                                                                  PlannerDecision)
from libra_b200.infra.cost_model.startup_profile import summarize_length_profile


@dataclass
class PreflightPlannerResult:
    decision: PlannerDecision
    applied: bool
    planned_config: AsyncRLConfig
    applied_plan: Optional[GlobalResourcePlan] = None
    metadata: Dict[str, Any] = field(default_factory=dict)

    def to_dict(self) -> Dict[str, Any]:
        return {"applied": self.applied, "decision": self.decision.to_dict(),
                "applied_plan": self.applied_plan.to_dict() if self.applied_plan else None,
                "metadata": dict(self.metadata)}


class PreflightPlanner:
    def __init__(self, config: AsyncRLConfig, *, planner: Optional[GlobalResourcePlanner] = None,
                 apply_best_candidate: bool = True):
        self.config = copy.deepcopy(config)
        self.planner = planner or GlobalResourcePlanner.from_config(self.config)
        self.apply_best_candidate = apply_best_candidate

    @contextmanager
    def _gates_open(self, n_records: int):
        p, t = self.planner, self.planner.trigger
        saved = (p.plan_interval, t.interval, p.warmup_steps, p.min_history_size, p.reconfiguration_cost_s,
                 p.min_gain_ratio, p.fixed_train_gpus, t.online, t.last_replan_step)
        try:
            p.plan_interval = t.interval = 1
            p.warmup_steps = 0
            p.min_history_size = max(1, min(n_records, saved[3]))
            if self.apply_best_candidate:
                p.reconfiguration_cost_s = 0.0
                p.min_gain_ratio = 0.0
            if p.initial_allocation_strategy == "grp":
                p.fixed_train_gpus = 0
            t.online = True
            t.last_replan_step = -10 ** 9
            yield
        finally:
            (p.plan_interval, t.interval, p.warmup_steps, p.min_history_size, p.reconfiguration_cost_s,
             p.min_gain_ratio, p.fixed_train_gpus, t.online, _) = saved

    def run(self, history: Iterable[dict]) -> PreflightPlannerResult:
        batch = list(history)
        with self._gates_open(len(batch)):
            decision = self.planner.plan_if_needed(step=0, config=self.config, batch=batch)
        plan = self._select_plan(decision)
        if plan is not None:
            self.planner.apply_plan_to_config(plan, self.config)
            self.config.global_resource_planner.initial_allocation_applied = True
        return PreflightPlannerResult(decision, plan is not None, self.config, plan,
                                      {"num_history_records": len(batch),
                                       "apply_best_candidate": self.apply_best_candidate,
                                       "initial_allocation_strategy": self.planner.initial_allocation_strategy,
                                       "length_profile": summarize_length_profile(batch)})

    def _select_plan(self, d: PlannerDecision) -> Optional[GlobalResourcePlan]:
        cand, cur = d.candidate_plan, d.current_plan
        if cand is None:
            return None
        if self.planner.initial_allocation_strategy == "grp" or d.should_reconfigure:
            return cand
        if self.apply_best_candidate and cur is not None and cand.t_global <= cur.t_global:
            return cand
        return None


def load_history_jsonl(path) -> List[dict]:
    out = []
    with open(path, "r", encoding="utf-8") as fh:
        for line in fh:
            line = line.strip()
            if line:
                obj = json.loads(line)
                if isinstance(obj, dict):
                    out.append(obj)
    return out


def synthetic_history(*, num_requests: int, input_len: int = 1024, output_len: int = 2048) -> List[dict]:
    return [{"input_len": max(1, int(input_len)), "output_len": max(1, int(output_len))}
            for _ in range(max(1, int(num_requests)))]
