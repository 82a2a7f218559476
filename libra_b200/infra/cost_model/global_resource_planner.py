"""Global Resource Planner (GRP): online replanning of the training/rollout split.

Behaviour (reference ``infra/cost_model/global_resource_planner.py``):

* keeps a bounded window of observed (prompt, generation) lengths and runtime
  pressure snapshots from the dispatcher;
* decides *when* to plan (``ReplanTrigger``): never during warm-up or a
  cooldown after a reconfiguration; on the plan interval; or early on queue
  pressure >= 0.75, active-rollout pressure >= 0.85, >= 8 newly rejected
  rollouts, or rollout/train time ratio >= 1.25;
* runs the two-level optimizer, compares the candidate with the current plan
  and reconfigures only if the net gain (raw gain minus the reconfiguration
  cost) is positive and the relative gain reaches ``min_gain_ratio``;
  ``GRP_FORCE_ROLLOUT_TP_LIST`` / ``GRP_FORCE_TRAIN_GPUS`` /
  ``GRP_FORCE_RUNTIME_RECONFIGURE`` override the search;
* emits an Elastic-Hybrid-Pool signal (``ElasticHybridPolicy``) in units of
  complete DP replicas with borrow/release hysteresis (1.15 / 0.90 train/rollout
  ratio) and rollout-pressure protection (0.80);
* rewrites the config (GPU split, TP/PP/DP, rollout instances/ports/GPUs).

On one 8xB200 box the planner's GPU budget is at most 8 and every rollout
instance lives on the same host; GPU ids are assigned contiguously.
"""

from __future__ import annotations

import logging
import os
import re
from dataclasses import dataclass, field
from typing import Any, Dict, List, Optional, Tuple

from libra_b200.config import AsyncRLConfig, HeterogeneousInstanceConfig
from libra_b200.infra.cost_model.model import RequestInfo, RolloutClusterConfig, TrainParallelConfig
from libra_b200.infra.cost_model.optimizer import OptimizationResult, TwoLevelNestedOptimizer
from libra_b200.infra.cost_model.simulator_adapters import HybridSimulatorCostModel

log = logging.getLogger(__name__)


@dataclass
class GlobalResourcePlan:
    train_config: TrainParallelConfig
    rollout_config: RolloutClusterConfig
    t_train: float
    t_rollout: float
    t_global: float
    n_total_gpus: int
    max_concurrent_rollouts: int
    expected_gain_s: float = 0.0
    expected_gain_ratio: float = 0.0
    reconfiguration_cost_s: float = 0.0
    metadata: Dict[str, Any] = field(default_factory=dict)

    @property
    def train_gpus(self) -> int:
        return self.train_config.n_gpus

    @property
    def rollout_gpus(self) -> int:
        return self.rollout_config.n_gpus

    @property
    def rollout_tp_list(self) -> List[int]:
        return list(self.rollout_config.tp_list)

    def to_dict(self) -> Dict[str, Any]:
        t = self.train_config
        return {"train": {"tp": t.tp, "pp": t.pp, "dp": t.dp, "cp": t.cp, "b_micro": t.b_micro, "n_gpus": t.n_gpus},
                "rollout": {"tp_list": self.rollout_tp_list, "n_gpus": self.rollout_gpus,
                            "n_instances": self.rollout_config.n_instances},
                "t_train": self.t_train, "t_rollout": self.t_rollout, "t_global": self.t_global,
                "n_total_gpus": self.n_total_gpus, "max_concurrent_rollouts": self.max_concurrent_rollouts,
                "expected_gain_s": self.expected_gain_s, "expected_gain_ratio": self.expected_gain_ratio,
                "reconfiguration_cost_s": self.reconfiguration_cost_s, "metadata": dict(self.metadata)}


@dataclass
class RuntimeResourceMetrics:
    step: int = 0
    queue_pressure: float = 0.0
    active_rollout_pressure: float = 0.0
    accepted_rollouts: int = 0
    rejected_rollouts: int = 0
    rollout_time_s: float = 0.0
    train_time_s: float = 0.0
    step_time_s: float = 0.0
    raw: Dict[str, Any] = field(default_factory=dict)

    @property
    def rollout_train_ratio(self) -> float:
        return self.rollout_time_s / max(self.train_time_s, 1e-6)

    def to_dict(self) -> Dict[str, Any]:
        return {"step": self.step, "queue_pressure": self.queue_pressure,
                "active_rollout_pressure": self.active_rollout_pressure, "accepted_rollouts": self.accepted_rollouts,
                "rejected_rollouts": self.rejected_rollouts, "rollout_time_s": self.rollout_time_s,
                "train_time_s": self.train_time_s, "step_time_s": self.step_time_s,
                "rollout_train_ratio": self.rollout_train_ratio, "raw": dict(self.raw)}


@dataclass
class ElasticHybridSignal:
    """Versioned EHP command; every ``*_workers`` count is in complete DP replicas."""

    step: int
    desired_workers: int
    current_workers: int
    max_workers: int
    action: str
    reason: str
    train_rollout_ratio: float
    rollout_pressure: float
    ttl_steps: int
    active_workers: int = 0
    joining_workers: int = 0
    replica_size_gpus: int = 1

    desired_replicas = property(lambda self: self.desired_workers)
    current_replicas = property(lambda self: self.current_workers)
    capacity_replicas = property(lambda self: self.max_workers)

    @property
    def should_adjust(self) -> bool:
        return self.desired_workers != self.current_workers

    def to_dict(self) -> Dict[str, Any]:
        return {"step": self.step, "desired_workers": self.desired_workers, "current_workers": self.current_workers,
                "max_workers": self.max_workers, "action": self.action, "reason": self.reason,
                "train_rollout_ratio": self.train_rollout_ratio, "rollout_pressure": self.rollout_pressure,
                "ttl_steps": self.ttl_steps, "expires_step": self.step + self.ttl_steps,
                "active_workers": self.active_workers, "joining_workers": self.joining_workers,
                "desired_replicas": self.desired_replicas, "current_replicas": self.current_replicas,
                "capacity_replicas": self.capacity_replicas, "replica_size_gpus": self.replica_size_gpus}


@dataclass
class PlannerDecision:
    step: int
    should_reconfigure: bool
    reason: str
    current_plan: Optional[GlobalResourcePlan] = None
    candidate_plan: Optional[GlobalResourcePlan] = None
    optimization_result: Optional[OptimizationResult] = None
    num_requests: int = 0
    trigger: str = ""
    runtime_metrics: Optional[RuntimeResourceMetrics] = None
    elastic_hybrid_signal: Optional[ElasticHybridSignal] = None

    def to_dict(self) -> Dict[str, Any]:
        d = lambda o: o.to_dict() if o is not None else None  # noqa: E731
        return {"step": self.step, "should_reconfigure": self.should_reconfigure, "reason": self.reason,
                "trigger": self.trigger, "num_requests": self.num_requests,
                "runtime_metrics": d(self.runtime_metrics), "current_plan": d(self.current_plan),
                "candidate_plan": d(self.candidate_plan), "elastic_hybrid_signal": d(self.elastic_hybrid_signal)}


# =============================================================================== policies
@dataclass
class ReplanTrigger:
    online: bool = True
    interval: int = 10
    cooldown: int = 1
    queue_pressure: float = 0.75
    active_pressure: float = 0.85
    rejected_delta: int = 8
    imbalance: float = 1.25
    last_replan_step: int = -10 ** 9
    last_rejected: int = 0

    def __call__(self, step: int, m: Optional[RuntimeResourceMetrics]) -> str:
        if not self.online:
            return "interval_skip"
        if step - self.last_replan_step < self.cooldown:
            return "cooldown"
        if step % self.interval == 0:
            return "interval"
        if m is None:
            return "interval_skip"
        if m.queue_pressure >= self.queue_pressure:
            return "queue_pressure"
        if m.active_rollout_pressure >= self.active_pressure:
            return "active_rollout_pressure"
        if m.rejected_rollouts - self.last_rejected >= self.rejected_delta:
            return "rejected_rollout_delta"
        if m.train_time_s > 0 and m.rollout_train_ratio >= self.imbalance:
            return "rollout_train_imbalance"
        return "interval_skip"

    def observed(self, trigger: str, m: Optional[RuntimeResourceMetrics]) -> None:
        if trigger == "rejected_rollout_delta" and m is not None:
            self.last_rejected = m.rejected_rollouts


@dataclass
class ElasticHybridPolicy:
    enabled: bool = False
    borrow_ratio: float = 1.15
    release_ratio: float = 0.90
    max_rollout_pressure: float = 0.80
    ttl_steps: int = 20

    def __post_init__(self):
        if self.release_ratio > self.borrow_ratio:
            raise ValueError("elastic hybrid release ratio cannot exceed borrow ratio")

    @staticmethod
    def _count(stats: dict, *keys: str) -> int:
        for k in keys:
            if k in stats:
                return max(0, int(stats.get(k) or 0))
        return 0

    def signal(self, step: int, config: AsyncRLConfig, current: GlobalResourcePlan, candidate: GlobalResourcePlan,
               m: Optional[RuntimeResourceMetrics]) -> Optional[ElasticHybridSignal]:
        if not self.enabled:
            return None
        pc = config.global_resource_planner
        width = max(1, config.train_tp_size) * max(1, config.train_pp_size) * max(1, config.train_cp_size)
        replica = int(pc.elastic_hybrid_replica_size_gpus or 0)
        if replica > 0 and replica != width:
            raise ValueError(f"elastic_hybrid_replica_size_gpus must equal one complete DP Replica ({width}); "
                             f"got {replica}")
        replica = replica or width
        capacity = max(0, (int(config.rollout_gpus) - max(0, int(pc.elastic_hybrid_min_rollout_gpus or 0))) // replica)
        stats = m.raw.get("step_stats", {}) if m is not None else {}
        active = self._count(stats, "active_hybrid_replicas", "active_hybrid_workers")
        joining = max(self._count(stats, "joining_hybrid_replicas", "joining_hybrid_workers"),
                      self._count(stats, "pending_hybrid_replica_joins", "pending_hybrid_joins"))
        cur = active + joining
        t_train = m.train_time_s if m is not None and m.train_time_s > 0 else (candidate.t_train or current.t_train)
        t_roll = m.rollout_time_s if m is not None and m.rollout_time_s > 0 else (candidate.t_rollout or current.t_rollout)
        ratio = float(t_train) / max(float(t_roll), 1e-6)
        pressure = max(m.queue_pressure, m.active_rollout_pressure) if m is not None else 0.0
        extra = max(0, (candidate.train_gpus - int(config.train_gpus)) // replica)
        if capacity <= 0:
            want, why = 0, "no_complete_replica_capacity"
        elif pressure >= self.max_rollout_pressure:
            want, why = 0, "protect_rollout_capacity"
        elif extra > 0:
            want, why = min(capacity, extra), "candidate_requests_more_training_capacity"
        elif ratio >= self.borrow_ratio:
            want, why = capacity, "training_bottleneck"
        elif ratio <= self.release_ratio:
            want, why = 0, "rollout_bottleneck"
        else:
            want, why = cur, "hysteresis_hold"
        action = "join" if want > cur else "release" if want < cur else "hold"
        return ElasticHybridSignal(int(step), int(want), int(cur), int(capacity), action, why, float(ratio),
                                   float(pressure), int(self.ttl_steps), active, joining, replica)


def _env_ints(name: str) -> Optional[List[int]]:
    raw = os.environ.get(name, "").strip()
    if not raw:
        return None
    try:
        return [int(x) for x in re.split(r"[,;:]", raw) if x.strip()]
    except ValueError as exc:
        raise ValueError(f"Invalid {name}={raw!r}") from exc


# =============================================================================== planner
class GlobalResourcePlanner:
    """Periodic planner minimising max(T_train, T_rollout)."""

    def __init__(self, evaluator, n_total_gpus: int, plan_interval: int = 10, warmup_steps: int = 1,
                 min_history_size: int = 8, min_gain_ratio: float = 0.05, reconfiguration_cost_s: float = 15.0,
                 allowed_rollout_tp: Optional[List[int]] = None, require_heterogeneous_rollout_tp: bool = False,
                 allowed_train_tp: Optional[List[int]] = None, allowed_train_pp: Optional[List[int]] = None,
                 fixed_train_gpus: int = 0, initial_allocation_strategy: str = "grp",
                 allocation_granularity_gpus: int = 1, min_train_gpus: int = 1, min_rollout_gpus: int = 1,
                 micro_batch_sizes: Optional[List[int]] = None, max_history_size: int = 4096,
                 online_replanning: bool = True, replan_cooldown_steps: int = 1, queue_pressure_threshold: float = 0.75,
                 active_rollout_pressure_threshold: float = 0.85, rejected_rollout_delta_threshold: int = 8,
                 rollout_train_imbalance_threshold: float = 1.25, elastic_hybrid_planning_enabled: bool = False,
                 elastic_hybrid_max_workers: int = 0, elastic_hybrid_borrow_train_rollout_ratio: float = 1.15,
                 elastic_hybrid_release_train_rollout_ratio: float = 0.90,
                 elastic_hybrid_max_rollout_pressure: float = 0.80, elastic_hybrid_signal_ttl_steps: int = 20,
                 verbose: bool = False):
        if initial_allocation_strategy not in ("grp", "configured"):
            raise ValueError("initial_allocation_strategy must be 'grp' or 'configured'")
        self.evaluator = evaluator
        self.n_total_gpus = int(n_total_gpus)
        self.warmup_steps = max(0, int(warmup_steps))
        self.min_history_size = max(1, int(min_history_size))
        self.min_gain_ratio = max(0.0, float(min_gain_ratio))
        self.reconfiguration_cost_s = max(0.0, float(reconfiguration_cost_s))
        self.allowed_rollout_tp = allowed_rollout_tp or [1, 2, 4, 8]
        self.allowed_train_tp, self.allowed_train_pp = allowed_train_tp, allowed_train_pp
        self.fixed_train_gpus = int(fixed_train_gpus or 0)
        self.initial_allocation_strategy = initial_allocation_strategy
        self.allocation_granularity_gpus = max(1, int(allocation_granularity_gpus))
        self.min_train_gpus, self.min_rollout_gpus = max(1, int(min_train_gpus)), max(1, int(min_rollout_gpus))
        self.micro_batch_sizes = micro_batch_sizes
        self.max_history_size = max(1, int(max_history_size))
        self.plan_interval = max(1, int(plan_interval))
        self.trigger = ReplanTrigger(bool(online_replanning), self.plan_interval, max(0, int(replan_cooldown_steps)),
                                     float(queue_pressure_threshold), float(active_rollout_pressure_threshold),
                                     int(rejected_rollout_delta_threshold), float(rollout_train_imbalance_threshold))
        self.elastic = ElasticHybridPolicy(bool(elastic_hybrid_planning_enabled),
                                           float(elastic_hybrid_borrow_train_rollout_ratio),
                                           float(elastic_hybrid_release_train_rollout_ratio),
                                           float(elastic_hybrid_max_rollout_pressure),
                                           max(1, int(elastic_hybrid_signal_ttl_steps)))
        self.elastic_hybrid_max_workers = max(0, int(elastic_hybrid_max_workers))
        self.verbose = verbose
        self.optimizer = TwoLevelNestedOptimizer(evaluator, self.allowed_rollout_tp,
                                                 require_heterogeneous_rollout_tp=require_heterogeneous_rollout_tp,
                                                 verbose=verbose)
        self._history: List[RequestInfo] = []
        self._metrics: List[RuntimeResourceMetrics] = []
        self._active_plan: Optional[GlobalResourcePlan] = None
        self._last_decision: Optional[PlannerDecision] = None

    @classmethod
    def from_config(cls, config: AsyncRLConfig, evaluator=None) -> "GlobalResourcePlanner":
        p = config.global_resource_planner
        return cls(evaluator=evaluator or HybridSimulatorCostModel(config),
                   n_total_gpus=config.n_total_gpus or (config.train_gpus + config.rollout_gpus),
                   plan_interval=p.plan_interval, warmup_steps=p.warmup_steps, min_history_size=p.min_history_size,
                   min_gain_ratio=p.min_gain_ratio, reconfiguration_cost_s=p.reconfiguration_cost_s,
                   allowed_rollout_tp=p.allowed_rollout_tp,
                   require_heterogeneous_rollout_tp=p.require_heterogeneous_rollout_tp,
                   allowed_train_tp=p.allowed_train_tp or None, allowed_train_pp=p.allowed_train_pp or None,
                   fixed_train_gpus=p.fixed_train_gpus, initial_allocation_strategy=p.initial_allocation_strategy,
                   allocation_granularity_gpus=p.allocation_granularity_gpus, min_train_gpus=p.min_train_gpus,
                   min_rollout_gpus=p.min_rollout_gpus, micro_batch_sizes=p.micro_batch_sizes or None,
                   max_history_size=p.max_history_size, online_replanning=p.runtime_online_replanning,
                   replan_cooldown_steps=p.runtime_replan_cooldown_steps,
                   queue_pressure_threshold=p.runtime_queue_pressure_threshold,
                   active_rollout_pressure_threshold=p.runtime_active_rollout_pressure_threshold,
                   rejected_rollout_delta_threshold=p.runtime_rejected_rollout_delta_threshold,
                   rollout_train_imbalance_threshold=p.runtime_rollout_train_imbalance_threshold,
                   elastic_hybrid_planning_enabled=p.elastic_hybrid_planning_enabled,
                   elastic_hybrid_max_workers=p.elastic_hybrid_max_workers,
                   elastic_hybrid_borrow_train_rollout_ratio=p.elastic_hybrid_borrow_train_rollout_ratio,
                   elastic_hybrid_release_train_rollout_ratio=p.elastic_hybrid_release_train_rollout_ratio,
                   elastic_hybrid_max_rollout_pressure=p.elastic_hybrid_max_rollout_pressure,
                   elastic_hybrid_signal_ttl_steps=p.elastic_hybrid_signal_ttl_steps, verbose=p.verbose)

    # -------------------------------------------------------------- state
    active_plan = property(lambda self: self._active_plan)
    last_decision = property(lambda self: self._last_decision)
    history_size = property(lambda self: len(self._history))
    latest_runtime_metrics = property(lambda self: self._metrics[-1] if self._metrics else None)

    @staticmethod
    def _extract_requests(items) -> List[RequestInfo]:
        out = []
        for it in items or []:
            if not isinstance(it, dict):
                continue
            try:
                p = int(it.get("input_len", it.get("prompt_length", 0)))
                g = int(it.get("output_len", it.get("gen_length", 0)))
            except (TypeError, ValueError):
                continue
            if p > 0 or g > 0:
                out.append(RequestInfo(max(1, p), max(1, g)))
        return out

    def _trim(self) -> None:
        del self._history[:-self.max_history_size]

    def observe_batch(self, batch) -> int:
        reqs = self._extract_requests(batch)
        self._history.extend(reqs)
        self._trim()
        return len(reqs)

    extend_history = observe_batch

    def replace_history(self, history) -> int:
        self._history = self._extract_requests(history)[-self.max_history_size:]
        return len(self._history)

    def observe_runtime(self, *, step: int, dispatcher_metrics: Optional[dict] = None,
                        step_stats: Optional[dict] = None) -> RuntimeResourceMetrics:
        d, s = dict(dispatcher_metrics or {}), dict(step_stats or {})
        gi = lambda src, k: int(src.get(k, 0) or 0)  # noqa: E731
        queued = gi(d, "pending_inputs") + gi(d, "runner_input_queue") + gi(d, "runner_output_queue")
        cap = max(1, gi(d, "runner_max_queue") + gi(d, "runner_max_queue_size") + gi(d, "staleness_pending_limit"))
        running = gi(d, "staleness_running")
        max_conc = gi(s, "max_concurrent_rollouts")
        if max_conc <= 1:
            max_conc = running + gi(d, "staleness_capacity")
        m = RuntimeResourceMetrics(int(step), queued / cap, running / max(1, max_conc), gi(d, "staleness_accepted"),
                                   gi(d, "staleness_rejected"), float(s.get("rollout_time", 0.0) or 0.0),
                                   float(s.get("train_time", 0.0) or 0.0), float(s.get("step_time", 0.0) or 0.0),
                                   {"dispatcher": d, "step_stats": s})
        self._metrics.append(m)
        del self._metrics[:-self.max_history_size]
        return m

    def _remember(self, d: PlannerDecision) -> PlannerDecision:
        self._last_decision = d
        return d

    # -------------------------------------------------------------- planning
    def _avg_len(self) -> int:
        return int(sum(r.total_length for r in self._history) / len(self._history)) if self._history else 1024

    def _plan(self, tc: TrainParallelConfig, rc: RolloutClusterConfig, config: AsyncRLConfig,
              source: str) -> GlobalResourcePlan:
        tt, td = self.evaluator.evaluate_training(tc, config.batch_size, self._avg_len())
        tr, rd = self.evaluator.evaluate_rollout(rc, list(self._history))
        return GlobalResourcePlan(tc, rc, tt, tr, max(tt, tr), self.n_total_gpus, config.max_concurrent_rollouts,
                                  metadata={"source": source, "training": td, "rollout": rd})

    def _build_current_plan(self, config: AsyncRLConfig, history=None) -> GlobalResourcePlan:
        tc = TrainParallelConfig(tp=max(1, config.train_tp_size), pp=max(1, config.train_pp_size),
                                 dp=max(1, config.train_dp_size), b_micro=max(1, config.micro_batch_size),
                                 cp=max(1, config.train_cp_size))
        tps = config.heterogeneous_rollout.tp_list if config.heterogeneous_rollout.instances else \
            [max(1, config.vllm_tp_size)] * max(1, config.rollout_gpus // max(1, config.vllm_tp_size))
        return self._plan(tc, RolloutClusterConfig(list(tps)), config, "current_config")

    def _forced_train(self, config: AsyncRLConfig, current: GlobalResourcePlan, rollout_gpus: int):
        raw = os.environ.get("GRP_FORCE_TRAIN_GPUS", "").strip()
        if not raw:
            return None
        try:
            n = int(raw)
        except ValueError as exc:
            raise ValueError(f"Invalid GRP_FORCE_TRAIN_GPUS={raw!r}") from exc
        if n <= 0:
            raise ValueError(f"GRP_FORCE_TRAIN_GPUS must be positive: {n}")
        if n + rollout_gpus > self.n_total_gpus:
            raise ValueError(f"GRP_FORCE_TRAIN_GPUS plus rollout_gpus must fit n_total_gpus={self.n_total_gpus}, "
                             f"got train={n} rollout={rollout_gpus}")
        c = current.train_config
        width = c.tp * c.pp * max(1, config.train_cp_size)
        if n % width:
            raise ValueError(f"GRP_FORCE_TRAIN_GPUS must be divisible by train TP*PP*CP={width}, got {n}")
        return TrainParallelConfig(tp=c.tp, pp=c.pp, cp=max(1, config.train_cp_size), dp=n // width,
                                   b_micro=c.b_micro, zero_level=c.zero_level)

    def _forced_rollout(self, config: AsyncRLConfig) -> Optional[List[int]]:
        tps = _env_ints("GRP_FORCE_ROLLOUT_TP_LIST")
        if not tps:
            return None
        if any(t <= 0 for t in tps):
            raise ValueError(f"GRP_FORCE_ROLLOUT_TP_LIST must be positive: {tps}")
        forced_train = _env_ints("GRP_FORCE_TRAIN_GPUS")
        budget = self.n_total_gpus - forced_train[0] if forced_train else int(config.rollout_gpus or sum(tps))
        if sum(tps) != budget:
            raise ValueError(f"GRP_FORCE_ROLLOUT_TP_LIST must sum to rollout_gpus={budget}, got {tps}")
        return tps

    def plan_if_needed(self, step: int, config: AsyncRLConfig, batch=None,
                       runtime_metrics: Optional[RuntimeResourceMetrics] = None) -> PlannerDecision:
        if batch is not None:
            self.observe_batch(batch)
        m = runtime_metrics if runtime_metrics is not None else self.latest_runtime_metrics
        base = dict(num_requests=len(self._history), runtime_metrics=m)
        if step < self.warmup_steps:
            return self._remember(PlannerDecision(step, False, "warmup", trigger="warmup", **base))
        trig = self.trigger(step, m)
        if trig in ("cooldown", "interval_skip"):
            return self._remember(PlannerDecision(step, False, trig, current_plan=self._active_plan, trigger=trig,
                                                  **base))
        if len(self._history) < self.min_history_size:
            return self._remember(PlannerDecision(step, False, "insufficient_history", current_plan=self._active_plan,
                                                  trigger=trig, **base))
        current = self._build_current_plan(config)
        result = self.optimizer.optimize(
            n_total_gpus=self.n_total_gpus, requests=list(self._history), B_global=config.batch_size,
            allowed_train_tp=self.allowed_train_tp, allowed_train_pp=self.allowed_train_pp,
            micro_batch_sizes=self.micro_batch_sizes,
            fixed_train_gpus=0 if self.initial_allocation_strategy == "grp" else self.fixed_train_gpus,
            allocation_granularity_gpus=self.allocation_granularity_gpus, min_train_gpus=self.min_train_gpus,
            min_rollout_gpus=self.min_rollout_gpus,
            rollout_node_tp_pattern=list(config.global_resource_planner.rollout_node_tp_pattern or []),
            train_cp_size=max(1, config.train_cp_size), dp_batch_group_size=max(1, config.n_samples))
        if result.train_config is None or result.rollout_config is None:
            self.trigger.observed(trig, m)
            return self._remember(PlannerDecision(step, False, "no_feasible_candidate", current_plan=current,
                                                  optimization_result=result, trigger=trig, **base))
        candidate = GlobalResourcePlan(result.train_config, result.rollout_config, result.t_train, result.t_rollout,
                                       result.t_global, self.n_total_gpus, config.max_concurrent_rollouts,
                                       metadata={"source": "optimizer"})
        forced_tps = self._forced_rollout(config)
        forced_tc = self._forced_train(config, current, sum(forced_tps) if forced_tps else int(config.rollout_gpus))
        forced = forced_tps is not None or forced_tc is not None
        if forced:
            rc = RolloutClusterConfig(forced_tps) if forced_tps is not None else current.rollout_config
            candidate = self._plan(forced_tc or current.train_config, rc, config,
                                   "forced_runtime_train_and_rollout" if forced_tps is not None and forced_tc is not None
                                   else "forced_runtime_rollout_tp" if forced_tps is not None
                                   else "forced_runtime_train_gpus")
        raw_gain = current.t_global - candidate.t_global
        candidate.expected_gain_s = raw_gain - self.reconfiguration_cost_s
        candidate.expected_gain_ratio = raw_gain / max(current.t_global, 1e-6)
        candidate.reconfiguration_cost_s = self.reconfiguration_cost_s
        same = (candidate.train_config.tp, candidate.train_config.pp, candidate.train_config.dp,
                sorted(candidate.rollout_tp_list)) == (current.train_config.tp, current.train_config.pp,
                                                       current.train_config.dp, sorted(current.rollout_tp_list))
        ehp = self.elastic.signal(step, config, current, candidate, m)
        ehp_adjust = bool(ehp is not None and ehp.should_adjust)
        force_all = os.environ.get("GRP_FORCE_RUNTIME_RECONFIGURE", "0") == "1"
        worth = candidate.expected_gain_s > 0.0 and candidate.expected_gain_ratio >= self.min_gain_ratio
        resource = (not same or force_all) and (forced or force_all or worth)
        should = resource or ehp_adjust
        if ehp_adjust:
            reason = "elastic_hybrid_adjustment"
        elif should and forced:
            reason = "forced_reconfigure"
        elif should and force_all:
            reason = "forced_runtime_reconfigure"
        elif should:
            reason = "reconfigure"
        else:
            reason = "same_plan" if same else "gain_below_threshold"
        decision = PlannerDecision(step, should, reason, current, candidate, result, trigger=trig,
                                   elastic_hybrid_signal=ehp, **base)
        if should:
            self._active_plan = candidate
            self.trigger.last_replan_step = int(step)
        elif self._active_plan is None:
            self._active_plan = current
        self.trigger.observed(trig, m)
        return self._remember(decision)

    # -------------------------------------------------------------- applying
    def apply_plan_to_config(self, plan: GlobalResourcePlan, config: AsyncRLConfig) -> None:
        t = plan.train_config
        config.n_total_gpus = plan.n_total_gpus
        config.train_gpus, config.rollout_gpus = plan.train_gpus, plan.rollout_gpus
        config.train_tp_size = config.tp_size = t.tp
        config.train_pp_size, config.train_cp_size, config.train_dp_size = t.pp, t.cp, t.dp
        config.micro_batch_size = t.b_micro
        config.max_concurrent_rollouts = plan.max_concurrent_rollouts
        h = config.heterogeneous_rollout
        h.enabled = True
        h.total_gpus = plan.rollout_gpus
        pools = self._host_pools(config, plan.rollout_gpus)
        h.available_gpus = sorted({g for _, gs in pools for g in gs})
        instances = []
        for i, tp in enumerate(plan.rollout_tp_list):
            host, gpus = self._take(pools, tp)
            instances.append(HeterogeneousInstanceConfig(instance_id=f"grp_tp{tp}_{i}", tp=tp, gpus=gpus,
                                                         host=host or h.vllm_host, port=int(h.vllm_base_port) + i,
                                                         description="managed_by_global_resource_planner"))
        h.instances = instances

    @staticmethod
    def _host_pools(config: AsyncRLConfig, rollout_gpus: int) -> List[Tuple[str, List[int]]]:
        """GPU ids available to rollout instances.

        Single box: the training pool occupies GPUs [0, train_gpus) and the
        rollout pool the next ``rollout_gpus`` ids, unless ``available_gpus``
        lists enough ids explicitly.  Instances spread over several hosts keep
        one pool per host.
        """
        h = config.heterogeneous_rollout
        hosts = {inst.host or h.vllm_host for inst in h.instances}
        if len(hosts) > 1:
            pools: Dict[str, List[int]] = {}
            for inst in h.instances:
                pools.setdefault(inst.host or h.vllm_host, []).extend(int(g) for g in inst.gpus)
            return [(host, sorted(set(gs))) for host, gs in pools.items()]
        if len(h.available_gpus) >= rollout_gpus and not set(h.available_gpus) & set(range(config.train_gpus)):
            return [(h.vllm_host, sorted(h.available_gpus))]
        return [(h.vllm_host, list(range(config.train_gpus, config.train_gpus + rollout_gpus)))]

    @staticmethod
    def _take(pools: List[Tuple[str, List[int]]], tp: int) -> Tuple[str, List[int]]:
        for i, (host, gpus) in enumerate(pools):
            if len(gpus) >= tp:
                pools[i] = (host, gpus[tp:])
                return host, gpus[:tp]
        return (pools[0][0] if pools else ""), list(range(tp))
