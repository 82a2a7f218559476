"""Baseline rollout schedulers: load balance, length-aware and LA-MLFQ.

* ``LoadBalanceScheduler`` (reference ``infra/scheduling/load_balance.py``):
  round robin, weighted (active / TP weight) or least-connections with a
  rotating tie-break so equally loaded endpoints are used in turn.
* ``LengthAwareScheduler`` (reference ``infra/scheduling/length_aware.py``):
  input length -> short/medium/long/extra_long -> preferred TP list, then
  fallback TP list, then the globally least-loaded instance.
* ``LAMLFQScheduler`` (reference ``infra/scheduling/la_mlfq.py``): per-prompt
  history table with epoch TTL; for n_samples > 1 the first sample of a prompt
  is a *scout* in the short bucket and the other samples wait (``pending``)
  until the scout migrates (token threshold exceeded) or finishes; the waiting
  samples then follow the scout's bucket.
"""

from __future__ import annotations

import asyncio
import logging
import threading
import time
from collections import defaultdict
from dataclasses import dataclass, field
from enum import Enum
from typing import Any, Dict, List, Optional

from libra_b200.infra.scheduling.base import (BaseScheduler, InstanceHandle, LoadBalanceStrategy, RoutingRule,
                                              SchedulingResult)

log = logging.getLogger(__name__)


# ============================================================================ load balance
class LoadBalanceScheduler(BaseScheduler):
    def __init__(self, load_balance_strategy: str = "least_connections", max_queue_length: int = 100,
                 weights: Optional[Dict[int, float]] = None):
        super().__init__(name="LoadBalance")
        self._strategy = LoadBalanceStrategy.parse(load_balance_strategy, allow_weighted=True)
        self._max_queue_length = max_queue_length
        self._weights = weights or {}
        self._cursor = 0

    def _choose(self, cands: List[InstanceHandle]) -> InstanceHandle:
        if self._strategy == LoadBalanceStrategy.ROUND_ROBIN:
            h = cands[self._cursor % len(cands)]
            self._cursor += 1
            return h
        if self._strategy == LoadBalanceStrategy.WEIGHTED:
            return min(cands, key=lambda h: h.active_requests / max(self._weights.get(h.tp_degree, 1.0), 0.01))
        # least connections; among ties continue after the previously chosen position
        low = min(h.active_requests for h in cands)
        tied = {id(h) for h in cands if h.active_requests == low}
        n = len(self._instances)
        for step in range(n):
            pos = (self._cursor + step) % n
            if id(self._instances[pos]) in tied:
                self._cursor = (pos + 1) % n
                return self._instances[pos]
        raise RuntimeError("least-connections tie set is inconsistent")

    def schedule(self, input_tokens: int, prompt_id: str = "", n_samples: int = 1, epoch: int = -1) -> SchedulingResult:
        with self._lock:
            self._stats.total_requests += 1
            ready = [h for h in self._instances if h.is_ready]
            cands = [h for h in ready if self._max_queue_length <= 0 or h.active_requests < self._max_queue_length]
            cands = cands or ready
            if not cands:
                self._stats.failed_routes += 1
                return SchedulingResult(-1, 0, "any", False, "no_available_instance", prompt_id=prompt_id)
            h = self._choose(cands)
            self._stats.preferred_routes += 1
            self._stats.category_counts["any"] += 1
            self._stats.category_tp_counts["any"][h.tp_degree] += 1
            h.inc_active()
            return SchedulingResult(h.index, h.tp_degree, "any", False, prompt_id=prompt_id)

    @classmethod
    def from_config(cls, hetero_config: Any) -> "LoadBalanceScheduler":
        s = hetero_config.scheduling
        return cls(load_balance_strategy=s.load_balance_strategy, max_queue_length=s.max_queue_length)


# ============================================================================ length aware
class LengthAwareScheduler(BaseScheduler):
    DEFAULT_ROUTING_RULES = {
        "short": ([1, 2], [4, 8]),
        "medium": ([2, 4], [1, 8]),
        "long": ([4, 8], [2, 1]),
        "extra_long": ([8, 4], [2, 1]),
    }

    def __init__(self, routing_rules: Optional[Dict[str, List[int]]] = None,
                 length_thresholds: Optional[Dict[str, int]] = None, load_balance_strategy: str = "least_connections",
                 max_queue_length: int = 100, enable_fallback: bool = True):
        super().__init__(name="LengthAware")
        self._rules = {c: RoutingRule(c, list(p), list(f)) for c, (p, f) in self.DEFAULT_ROUTING_RULES.items()}
        for cat, tps in (routing_rules or {}).items():
            if cat in self._rules:
                self._rules[cat].preferred_tp_degrees = list(tps)
            else:
                self._rules[cat] = RoutingRule(cat, list(tps), [])
        self._thresholds = length_thresholds or {"short": 5000, "medium": 10000, "long": 15000}
        self._strategy = LoadBalanceStrategy.parse(load_balance_strategy)
        self._max_queue_length = max_queue_length
        self._enable_fallback = enable_fallback
        self._perf_history: Dict[tuple, List[float]] = defaultdict(list)

    def categorize(self, input_tokens: int) -> str:
        for cat in ("short", "medium", "long"):
            if input_tokens <= self._thresholds.get(cat, {"short": 5000, "medium": 10000, "long": 15000}[cat]):
                return cat
        return "extra_long"

    def schedule(self, input_tokens: int, prompt_id: str = "", n_samples: int = 1, epoch: int = -1) -> SchedulingResult:
        cat = self.categorize(input_tokens)
        rule = self._rules.get(cat, self._rules["medium"])
        with self._lock:
            self._stats.total_requests += 1
        return self._route(cat, rule.preferred_tp_degrees, rule.fallback_tp_degrees, prompt_id)

    def record_latency(self, category: str, tp_degree: int, latency: float) -> None:
        hist = self._perf_history[(category, tp_degree)]
        hist.append(latency)
        del hist[:-200]

    def reset_stats(self) -> None:
        super().reset_stats()
        self._perf_history.clear()

    @classmethod
    def from_config(cls, hetero_config: Any) -> "LengthAwareScheduler":
        s = hetero_config.scheduling
        return cls(routing_rules=s.routing_rules if isinstance(s.routing_rules, dict) else {},
                   length_thresholds=s.length_thresholds if isinstance(s.length_thresholds, dict) else {},
                   load_balance_strategy=s.load_balance_strategy, max_queue_length=s.max_queue_length,
                   enable_fallback=s.enable_fallback)


# ============================================================================ LA-MLFQ
class ScoutStatus(Enum):
    RUNNING = "running"
    MIGRATED = "migrated"
    COMPLETED = "completed"


@dataclass
class ScoutState:
    prompt_id: str
    instance_index: int
    initial_bucket: str
    current_bucket: str
    status: ScoutStatus = ScoutStatus.RUNNING
    created_at: float = field(default_factory=time.time)
    generated_tokens: int = 0


@dataclass
class WaitingRequest:
    prompt_id: str
    input_tokens: int
    n_samples: int
    epoch: int
    sample_index: int
    created_at: float = field(default_factory=time.time)
    future: Optional[asyncio.Future] = None


@dataclass
class MigrationDecision:
    should_migrate: bool
    reason: str
    current_bucket: str
    target_bucket: str = ""
    generated_tokens: int = 0


@dataclass
class RequestMigrationState:
    request_id: str
    prompt_id: str
    instance_index: int
    current_bucket: str
    generated_tokens: int = 0
    is_scout: bool = False


class HistoryTable:
    """prompt_id -> (final bucket, epoch) with an epoch TTL."""

    def __init__(self, ttl_epochs: int = 5):
        self._table: Dict[str, dict] = {}
        self._ttl = ttl_epochs
        self._lock = threading.Lock()

    def _expired(self, entry: dict, epoch: int) -> bool:
        return epoch >= 0 and self._ttl > 0 and epoch - entry["epoch"] > self._ttl

    def lookup(self, prompt_id: str, current_epoch: int = -1) -> Optional[str]:
        with self._lock:
            e = self._table.get(prompt_id)
            if e is None:
                return None
            if self._expired(e, current_epoch):
                del self._table[prompt_id]
                return None
            return e["bucket"]

    def update(self, prompt_id: str, bucket: str, epoch: int = -1) -> None:
        with self._lock:
            self._table[prompt_id] = {"bucket": bucket, "epoch": epoch}

    def on_epoch_end(self, epoch: int) -> None:
        if self._ttl <= 0:
            return
        with self._lock:
            for pid in [p for p, e in self._table.items() if epoch - e["epoch"] > self._ttl]:
                del self._table[pid]

    @property
    def size(self) -> int:
        return len(self._table)


class ScoutManager:
    def __init__(self, scout_timeout: float = 30.0):
        self._scouts: Dict[str, ScoutState] = {}
        self._waiting: Dict[str, List[WaitingRequest]] = defaultdict(list)
        self._timeout = scout_timeout
        self._lock = threading.Lock()

    def should_scout(self, prompt_id: str) -> bool:
        with self._lock:
            return prompt_id not in self._scouts

    def register_scout(self, prompt_id: str, instance_index: int, bucket: str) -> None:
        with self._lock:
            self._scouts[prompt_id] = ScoutState(prompt_id, instance_index, bucket, bucket)

    def add_waiting(self, waiting: WaitingRequest) -> None:
        with self._lock:
            self._waiting[waiting.prompt_id].append(waiting)

    def is_scout(self, prompt_id: str, instance_index: int) -> bool:
        with self._lock:
            s = self._scouts.get(prompt_id)
            return s is not None and s.instance_index == instance_index

    def _settle(self, prompt_id: str, bucket: str, status: ScoutStatus) -> List[WaitingRequest]:
        with self._lock:
            s = self._scouts.get(prompt_id)
            if s is None:
                return []
            s.current_bucket, s.status = bucket, status
            return self._waiting.pop(prompt_id, [])

    def on_scout_migrated(self, prompt_id: str, new_bucket: str) -> List[WaitingRequest]:
        return self._settle(prompt_id, new_bucket, ScoutStatus.MIGRATED)

    def on_scout_completed(self, prompt_id: str, final_bucket: str) -> List[WaitingRequest]:
        return self._settle(prompt_id, final_bucket, ScoutStatus.COMPLETED)

    def get_scout_bucket(self, prompt_id: str) -> Optional[str]:
        with self._lock:
            s = self._scouts.get(prompt_id)
            return s.current_bucket if s else None

    def get_scout_status(self, prompt_id: str) -> Optional[ScoutStatus]:
        with self._lock:
            s = self._scouts.get(prompt_id)
            return s.status if s else None

    def check_timeouts(self) -> List[str]:
        now = time.time()
        with self._lock:
            return [p for p, s in self._scouts.items()
                    if s.status == ScoutStatus.RUNNING and now - s.created_at > self._timeout]

    def force_release(self, prompt_id: str) -> List[WaitingRequest]:
        with self._lock:
            waiting = self._waiting.pop(prompt_id, [])
            s = self._scouts.get(prompt_id)
            if s:
                s.status = ScoutStatus.COMPLETED
        return waiting

    def reset(self) -> None:
        with self._lock:
            self._scouts.clear()
            self._waiting.clear()

    @property
    def active_scouts(self) -> int:
        with self._lock:
            return sum(s.status == ScoutStatus.RUNNING for s in self._scouts.values())

    @property
    def total_waiting(self) -> int:
        with self._lock:
            return sum(len(w) for w in self._waiting.values())


class MigrationController:
    """Demote a request to the long bucket once it generated more tokens than
    its bucket's threshold."""

    def __init__(self, bucket_thresholds: Optional[Dict[str, int]] = None):
        self._thresholds = bucket_thresholds or {"short": 3000, "medium": 10000}
        self._demote = {"short": "long", "medium": "long"}
        self._active: Dict[str, RequestMigrationState] = {}
        self._lock = threading.Lock()
        self._migrations = 0
        self._checks = 0

    def register_request(self, request_id: str, prompt_id: str, instance_index: int, bucket: str,
                         is_scout: bool = False) -> None:
        with self._lock:
            self._active[request_id] = RequestMigrationState(request_id, prompt_id, instance_index, bucket,
                                                             is_scout=is_scout)

    def check_migration(self, request_id: str, generated_tokens: int) -> MigrationDecision:
        self._checks += 1
        with self._lock:
            st = self._active.get(request_id)
            if st is None:
                return MigrationDecision(False, "request_not_tracked", "unknown")
            st.generated_tokens = generated_tokens
        limit = self._thresholds.get(st.current_bucket)
        if limit is None:
            return MigrationDecision(False, "no_threshold_for_bucket", st.current_bucket)
        if generated_tokens <= limit:
            return MigrationDecision(False, "below_threshold", st.current_bucket, generated_tokens=generated_tokens)
        return MigrationDecision(True, "threshold_exceeded", st.current_bucket,
                                 self._demote.get(st.current_bucket, "long"), generated_tokens)

    def on_migration_executed(self, request_id: str, new_bucket: str) -> None:
        with self._lock:
            st = self._active.get(request_id)
            if st:
                st.current_bucket = new_bucket
                self._migrations += 1

    def on_request_done(self, request_id: str) -> None:
        with self._lock:
            self._active.pop(request_id, None)

    def get_request_state(self, request_id: str) -> Optional[RequestMigrationState]:
        with self._lock:
            return self._active.get(request_id)

    def get_stats(self) -> dict:
        return {"active_tracked": len(self._active), "total_migrations": self._migrations,
                "total_checks": self._checks}

    def reset(self) -> None:
        with self._lock:
            self._active.clear()
            self._migrations = self._checks = 0


class LAMLFQScheduler(BaseScheduler):
    DEFAULT_BUCKETS = {
        "short": {"tp_degrees": [1, 2], "max_tokens": 5000},
        "long": {"tp_degrees": [4, 8], "max_tokens": 50000},
    }

    def __init__(self, buckets: Optional[Dict[str, dict]] = None, length_thresholds: Optional[Dict[str, int]] = None,
                 migration_threshold: int = 3000, scout_timeout: float = 30.0, history_ttl: int = 5,
                 load_balance_strategy: str = "least_connections", max_queue_length: int = 100,
                 enable_fallback: bool = True):
        super().__init__(name="LA-MLFQ")
        self._buckets = dict(buckets or self.DEFAULT_BUCKETS)
        self._bucket_rules = {
            n: RoutingRule(n, list(c.get("tp_degrees", [1, 2])),
                           [tp for o, oc in self._buckets.items() if o != n for tp in oc.get("tp_degrees", [])])
            for n, c in self._buckets.items()}
        self._thresholds = length_thresholds or {"short": 5000, "medium": 10000, "long": 15000}
        self._strategy = LoadBalanceStrategy.parse(load_balance_strategy)
        self._max_queue_length = max_queue_length
        self._enable_fallback = enable_fallback
        self.migration_threshold = migration_threshold
        self.history_table = HistoryTable(history_ttl)
        self.scout_manager = ScoutManager(scout_timeout)
        self.migration_controller = MigrationController(
            {n: c.get("max_tokens", 5000) for n, c in self._buckets.items() if n not in ("long", "extra_long")})
        self._current_epoch = -1

    def _route_to_bucket(self, bucket: str, input_tokens: int, prompt_id: str = "", reason: str = "") -> SchedulingResult:
        rule = self._bucket_rules.get(bucket)
        if rule is None:
            return self._default_length_route(input_tokens, prompt_id)
        return self._route(bucket, rule.preferred_tp_degrees, rule.fallback_tp_degrees, prompt_id, reason)

    def _default_length_route(self, input_tokens: int, prompt_id: str = "") -> SchedulingResult:
        bucket = "short" if input_tokens <= self._thresholds.get("short", 5000) else "long"
        return self._route_to_bucket(bucket, input_tokens, prompt_id, "default")

    def schedule(self, input_tokens: int, prompt_id: str = "", n_samples: int = 1, epoch: int = -1) -> SchedulingResult:
        if epoch >= 0:
            self._current_epoch = epoch
        with self._lock:
            self._stats.total_requests += 1
        if not prompt_id:
            return self._default_length_route(input_tokens, prompt_id)
        remembered = self.history_table.lookup(prompt_id, self._current_epoch)
        if remembered:
            res = self._route_to_bucket(remembered, input_tokens, prompt_id, "history_hit")
            if res.instance_index >= 0:
                return res
        if n_samples <= 1:
            return self._default_length_route(input_tokens, prompt_id)
        if self.scout_manager.should_scout(prompt_id):
            res = self._route_to_bucket("short", input_tokens, prompt_id, "scout")
            if res.instance_index < 0:
                return self._default_length_route(input_tokens, prompt_id)
            self.scout_manager.register_scout(prompt_id, res.instance_index, "short")
            self.migration_controller.register_request(f"{prompt_id}_scout", prompt_id, res.instance_index, "short",
                                                       is_scout=True)
            return res
        if self.scout_manager.get_scout_status(prompt_id) in (ScoutStatus.MIGRATED, ScoutStatus.COMPLETED):
            target = self.scout_manager.get_scout_bucket(prompt_id)
            if target:
                return self._route_to_bucket(target, input_tokens, prompt_id, "scout_follow")
        with self._lock:
            self._stats.pending_routes += 1
        return SchedulingResult(-1, 0, "pending", False, "waiting_for_scout", pending=True, prompt_id=prompt_id)

    def on_request_done(self, instance_index: int, prompt_id: str = "", final_bucket: str = "",
                        output_tokens: int = 0) -> None:
        self._release(instance_index)
        if prompt_id and final_bucket:
            self.history_table.update(prompt_id, final_bucket, self._current_epoch)
        if prompt_id and self.scout_manager.is_scout(prompt_id, instance_index):
            bucket = final_bucket or self.scout_manager.get_scout_bucket(prompt_id) or "short"
            self._release_waiters(self.scout_manager.on_scout_completed(prompt_id, bucket), bucket)
        if prompt_id:
            self.migration_controller.on_request_done(f"{prompt_id}_scout")

    def check_and_migrate(self, request_id: str, generated_tokens: int) -> MigrationDecision:
        d = self.migration_controller.check_migration(request_id, generated_tokens)
        if d.should_migrate:
            self.migration_controller.on_migration_executed(request_id, d.target_bucket)
            with self._lock:
                self._stats.migrated_routes += 1
            st = self.migration_controller.get_request_state(request_id)
            if st and st.is_scout:
                self._release_waiters(self.scout_manager.on_scout_migrated(st.prompt_id, d.target_bucket),
                                      d.target_bucket)
        return d

    def _release_waiters(self, waiting: List[WaitingRequest], bucket: str) -> None:
        for w in waiting:
            res = self._route_to_bucket(bucket, w.input_tokens, w.prompt_id, "scout_released")
            if w.future is not None and not w.future.done():
                w.future.set_result(res)

    def on_epoch_start(self, epoch: int) -> None:
        self._current_epoch = epoch

    def on_epoch_end(self, epoch: int) -> None:
        self.history_table.on_epoch_end(epoch)
        for pid in self.scout_manager.check_timeouts():
            for w in self.scout_manager.force_release(pid):
                res = self._default_length_route(w.input_tokens, w.prompt_id)
                if w.future is not None and not w.future.done():
                    w.future.set_result(res)
        self.scout_manager.reset()
        self.migration_controller.reset()

    def print_stats(self) -> None:
        super().print_stats()
        print(f"  [LA-MLFQ] history={self.history_table.size} scouts={self.scout_manager.active_scouts} "
              f"waiting={self.scout_manager.total_waiting} migration={self.migration_controller.get_stats()}")

    @classmethod
    def from_config(cls, hetero_config: Any) -> "LAMLFQScheduler":
        s = hetero_config.scheduling
        return cls(buckets=getattr(s, "la_mlfq_buckets", None) or cls.DEFAULT_BUCKETS,
                   length_thresholds=s.length_thresholds if isinstance(s.length_thresholds, dict) else {},
                   migration_threshold=getattr(s, "la_mlfq_migration_threshold", 3000),
                   scout_timeout=getattr(s, "la_mlfq_scout_timeout", 30.0),
                   history_ttl=getattr(s, "la_mlfq_history_ttl", 5),
                   load_balance_strategy=s.load_balance_strategy, max_queue_length=s.max_queue_length,
                   enable_fallback=s.enable_fallback)
