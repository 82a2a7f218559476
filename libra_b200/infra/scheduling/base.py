"""Scheduler base types and the shared instance-selection logic.

Types and hooks mirror the reference (``infra/scheduling/base.py``):
``SchedulingResult`` (instance, tp, category, fallback flag, pending flag,
request id), ``InstanceHandle`` with an active-request counter and
``BaseScheduler`` with ``register_instance / schedule / on_request_done`` and
epoch hooks.  All schedulers here route through one helper,
``BaseScheduler._route``, which implements the common cascade:

    preferred TP degrees -> fallback TP degrees -> least-loaded ready instance

with per-TP round-robin or least-connections selection and a per-instance
queue cap.
"""

from __future__ import annotations

import logging
import threading
from abc import ABC, abstractmethod
from collections import defaultdict
from dataclasses import dataclass, field
from enum import Enum
from typing import Any, Callable, Dict, List, Optional, Sequence

log = logging.getLogger(__name__)


class LoadBalanceStrategy(Enum):
    ROUND_ROBIN = "round_robin"
    LEAST_CONNECTIONS = "least_connections"
    WEIGHTED = "weighted"

    @classmethod
    def parse(cls, name: str, allow_weighted: bool = False) -> "LoadBalanceStrategy":
        if name == "round_robin":
            return cls.ROUND_ROBIN
        if name == "weighted" and allow_weighted:
            return cls.WEIGHTED
        return cls.LEAST_CONNECTIONS


@dataclass
class RoutingRule:
    category: str
    preferred_tp_degrees: List[int]
    fallback_tp_degrees: List[int] = field(default_factory=list)


@dataclass
class SchedulingResult:
    instance_index: int
    tp_degree: int
    category: str
    is_fallback: bool
    reason: str = ""
    pending: bool = False
    prompt_id: str = ""
    request_id: str = ""


def _nested_counter():
    return defaultdict(int)


@dataclass
class SchedulerStats:
    total_requests: int = 0
    preferred_routes: int = 0
    fallback_routes: int = 0
    failed_routes: int = 0
    pending_routes: int = 0
    migrated_routes: int = 0
    category_counts: dict = field(default_factory=lambda: defaultdict(int))
    category_tp_counts: dict = field(default_factory=lambda: defaultdict(_nested_counter))

    @property
    def success_rate(self) -> float:
        if not self.total_requests:
            return 1.0
        return (self.preferred_routes + self.fallback_routes) / self.total_requests

    def to_dict(self) -> dict:
        return {
            "total_requests": self.total_requests, "preferred_routes": self.preferred_routes,
            "fallback_routes": self.fallback_routes, "failed_routes": self.failed_routes,
            "pending_routes": self.pending_routes, "migrated_routes": self.migrated_routes,
            "success_rate": self.success_rate, "category_counts": dict(self.category_counts),
            "category_tp_counts": {c: dict(v) for c, v in self.category_tp_counts.items()},
        }


@dataclass
class InstanceHandle:
    index: int
    instance_id: str
    tp_degree: int
    is_ready: bool = True
    active_requests: int = 0

    def inc_active(self):
        self.active_requests += 1

    def dec_active(self):
        self.active_requests = max(0, self.active_requests - 1)


class BaseScheduler(ABC):
    def __init__(self, name: str = "base"):
        self.name = name
        self._instances: List[InstanceHandle] = []
        self._instances_by_tp: Dict[int, List[InstanceHandle]] = defaultdict(list)
        self._lock = threading.Lock()
        self._stats = SchedulerStats()
        self._rr_cursor: Dict[int, int] = defaultdict(int)
        self._strategy = LoadBalanceStrategy.LEAST_CONNECTIONS
        self._max_queue_length = 0
        self._enable_fallback = True

    # -------------------------------------------------------------- instances
    def register_instance(self, index: int, instance_id: str, tp_degree: int) -> None:
        handle = InstanceHandle(index=index, instance_id=instance_id, tp_degree=tp_degree)
        self._instances.append(handle)
        self._instances_by_tp[tp_degree].append(handle)
        log.info("[%s] registered %s index=%d TP=%d", self.name, instance_id, index, tp_degree)

    def get_instance_handle(self, index: int) -> Optional[InstanceHandle]:
        return next((h for h in self._instances if h.index == index), None)

    # -------------------------------------------------------------- selection
    def _load(self, handle: InstanceHandle) -> int:
        """Active-request count used for least-connections (overridable)."""
        return handle.active_requests

    def _pick_in_tp(self, tp: int, load: Callable[[InstanceHandle], int]) -> Optional[InstanceHandle]:
        cands = [h for h in self._instances_by_tp.get(tp, []) if h.is_ready]
        if self._max_queue_length > 0:
            cands = [h for h in cands if load(h) < self._max_queue_length]
        if not cands:
            return None
        if self._strategy == LoadBalanceStrategy.ROUND_ROBIN:
            i = self._rr_cursor[tp] % len(cands)
            self._rr_cursor[tp] = i + 1
            return cands[i]
        return min(cands, key=load)

    def _pick(self, tps: Sequence[int], load: Callable[[InstanceHandle], int]) -> Optional[InstanceHandle]:
        for tp in tps:
            h = self._pick_in_tp(tp, load)
            if h is not None:
                return h
        return None

    def _on_selected(self, handle: InstanceHandle) -> None:
        handle.inc_active()

    def _route(self, category: str, preferred: Sequence[int], fallback: Sequence[int], prompt_id: str = "",
               reason: str = "", load: Optional[Callable[[InstanceHandle], int]] = None) -> SchedulingResult:
        """preferred -> fallback -> global least-loaded; updates stats and counters."""
        load = load or self._load
        with self._lock:
            self._stats.category_counts[category] += 1
            chosen, is_fb, why = self._pick(preferred, load), False, reason
            if chosen is None and self._enable_fallback and fallback:
                chosen, is_fb = self._pick(fallback, load), True
                why = f"{reason}_fallback" if reason else ""
            if chosen is None:
                ready = [h for h in self._instances if h.is_ready]
                if ready:
                    chosen, is_fb, why = min(ready, key=load), True, "global_fallback"
            if chosen is None:
                self._stats.failed_routes += 1
                return SchedulingResult(-1, 0, category, False, "no_available_instance", prompt_id=prompt_id)
            if is_fb:
                self._stats.fallback_routes += 1
            else:
                self._stats.preferred_routes += 1
            self._stats.category_tp_counts[category][chosen.tp_degree] += 1
            self._on_selected(chosen)
            return SchedulingResult(chosen.index, chosen.tp_degree, category, is_fb, why, prompt_id=prompt_id)

    def _release(self, index: int) -> None:
        h = self.get_instance_handle(index)
        if h is not None:
            with self._lock:
                self._on_released(h)

    def _on_released(self, handle: InstanceHandle) -> None:
        handle.dec_active()

    # -------------------------------------------------------------- hooks
    @abstractmethod
    def schedule(self, input_tokens: int, prompt_id: str = "", n_samples: int = 1, epoch: int = -1) -> SchedulingResult:
        ...

    def on_request_done(self, instance_index: int, prompt_id: str = "", final_bucket: str = "",
                        output_tokens: int = 0) -> None:
        self._release(instance_index)

    def on_epoch_start(self, epoch: int) -> None:
        pass

    def on_epoch_end(self, epoch: int) -> None:
        pass

    def get_stats(self) -> SchedulerStats:
        return self._stats

    def reset_stats(self) -> None:
        self._stats = SchedulerStats()

    def print_stats(self) -> None:
        s = self._stats.to_dict()
        print(f"\n{self.name} scheduler: " + ", ".join(f"{k}={v}" for k, v in s.items() if not isinstance(v, dict)))
        for cat, per_tp in sorted(s["category_tp_counts"].items()):
            for tp, n in sorted(per_tp.items()):
                print(f"  {cat} -> TP={tp}: {n}")
        for h in self._instances:
            print(f"  {h.instance_id}: TP={h.tp_degree}, active={h.active_requests}, ready={h.is_ready}")

    @classmethod
    def from_config(cls, hetero_config: Any) -> "BaseScheduler":
        raise NotImplementedError(f"{cls.__name__} does not implement from_config(); use SchedulerFactory.create()")
