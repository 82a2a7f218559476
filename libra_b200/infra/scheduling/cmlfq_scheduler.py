"""C-MLFQ: causality-aware multi-level feedback queue over TP buckets.

Policy (reference ``infra/scheduling/cmlfq_scheduler.py``):

1. A new request always starts in the **shortest** bucket (lowest
   ``max_tokens``), e.g. the TP-1/TP-2 bucket.
2. On every tool return the request's tool-return state is appended to its
   path; the causal prefix tree is queried (prompt tree, else global tree) and
   both the node's mean and p90 remaining length are mapped to a bucket.  The
   request migrates only if the two agree **and** differ from its current
   bucket.
3. When the request finishes, the exact remaining output length after each
   tool return is inserted into the tree, which is periodically rebuilt from
   the most recent trajectories and persisted per rank.

Routing inside a bucket uses the shared cascade in ``BaseScheduler._route``;
when ``cmlfq_shared_load_dir`` is set, least-connections uses the active
counts summed over all trainer ranks.
"""

from __future__ import annotations

import logging
import os
import time
import uuid
from dataclasses import dataclass, field
from pathlib import Path
from typing import Any, Dict, List, Optional

from libra_b200.infra.scheduling.base import BaseScheduler, InstanceHandle, LoadBalanceStrategy, SchedulingResult
from libra_b200.infra.scheduling.cmlfq_prefix_tree import CausalPrefixTree, PrefixTreeNode, Trajectory
from libra_b200.infra.scheduling.cmlfq_shared_state import SharedCMLFQLoadState
from libra_b200.infra.scheduling.cmlfq_tool_state import (DefaultToolStateExtractor, ToolReturnState,
                                                          ToolStateExtractor, ToolStateExtractorRegistry)

log = logging.getLogger(__name__)


@dataclass
class CMLFQRequestState:
    request_id: str
    prompt_id: str
    current_bucket: str
    current_instance_index: int = -1
    collected_return_states: List[ToolReturnState] = field(default_factory=list)
    generated_tokens: int = 0
    tool_return_token_positions: List[int] = field(default_factory=list)
    total_output_tokens: int = 0
    created_at: float = field(default_factory=time.time)
    has_migrated: bool = False


@dataclass
class CMLFQMigrationDecision:
    should_migrate: bool
    reason: str
    current_bucket: str
    target_bucket: str = ""
    mean_remaining_length: float = 0.0
    p90_remaining_length: float = 0.0


def rank_file(path: str, rank: int, step: Optional[int] = None) -> str:
    """``tree.json`` -> ``tree.rank_<R>[.step_<S>].json``."""
    p = Path(path)
    suffix = p.suffix or ".json"
    stem = p.name[: -len(p.suffix)] if p.suffix else p.name
    tag = f".step_{step}" if step is not None else ""
    return str(p.with_name(f"{stem}.rank_{rank}{tag}{suffix}"))


class CMLFQScheduler(BaseScheduler):
    DEFAULT_BUCKETS = {
        "short": {"tp_degrees": [1, 2], "max_tokens": 5000},
        "long": {"tp_degrees": [4, 8], "max_tokens": 50000},
    }

    def __init__(self, buckets: Optional[Dict[str, dict]] = None, bucket_thresholds: Optional[Dict[str, int]] = None,
                 tool_state_extractor: Optional[ToolStateExtractor] = None,
                 prefix_tree: Optional[CausalPrefixTree] = None, load_balance_strategy: str = "least_connections",
                 max_queue_length: int = 100, enable_fallback: bool = True, rebuild_interval: int = 50,
                 max_recent_trajectories: int = 5000, tree_path: str = "", tree_persist_interval: int = 1,
                 shared_load_dir: str = "", shared_load_ttl_s: float = 60.0, shared_load_heartbeat_s: float = 10.0):
        super().__init__(name="C-MLFQ")
        self._buckets = dict(buckets or self.DEFAULT_BUCKETS)
        self._bucket_thresholds = dict(bucket_thresholds or {n: c.get("max_tokens", 5000)
                                                              for n, c in self._buckets.items()})
        self._sorted_bucket_names = sorted(self._bucket_thresholds, key=self._bucket_thresholds.get)
        # each bucket prefers its own TP degrees and falls back to every other bucket's
        self._bucket_rules = {
            name: {"preferred_tp_degrees": list(cfg.get("tp_degrees", [1, 2])),
                   "fallback_tp_degrees": [tp for other, oc in self._buckets.items() if other != name
                                           for tp in oc.get("tp_degrees", [])]}
            for name, cfg in self._buckets.items()
        }
        self._strategy = LoadBalanceStrategy.parse(load_balance_strategy)
        self._max_queue_length = max_queue_length
        self._enable_fallback = enable_fallback
        self._rebuild_interval = max(0, rebuild_interval)
        self._max_recent = max(1, max_recent_trajectories)
        self._tree_path = tree_path
        self._tree_persist_interval = max(1, tree_persist_interval)
        self._rank = int(os.environ.get("RANK", "0"))
        self._world_size = int(os.environ.get("WORLD_SIZE", "1"))
        self._current_epoch = -1
        self._shared_load = (SharedCMLFQLoadState(shared_load_dir, shared_load_ttl_s, shared_load_heartbeat_s)
                             if shared_load_dir else None)
        self._global_counts: Optional[Dict[str, int]] = None
        self.prefix_tree = prefix_tree or CausalPrefixTree()
        if tool_state_extractor is not None:
            self._tool_registry = ToolStateExtractorRegistry()
            self._tool_registry.register(tool_state_extractor)
        else:
            self._tool_registry = ToolStateExtractorRegistry.create_default_registry()
        self._request_states: Dict[str, CMLFQRequestState] = {}
        self._recent_trajectories: List[Trajectory] = []
        self._migration_count = 0
        self._tool_return_count = 0
        self._tree_update_count = 0

    # -------------------------------------------------------------- load accounting
    def _load(self, handle: InstanceHandle) -> int:
        if self._global_counts is None:
            return handle.active_requests
        return int(self._global_counts.get(handle.instance_id, 0))

    def _on_selected(self, handle: InstanceHandle) -> None:
        handle.inc_active()
        if self._shared_load is not None:
            self._shared_load.increment(handle.instance_id)

    def _on_released(self, handle: InstanceHandle) -> None:
        handle.dec_active()
        if self._shared_load is not None:
            self._shared_load.decrement(handle.instance_id)

    def _route_to_bucket(self, bucket: str, input_tokens: int, prompt_id: str = "", reason: str = "") -> SchedulingResult:
        if bucket not in self._bucket_rules:
            bucket = self._sorted_bucket_names[0] if self._sorted_bucket_names else "short"
        rule = self._bucket_rules[bucket]
        self._global_counts = self._shared_load.aggregate() if self._shared_load is not None else None
        try:
            return self._route(bucket, rule["preferred_tp_degrees"], rule["fallback_tp_degrees"], prompt_id, reason)
        finally:
            self._global_counts = None

    # -------------------------------------------------------------- request lifecycle
    def schedule(self, input_tokens: int, prompt_id: str = "", n_samples: int = 1, epoch: int = -1) -> SchedulingResult:
        with self._lock:
            self._stats.total_requests += 1
        first = self._sorted_bucket_names[0] if self._sorted_bucket_names else "short"
        res = self._route_to_bucket(first, input_tokens, prompt_id, "cmlfq_initial_placement")
        if res.instance_index >= 0:
            rid = uuid.uuid4().hex
            self._request_states[rid] = CMLFQRequestState(rid, prompt_id, first, res.instance_index)
            res.request_id = rid
        return res

    def on_tool_return(self, request_id: str, tool_result: Any, generated_tokens: int = 0) -> CMLFQMigrationDecision:
        self._tool_return_count += 1
        st = self._request_states.get(request_id)
        if st is None:
            return CMLFQMigrationDecision(False, "request_not_found", "unknown")
        st.generated_tokens = generated_tokens
        state = self._tool_registry.extract(tool_result)
        st.collected_return_states.append(state)
        st.tool_return_token_positions.append(generated_tokens)
        node = self.prefix_tree.lookup_with_fallback(st.prompt_id, st.collected_return_states)
        if node is None or node.visit_count == 0:
            return CMLFQMigrationDecision(False, "tree_node_not_found", st.current_bucket)
        target = self.prefix_tree.get_bucket_for_node(node, self._bucket_thresholds)
        stats = dict(mean_remaining_length=node.mean_remaining_length, p90_remaining_length=node.p90_remaining_length)
        if target is None:
            return CMLFQMigrationDecision(False, "mean_p90_disagree", st.current_bucket, **stats)
        if target == st.current_bucket:
            return CMLFQMigrationDecision(False, "already_in_target_bucket", st.current_bucket, target, **stats)
        log.info("[CMLFQ] migrate %s: %s -> %s (mean=%.0f p90=%.0f tool=%s)", request_id, st.current_bucket, target,
                 node.mean_remaining_length, node.p90_remaining_length, state.to_key())
        return CMLFQMigrationDecision(True, "causal_signal_agree", st.current_bucket, target, **stats)

    def execute_migration(self, request_id: str, decision: CMLFQMigrationDecision) -> SchedulingResult:
        if not decision.should_migrate:
            raise ValueError("Cannot execute migration: decision.should_migrate is False")
        st = self._request_states.get(request_id)
        if st is None:
            raise ValueError(f"Request {request_id} not found")
        old = st.current_instance_index
        res = self._route_to_bucket(decision.target_bucket, 0, st.prompt_id, "cmlfq_migration")
        if res.instance_index >= 0:
            self._release(old)
            st.current_bucket = decision.target_bucket
            st.current_instance_index = res.instance_index
            st.has_migrated = True
            res.request_id = request_id
            self._migration_count += 1
            with self._lock:
                self._stats.migrated_routes += 1
        return res

    def has_request(self, request_id: str) -> bool:
        return request_id in self._request_states

    def get_request_route(self, request_id: str) -> Optional[SchedulingResult]:
        st = self._request_states.get(request_id)
        h = self.get_instance_handle(st.current_instance_index) if st else None
        if h is None:
            return None
        return SchedulingResult(h.index, h.tp_degree, st.current_bucket, False, "cmlfq_resume",
                                prompt_id=st.prompt_id, request_id=request_id)

    def on_request_done(self, instance_index: int, prompt_id: str = "", final_bucket: str = "",
                        output_tokens: int = 0) -> None:
        if prompt_id:
            rid = next((s.request_id for s in self._request_states.values()
                        if s.prompt_id == prompt_id and s.current_instance_index == instance_index), "")
            if rid:
                self.finish_request(rid, output_tokens)
                return
        self._release(instance_index)

    def finish_request(self, request_id: str, total_output_tokens: int) -> None:
        st = self._request_states.pop(request_id, None)
        if st is None:
            return
        self._release(st.current_instance_index)
        st.total_output_tokens = max(0, int(total_output_tokens))
        if not st.collected_return_states:
            return
        traj = Trajectory(st.prompt_id, list(st.collected_return_states),
                          [max(0, st.total_output_tokens - pos) for pos in st.tool_return_token_positions],
                          total_length=st.total_output_tokens)
        self.prefix_tree.insert(traj)
        self._recent_trajectories.append(traj)
        del self._recent_trajectories[:-self._max_recent]
        self._tree_update_count += 1
        if self._tree_update_count % self._tree_persist_interval == 0:
            self._persist_prefix_tree()

    def cancel_request(self, request_id: str) -> None:
        st = self._request_states.pop(request_id, None)
        if st is not None:
            self._release(st.current_instance_index)

    # -------------------------------------------------------------- tree maintenance
    def update_tree_from_trajectories(self, trajectories: List[Trajectory]) -> None:
        for t in trajectories:
            self.prefix_tree.insert(t)
        self._tree_update_count += len(trajectories)

    def rebuild_tree(self, trajectories: List[Trajectory]) -> None:
        self.prefix_tree.rebuild(trajectories)

    def _persist_prefix_tree(self, epoch: Optional[int] = None) -> None:
        if not self._tree_path:
            return
        self.prefix_tree.save(rank_file(self._tree_path, self._rank))
        if epoch is not None:
            self.prefix_tree.save(rank_file(self._tree_path, self._rank, epoch))

    def on_epoch_start(self, epoch: int) -> None:
        self._current_epoch = epoch

    def on_epoch_end(self, epoch: int) -> None:
        if (self._rebuild_interval > 0 and epoch > 0 and epoch % self._rebuild_interval == 0
                and self._recent_trajectories):
            self.prefix_tree.rebuild(self._recent_trajectories)
        self._persist_prefix_tree(epoch=epoch)

    def cmlfq_stats(self) -> dict:
        return {"tool_returns": self._tool_return_count, "migrations": self._migration_count,
                "tree_updates": self._tree_update_count, "active_requests": len(self._request_states),
                "tree": self.prefix_tree.get_stats()}

    def print_stats(self) -> None:
        super().print_stats()
        print(f"  [C-MLFQ] {self.cmlfq_stats()}")

    # -------------------------------------------------------------- construction
    @classmethod
    def from_config(cls, hetero_config: Any) -> "CMLFQScheduler":
        sched = hetero_config.scheduling
        buckets = getattr(sched, "cmlfq_buckets", None) or cls.DEFAULT_BUCKETS
        tree = CausalPrefixTree()
        tree_path = getattr(sched, "cmlfq_tree_path", "")
        if tree_path:
            for candidate in (rank_file(tree_path, int(os.environ.get("RANK", "0"))), tree_path):
                try:
                    tree.load(candidate)
                    break
                except FileNotFoundError:
                    continue
            else:
                log.warning("[CMLFQ] no prefix-tree file at %s", tree_path)
        return cls(
            buckets=buckets, bucket_thresholds={n: c.get("max_tokens", 5000) for n, c in buckets.items()},
            tool_state_extractor=DefaultToolStateExtractor(getattr(sched, "cmlfq_payload_small_threshold", 500),
                                                           getattr(sched, "cmlfq_payload_large_threshold", 5000)),
            prefix_tree=tree, load_balance_strategy=sched.load_balance_strategy,
            max_queue_length=sched.max_queue_length, enable_fallback=sched.enable_fallback,
            rebuild_interval=getattr(sched, "cmlfq_rebuild_interval", 50), tree_path=tree_path,
            tree_persist_interval=getattr(sched, "cmlfq_tree_persist_interval", 1),
            shared_load_dir=getattr(sched, "cmlfq_shared_load_dir", ""),
            shared_load_ttl_s=getattr(sched, "cmlfq_shared_load_ttl_s", 60.0),
            shared_load_heartbeat_s=getattr(sched, "cmlfq_shared_load_heartbeat_s", 10.0))
