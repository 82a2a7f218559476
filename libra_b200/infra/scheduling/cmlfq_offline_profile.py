"""Offline C-MLFQ tree construction and periodic online refresh.

Builds ``Trajectory`` records from history ``StepRecord``s or raw trajectory
dicts (each with ``tool_returns`` carrying either ``remaining_length`` or a
``token_position``) and inserts them into a ``CausalPrefixTree``; the updater
inserts per step and rebuilds from a bounded window every ``rebuild_interval``
steps (reference ``infra/scheduling/cmlfq_offline_profile.py``).
"""

from __future__ import annotations

from dataclasses import dataclass
from typing import Iterable, List, Optional

from libra_b200.infra.scheduling.cmlfq_prefix_tree import CausalPrefixTree, Trajectory
from libra_b200.infra.scheduling.cmlfq_tool_state import (ToolReturnState, ToolStateExtractor,
                                                          ToolStateExtractorRegistry)


@dataclass
class ExtractedTrajectory:
    prompt_id: str
    return_states: List[ToolReturnState]
    total_remaining_lengths: List[float]
    total_output_tokens: int


class TrajectoryExtractor:
    def __init__(self, tool_extractor: Optional[ToolStateExtractor] = None):
        if tool_extractor is not None:
            self._registry = ToolStateExtractorRegistry()
            self._registry.register(tool_extractor)
        else:
            self._registry = ToolStateExtractorRegistry.create_default_registry()

    def _one(self, prompt_id: str, total: float, tool_returns: Iterable[dict]) -> Optional[Trajectory]:
        states, remaining = [], []
        for tr in tool_returns:
            payload = dict(tr)
            payload.setdefault("result", tr.get("output", ""))
            payload.setdefault("output", tr.get("result", ""))
            states.append(self._registry.extract(payload))
            if "remaining_length" in tr:
                remaining.append(float(tr["remaining_length"]))
            else:
                remaining.append(max(0.0, total - float(tr.get("token_position", total))))
        if not states:
            return None
        return Trajectory(prompt_id, states, remaining, total_length=total)

    def extract_from_step_records(self, records) -> List[Trajectory]:
        out = []
        for rec in records:
            for seq in getattr(rec, "sequences", []) or []:
                pid = str(seq.get("prompt_id", f"step{rec.step}_seq{seq.get('index', 0)}"))
                total = float(seq.get("total_output_tokens", seq.get("output_len", 0)))
                t = self._one(pid, total, seq.get("tool_returns", []))
                if t is not None:
                    out.append(t)
        return out

    def extract_from_raw_data(self, raw_trajectories: List[dict]) -> List[Trajectory]:
        out = []
        for raw in raw_trajectories:
            total = float(raw.get("total_output_tokens", raw.get("output_len", 0)))
            t = self._one(str(raw.get("prompt_id", "")), total, raw.get("tool_returns", []))
            if t is not None:
                out.append(t)
        return out


class CMLFQOfflineProfiler:
    def __init__(self, tool_extractor: Optional[ToolStateExtractor] = None,
                 prefix_tree: Optional[CausalPrefixTree] = None):
        self.extractor = TrajectoryExtractor(tool_extractor)
        self.prefix_tree = prefix_tree or CausalPrefixTree()

    def profile_from_raw_trajectories(self, raw: List[dict]) -> CausalPrefixTree:
        for t in self.extractor.extract_from_raw_data(raw):
            self.prefix_tree.insert(t)
        return self.prefix_tree

    def profile_from_step_records(self, records) -> CausalPrefixTree:
        for t in self.extractor.extract_from_step_records(records):
            self.prefix_tree.insert(t)
        return self.prefix_tree

    def save_tree(self, path: str) -> None:
        self.prefix_tree.save(path)

    def load_tree(self, path: str) -> CausalPrefixTree:
        self.prefix_tree.load(path)
        return self.prefix_tree


class CMLFQTreeUpdater:
    def __init__(self, prefix_tree: CausalPrefixTree, rebuild_interval: int = 50, max_recent_trajectories: int = 5000):
        self.prefix_tree = prefix_tree
        self.rebuild_interval = rebuild_interval
        self.max_recent_trajectories = max_recent_trajectories
        self._recent: List[Trajectory] = []
        self._step = 0
        self._inserted = 0

    def update_from_step(self, step: int, trajectories: List[Trajectory]) -> None:
        self._step = step
        for t in trajectories:
            self.prefix_tree.insert(t)
        self._inserted += len(trajectories)
        self._recent = (self._recent + list(trajectories))[-self.max_recent_trajectories:]
        if step > 0 and self.rebuild_interval > 0 and step % self.rebuild_interval == 0:
            self.prefix_tree.rebuild(self._recent)

    def force_rebuild(self, trajectories: List[Trajectory]) -> None:
        self._recent = list(trajectories)
        self.prefix_tree.rebuild(self._recent)

    def get_stats(self) -> dict:
        return {"step_count": self._step, "total_insertions": self._inserted, "recent_trajectories": len(self._recent),
                "rebuild_interval": self.rebuild_interval, "tree_stats": self.prefix_tree.get_stats()}
