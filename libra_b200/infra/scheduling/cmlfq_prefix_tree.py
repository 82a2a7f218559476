"""Causal prefix tree over tool-return states (C-MLFQ).

For every prompt (plus one global root aggregating all prompts) the tree keys
children by ``ToolReturnState.to_key()``; each node keeps the running mean and
the 90th percentile (over the most recent 200 samples) of the remaining output
length observed after reaching that prefix.  Lookup descends as deep as the
observed prefix allows and falls back to the global root when the prompt is
unseen; a bucket is returned only when the mean and the p90 map to the same
bucket (reference ``infra/scheduling/cmlfq_prefix_tree.py``).

The persisted JSON layout (version 2: ``roots`` per prompt + ``global_root``;
version-1 files without ``global_root`` are upgraded on load) is the same as
the reference's so tree snapshots are interchangeable.
"""

from __future__ import annotations

import json
import logging
import os
import threading
import time
from dataclasses import dataclass, field
from typing import Dict, List, Optional

from libra_b200.infra.scheduling.cmlfq_tool_state import ToolReturnState

log = logging.getLogger(__name__)

WINDOW = 200
GLOBAL_KEY = "__global__"


def _p90(values: List[float]) -> float:
    """numpy-compatible linear-interpolated 90th percentile."""
    if not values:
        return 0.0
    s = sorted(values)
    pos = 0.9 * (len(s) - 1)
    lo = int(pos)
    hi = min(lo + 1, len(s) - 1)
    return float(s[lo] + (s[hi] - s[lo]) * (pos - lo))


@dataclass
class PrefixTreeNode:
    key: str
    depth: int = 0
    mean_remaining_length: float = 0.0
    p90_remaining_length: float = 0.0
    visit_count: int = 0
    remaining_lengths: List[float] = field(default_factory=list)
    children: Dict[str, "PrefixTreeNode"] = field(default_factory=dict)

    def update_statistics(self, remaining_length: float) -> None:
        self.visit_count += 1
        self.mean_remaining_length += (remaining_length - self.mean_remaining_length) / self.visit_count
        self.remaining_lengths.append(float(remaining_length))
        del self.remaining_lengths[:-WINDOW]
        self.p90_remaining_length = _p90(self.remaining_lengths)

    def absorb(self, other: "PrefixTreeNode") -> None:
        """Merge another node's statistics (and subtree) into this one."""
        total = self.visit_count + other.visit_count
        if total:
            self.mean_remaining_length = (self.mean_remaining_length * self.visit_count
                                          + other.mean_remaining_length * other.visit_count) / total
        self.visit_count = total
        self.remaining_lengths = (self.remaining_lengths + other.remaining_lengths)[-WINDOW:]
        if self.remaining_lengths:
            self.p90_remaining_length = _p90(self.remaining_lengths)
        for k, child in other.children.items():
            mine = self.children.get(k)
            if mine is None:
                self.children[k] = PrefixTreeNode.from_dict(child.to_dict())
            else:
                mine.absorb(child)

    def to_dict(self) -> dict:
        return {
            "key": self.key, "depth": self.depth,
            "mean_remaining_length": round(self.mean_remaining_length, 2),
            "p90_remaining_length": round(self.p90_remaining_length, 2),
            "visit_count": self.visit_count, "remaining_lengths": self.remaining_lengths,
            "children": {k: v.to_dict() for k, v in self.children.items()},
        }

    @classmethod
    def from_dict(cls, d: dict) -> "PrefixTreeNode":
        node = cls(key=d["key"], depth=d.get("depth", 0), mean_remaining_length=d.get("mean_remaining_length", 0.0),
                   p90_remaining_length=d.get("p90_remaining_length", 0.0), visit_count=d.get("visit_count", 0),
                   remaining_lengths=[float(x) for x in d.get("remaining_lengths", [])])
        node.children = {k: cls.from_dict(c) for k, c in d.get("children", {}).items()}
        return node

    def get_tree_stats(self) -> dict:
        nodes, depth, leaves = 1, self.depth, 0 if self.children else 1
        for c in self.children.values():
            s = c.get_tree_stats()
            nodes += s["total_nodes"]
            depth = max(depth, s["max_depth"])
            leaves += s["leaf_count"]
        return {"total_nodes": nodes, "max_depth": depth, "leaf_count": leaves}


@dataclass
class Trajectory:
    """A finished request: its tool-return states and the output tokens still to
    come after each of them (plus, optionally, the total output length)."""

    prompt_id: str
    return_states: List[ToolReturnState]
    total_remaining_lengths: List[float]
    total_length: Optional[float] = None

    def __post_init__(self):
        if len(self.return_states) != len(self.total_remaining_lengths):
            raise AssertionError(f"return_states ({len(self.return_states)}) and total_remaining_lengths "
                                 f"({len(self.total_remaining_lengths)}) have different lengths")


def _key(prefix: str, states: List[ToolReturnState]) -> str:
    if not states:
        return f"{prefix}:root"
    return f"{prefix}:[{','.join(s.to_key() for s in states)}]"


class CausalPrefixTree:
    def __init__(self):
        self._roots: Dict[str, PrefixTreeNode] = {}
        self._global_root: Optional[PrefixTreeNode] = None
        self._lock = threading.RLock()
        self._total_insertions = 0

    # -------------------------------------------------------------- updates
    @staticmethod
    def _insert_path(root: PrefixTreeNode, traj: Trajectory, prefix: str) -> None:
        first = traj.total_length if traj.total_length is not None else (
            traj.total_remaining_lengths[0] if traj.total_remaining_lengths else None)
        if first is not None:
            root.update_statistics(first)
        node = root
        for i, (state, remaining) in enumerate(zip(traj.return_states, traj.total_remaining_lengths)):
            k = state.to_key()
            child = node.children.get(k)
            if child is None:
                child = PrefixTreeNode(key=_key(prefix, traj.return_states[:i + 1]), depth=node.depth + 1)
                node.children[k] = child
            child.update_statistics(remaining)
            node = child

    def insert(self, trajectory: Trajectory) -> None:
        with self._lock:
            root = self._roots.setdefault(trajectory.prompt_id,
                                          PrefixTreeNode(key=_key(trajectory.prompt_id, []), depth=0))
            self._insert_path(root, trajectory, trajectory.prompt_id)
            if self._global_root is None:
                self._global_root = PrefixTreeNode(key=f"{GLOBAL_KEY}:root", depth=0)
            self._insert_path(self._global_root, trajectory, GLOBAL_KEY)
            self._total_insertions += 1

    def rebuild(self, trajectories: List[Trajectory]) -> None:
        with self._lock:
            self._roots.clear()
            self._global_root = None
            self._total_insertions = 0
            for t in trajectories:
                self.insert(t)
        log.info("[CausalPrefixTree] rebuilt: %d prompts, %d trajectories", len(self._roots), len(trajectories))

    def merge(self, other: "CausalPrefixTree") -> None:
        if other is self:
            return
        with other._lock:
            roots = {p: PrefixTreeNode.from_dict(r.to_dict()) for p, r in other._roots.items()}
            glob = PrefixTreeNode.from_dict(other._global_root.to_dict()) if other._global_root else None
            n = other._total_insertions
        with self._lock:
            for p, r in roots.items():
                if p in self._roots:
                    self._roots[p].absorb(r)
                else:
                    self._roots[p] = r
            if glob is not None:
                if self._global_root is None:
                    self._global_root = glob
                else:
                    self._global_root.absorb(glob)
            self._total_insertions += n

    # -------------------------------------------------------------- queries
    @staticmethod
    def _descend(root: Optional[PrefixTreeNode], states: List[ToolReturnState], exact: bool):
        if root is None:
            return None
        node = root
        for s in states:
            child = node.children.get(s.to_key())
            if child is None:
                return None if exact else node
            node = child
        return node

    def lookup(self, prompt_id: str, return_states: List[ToolReturnState]) -> Optional[PrefixTreeNode]:
        """Exact-path lookup in the prompt's own tree."""
        with self._lock:
            return self._descend(self._roots.get(prompt_id), return_states, exact=True)

    def lookup_with_fallback(self, prompt_id: str, return_states: List[ToolReturnState]) -> Optional[PrefixTreeNode]:
        """Deepest matching prefix in the prompt's tree, else in the global tree."""
        with self._lock:
            root = self._roots.get(prompt_id)
            return self._descend(root if root is not None else self._global_root, return_states, exact=False)

    @staticmethod
    def _length_to_bucket(length: float, thresholds: Dict[str, int]) -> str:
        ordered = sorted(thresholds.items(), key=lambda kv: kv[1])
        for name, limit in ordered:
            if length <= limit:
                return name
        return ordered[-1][0] if ordered else "long"

    def get_bucket_for_node(self, node: Optional[PrefixTreeNode], bucket_thresholds: Dict[str, int]) -> Optional[str]:
        if node is None or node.visit_count == 0:
            return None
        by_mean = self._length_to_bucket(node.mean_remaining_length, bucket_thresholds)
        by_p90 = self._length_to_bucket(node.p90_remaining_length, bucket_thresholds)
        return by_mean if by_mean == by_p90 else None

    def get_stats(self) -> dict:
        with self._lock:
            per = [r.get_tree_stats() for r in self._roots.values()]
            return {
                "n_prompts": len(self._roots), "total_nodes": sum(s["total_nodes"] for s in per),
                "max_depth": max((s["max_depth"] for s in per), default=0),
                "total_leaves": sum(s["leaf_count"] for s in per), "total_insertions": self._total_insertions,
                "global_nodes": self._global_root.get_tree_stats()["total_nodes"] if self._global_root else 0,
            }

    # -------------------------------------------------------------- persistence
    def save(self, path: str) -> None:
        with self._lock:
            payload = {"version": 2, "total_insertions": self._total_insertions,
                       "roots": {p: r.to_dict() for p, r in self._roots.items()},
                       "global_root": self._global_root.to_dict() if self._global_root else None}
        directory = os.path.dirname(os.path.abspath(path))
        os.makedirs(directory, exist_ok=True)
        tmp = f"{path}.tmp.{os.getpid()}.{threading.get_ident()}.{time.time_ns()}"
        with open(tmp, "w", encoding="utf-8") as fh:
            json.dump(payload, fh, ensure_ascii=False, indent=2)
            fh.flush()
            os.fsync(fh.fileno())
        os.replace(tmp, path)

    def load(self, path: str) -> None:
        with open(path, "r", encoding="utf-8") as fh:
            data = json.load(fh)
        with self._lock:
            self._total_insertions = data.get("total_insertions", 0)
            self._roots = {p: PrefixTreeNode.from_dict(r) for p, r in data.get("roots", {}).items()}
            g = data.get("global_root")
            if g is not None:
                self._global_root = PrefixTreeNode.from_dict(g)
            elif self._roots:  # version 1: rebuild the global view from the prompt trees
                self._global_root = PrefixTreeNode(key=f"{GLOBAL_KEY}:root", depth=0)
                for r in self._roots.values():
                    self._global_root.absorb(r)
            else:
                self._global_root = None
