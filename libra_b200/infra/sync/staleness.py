"""Off-policy (staleness) admission control for asynchronous rollouts.

Same bound as the reference (``infra/sync/staleness.py:46-61``, AReaL style):
a new rollout may start only while

    running < max_concurrent_rollouts
    accepted + running < (max_staleness + version + 1) * consumer_batch_size

so no accepted sample can be more than ``max_staleness`` policy versions older
than the model that trains on it.
"""

from __future__ import annotations

import threading
from dataclasses import dataclass, replace
from typing import Protocol


class VersionProvider(Protocol):
    def get_version(self) -> int: ...


@dataclass
class RolloutStat:
    enqueued: int = 0
    running: int = 0
    accepted: int = 0
    rejected: int = 0


class StalenessManager:
    def __init__(self, version_provider: VersionProvider, max_concurrent_rollouts: int, consumer_batch_size: int,
                 max_staleness: int):
        self.version_provider = version_provider
        self.max_concurrent_rollouts = max_concurrent_rollouts
        self.consumer_batch_size = consumer_batch_size
        self.max_staleness = max_staleness
        self._lock = threading.Lock()
        self._stat = RolloutStat()

    # the reference exposes these two names; keep them for callers/tests
    @property
    def lock(self):
        return self._lock

    @property
    def rollout_stat(self) -> RolloutStat:
        return self._stat

    def get_pending_limit(self) -> int:
        return (self.max_staleness + 1) * self.consumer_batch_size

    def get_capacity(self) -> int:
        with self._lock:
            version = int(self.version_provider.get_version())
            by_concurrency = max(1, self.max_concurrent_rollouts) - self._stat.running
            in_flight = self._stat.accepted + self._stat.running
            by_staleness = (self.max_staleness + version + 1) * max(1, self.consumer_batch_size) - in_flight
            return min(by_concurrency, by_staleness)

    def _bump(self, **delta: int) -> None:
        with self._lock:
            for key, d in delta.items():
                setattr(self._stat, key, getattr(self._stat, key) + d)

    def on_rollout_enqueued(self) -> None:
        self._bump(enqueued=1)

    def on_rollout_submitted(self) -> None:
        self._bump(enqueued=-1, running=1)

    def on_rollout_accepted(self) -> None:
        self._bump(running=-1, accepted=1)

    def on_rollout_rejected(self) -> None:
        self._bump(running=-1, rejected=1)

    def on_batch_consumed(self, count: int) -> None:
        self._bump(accepted=-int(count))

    def get_stats(self) -> RolloutStat:
        with self._lock:
            return replace(self._stat)

    def reset_runtime_state(self) -> None:
        """Forget queue accounting after a rollout-pool cutover (rejections are history)."""
        with self._lock:
            self._stat.enqueued = self._stat.running = self._stat.accepted = 0
