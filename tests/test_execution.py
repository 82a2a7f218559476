"""Async runner, dispatcher and staleness behaviour (reference tests/test_async_task_runner.py)."""

import asyncio
import itertools
import threading
import time

import pytest

from libra_b200.infra.execution.async_runner import AsyncTaskRunner
from libra_b200.infra.execution.batch_dispatcher import BatchTaskDispatcher, TaskInput
from libra_b200.infra.sync.staleness import StalenessManager


class _Ver:
    def __init__(self):
        self.v = 0

    def get_version(self):
        return self.v


def test_staleness_capacity_formula():
    ver = _Ver()
    sm = StalenessManager(ver, max_concurrent_rollouts=100, consumer_batch_size=8, max_staleness=1)
    assert sm.get_pending_limit() == 16
    assert sm.get_capacity() == 16
    for _ in range(10):
        sm.on_rollout_enqueued()
        sm.on_rollout_submitted()
    assert sm.get_capacity() == 6
    for _ in range(10):
        sm.on_rollout_accepted()
    sm.on_batch_consumed(8)
    ver.v = 1
    assert sm.get_capacity() == (1 + 1 + 1) * 8 - 2
    sm2 = StalenessManager(ver, max_concurrent_rollouts=3, consumer_batch_size=8, max_staleness=4)
    assert sm2.get_capacity() == 3


def test_runner_pause_drains_accepted_tasks():
    r = AsyncTaskRunner(max_queue_size=16)
    r.initialize()
    done = []

    async def job(i):
        await asyncio.sleep(0.05)
        done.append(i)
        return i

    for i in range(4):
        r.submit(job, i, task_id=i)
    r.pause()
    r.wait_until_idle(timeout=5)
    assert sorted(done) == [0, 1, 2, 3]
    res = r.wait(4, timeout=2)
    assert sorted(x.data for x in res) == [0, 1, 2, 3]
    with pytest.raises(ValueError):
        r.submit(job, 9, task_id=7)
        r.submit(job, 9, task_id=7)
    r.destroy()


def test_runner_idle_timeout_and_reset_drops_old_results():
    r = AsyncTaskRunner(max_queue_size=8)
    r.initialize()

    async def slow():
        await asyncio.sleep(10)
        return 1

    r.submit(slow, task_id=1)
    r.pause()
    with pytest.raises(TimeoutError):
        r.wait_until_idle(timeout=0.2)
    r.reset_runtime_state()
    assert r.paused.is_set()
    assert r.get_queue_sizes() == (0, 0)
    assert r.active_count() == 0
    r.destroy()


def test_dispatcher_collects_batch_skipping_rejections():
    ver = _Ver()
    sm = StalenessManager(ver, max_concurrent_rollouts=8, consumer_batch_size=4, max_staleness=2)
    runner = AsyncTaskRunner(max_queue_size=64)
    runner.initialize()

    def factory(ti):
        async def run():
            await asyncio.sleep(0.005)
            if ti.task_id % 3 == 0:
                sm.on_rollout_rejected()
                return None
            sm.on_rollout_accepted()
            return ti.task_id
        return run

    d = BatchTaskDispatcher(runner, sm, factory)
    d.initialize()
    gen = (TaskInput(task_id=i, data=i) for i in itertools.count())
    got = d.active_submit_and_wait(gen, batch_size=4, timeout=10)
    assert len(got) == 4 and all(g % 3 for g in got)
    sm.on_batch_consumed(4)
    m = d.get_runtime_metrics()
    assert 0.0 <= m["queue_pressure"] <= 1.0 and "staleness_capacity" in m
    d.pause()
    d.wait_until_idle(timeout=5)
    d.reset_after_reconfigure()
    assert d.get_runtime_metrics()["pending_results"] == 0
    d.destroy()


def test_dispatcher_timeout():
    ver = _Ver()
    sm = StalenessManager(ver, 4, 2, 0)
    runner = AsyncTaskRunner(max_queue_size=8)
    runner.initialize()

    def factory(ti):
        async def run():
            sm.on_rollout_rejected()
            return None
        return run

    d = BatchTaskDispatcher(runner, sm, factory)
    d.initialize()
    gen = (TaskInput(task_id=i, data=i) for i in itertools.count())
    with pytest.raises(TimeoutError):
        d.active_submit_and_wait(gen, batch_size=2, timeout=0.5)
    d.destroy()
