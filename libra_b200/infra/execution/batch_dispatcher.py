"""Producer/consumer dispatcher between the trainer and the rollout runner.

Reference behaviour (``infra/execution/batch_dispatcher.py``):

* a producer thread submits pending ``TaskInput``s while the runner is not
  paused, the staleness manager reports capacity and the runner queue has room;
* a consumer thread moves finished results into a pending-result map;
* ``active_submit_and_wait`` keeps feeding an infinite input generator until
  ``batch_size`` non-``None`` results have arrived (rejected rollouts return
  ``None`` and do not count), optionally with a timeout;
* ``get_runtime_metrics`` is the queue-pressure snapshot the online planner reads.
"""

from __future__ import annotations

import logging
import queue
import threading
import time
from collections import deque
from dataclasses import dataclass
from typing import Any, Awaitable, Callable, Dict, Generator, Generic, List, Optional, TypeVar

from libra_b200.infra.execution.async_runner import AsyncTaskRunner, TaskResult
from libra_b200.infra.sync.staleness import StalenessManager

log = logging.getLogger(__name__)
TInput = TypeVar("TInput")
TResult = TypeVar("TResult")

FETCH_MAX = 100
JOIN_TIMEOUT_S = 2.0
FOREVER_S = float(7 * 24 * 3600)


@dataclass
class TaskInput:
    task_id: int
    data: Any
    version: int = 0
    group_id: Optional[str] = None
    rollout_index: int = 0


class BatchTaskDispatcher(Generic[TInput, TResult]):
    def __init__(self, async_runner: AsyncTaskRunner, staleness_manager: StalenessManager,
                 task_factory: Callable[[TInput], Callable[..., Awaitable[Optional[TResult]]]],
                 enable_tracing: bool = False):
        self.runner = async_runner
        self.staleness_manager = staleness_manager
        self.task_factory = task_factory
        self.enable_tracing = enable_tracing
        self._inputs: deque = deque()
        self._results: Dict[int, TaskResult] = {}
        self._active: set = set()
        self._in_cv = threading.Condition()
        self._out_cv = threading.Condition()
        self._reconfig = threading.RLock()
        self._resetting = threading.Event()
        self._stop = threading.Event()
        self._error: Optional[BaseException] = None
        self._threads: List[threading.Thread] = []

    # -------------------------------------------------------------- lifecycle
    def initialize(self) -> None:
        self._stop.clear()
        self._threads = [threading.Thread(target=self._producer, daemon=True, name="dispatcher-producer"),
                         threading.Thread(target=self._consumer, daemon=True, name="dispatcher-consumer")]
        for t in self._threads:
            t.start()

    def destroy(self) -> None:
        self._stop.set()
        self._notify_all()
        for t in self._threads:
            t.join(timeout=JOIN_TIMEOUT_S)
            if t.is_alive():
                log.warning("%s did not exit before the timeout", t.name)
        self.runner.destroy()

    def _notify_all(self) -> None:
        with self._in_cv:
            self._in_cv.notify_all()
        with self._out_cv:
            self._out_cv.notify_all()

    def _fail(self, exc: BaseException) -> None:
        if self._error is None:
            self._error = exc
        self._notify_all()

    def _raise_if_failed(self) -> None:
        if self._error is not None:
            raise RuntimeError(f"background thread error: {self._error}") from self._error

    def _can_submit(self) -> bool:
        return (not self.runner.paused.is_set() and self.staleness_manager.get_capacity() > 0
                and self.runner.input_queue.qsize() < self.runner.max_queue_size)

    # -------------------------------------------------------------- threads
    def _producer(self) -> None:
        while not self._stop.is_set():
            try:
                with self._in_cv:
                    self._in_cv.wait_for(lambda: self._stop.is_set() or self._error is not None or (
                        self._inputs and not self.runner.paused.is_set()
                        and self.staleness_manager.get_capacity() > 0), timeout=0.5)
                    if self._stop.is_set():
                        return
                    self._raise_if_failed()
                    if not (self._inputs and not self.runner.paused.is_set()
                            and self.staleness_manager.get_capacity() > 0):
                        continue
                    item = self._inputs.popleft()
                with self._reconfig:
                    fn = self.task_factory(item)
                    try:
                        self.runner.submit(fn, task_id=item.task_id)
                        self.staleness_manager.on_rollout_submitted()
                    except queue.Full:
                        with self._in_cv:
                            self._inputs.appendleft(item)
                            self._in_cv.wait_for(lambda: self._stop.is_set() or self._can_submit(), timeout=1.0)
            except Exception as exc:  # noqa: BLE001
                log.error("Producer thread error: %s", exc, exc_info=True)
                self._fail(exc)
                return

    def _consumer(self) -> None:
        while not self._stop.is_set():
            try:
                n = max(1, min(self.runner.output_queue.qsize(), FETCH_MAX))
                try:
                    got = self.runner.wait(count=n, timeout=0.05)
                except TimeoutError:
                    continue
                with self._out_cv:
                    for r in got:
                        self._results[r.task_id] = r
                    self._out_cv.notify_all()
                with self._in_cv:
                    self._in_cv.notify()
            except Exception as exc:  # noqa: BLE001
                if self._resetting.is_set() and "shutting down" in str(exc):
                    time.sleep(0.01)
                    continue
                log.error("Consumer thread error: %s", exc, exc_info=True)
                self._fail(exc)
                return

    # -------------------------------------------------------------- API
    def submit_task_input(self, task_input: TInput) -> None:
        self._raise_if_failed()
        with self._in_cv:
            self._inputs.append(task_input)
            self.staleness_manager.on_rollout_enqueued()
            self._in_cv.notify()
        with self._out_cv:
            self._active.add(task_input.task_id)

    def wait_results(self, count: int, timeout: Optional[float] = None, raise_timeout: bool = True) -> List[TaskResult]:
        if count <= 0:
            raise ValueError(f"count must be positive; got {count}")
        deadline = time.perf_counter() + (FOREVER_S if timeout is None else timeout)
        with self._out_cv:
            while len(self._results) < count:
                self._raise_if_failed()
                left = deadline - time.perf_counter()
                if left <= 0:
                    if raise_timeout:
                        raise TimeoutError(f"waited for {count} results, received only {len(self._results)}")
                    return []
                self._out_cv.wait(timeout=min(left, 1.0))
            ordered = sorted(self._results.values(), key=lambda r: r.create_time)
            chosen, rest = ordered[:count], ordered[count:]
            self._results = {r.task_id: r for r in rest}
            for r in chosen:
                self._active.discard(r.task_id)
            if rest:
                self._out_cv.notify_all()
        return chosen

    def active_submit_and_wait(self, input_generator: Generator, batch_size: int,
                               timeout: Optional[float] = None) -> List[Any]:
        accepted: List[Any] = []
        t0 = time.monotonic()
        while len(accepted) < batch_size:
            if timeout is not None and timeout > 0 and time.monotonic() - t0 >= timeout:
                raise TimeoutError(f"active batch collection timed out: accepted={len(accepted)}/{batch_size}, "
                                   f"runtime_metrics={self.get_runtime_metrics()}")
            with self._in_cv:
                queued = len(self._inputs)
            room = min(self.staleness_manager.get_pending_limit() - queued,
                       self.runner.max_queue_size - (self.runner.input_queue.qsize() + batch_size))
            for _ in range(max(0, min(batch_size, room))):
                try:
                    self.submit_task_input(next(input_generator))
                except StopIteration:
                    raise RuntimeError("The input generator is exhausted; use an infinite generator") from None
            for r in self.wait_results(count=batch_size - len(accepted), timeout=1.0, raise_timeout=False):
                if r.data is None:
                    continue
                accepted.append(r.data)
                if len(accepted) >= batch_size:
                    break
        return accepted

    def pause(self) -> None:
        self.runner.pause()
        with self._in_cv:
            self._in_cv.notify()

    def resume(self) -> None:
        self.runner.resume()
        with self._in_cv:
            self._in_cv.notify()

    def is_paused(self) -> bool:
        return self.runner.paused.is_set()

    def wait_until_idle(self, timeout: float = 3600.0) -> None:
        if not self.is_paused():
            raise RuntimeError("pause() must be called before wait_until_idle()")
        self.runner.wait_until_idle(timeout=timeout)

    def reset_after_reconfigure(self) -> None:
        """Drop queued inputs/results that belong to the previous rollout pool."""
        self._resetting.set()
        try:
            with self._reconfig:
                with self._in_cv:
                    self._inputs.clear()
                with self._out_cv:
                    self._results.clear()
                    self._active.clear()
                if hasattr(self.runner, "reset_runtime_state"):
                    self.runner.reset_runtime_state()
                if hasattr(self.staleness_manager, "reset_runtime_state"):
                    self.staleness_manager.reset_runtime_state()
        finally:
            self._resetting.clear()
            self._notify_all()

    def get_runtime_metrics(self) -> Dict[str, Any]:
        with self._in_cv:
            pending_inputs = len(self._inputs)
        with self._out_cv:
            pending_results = len(self._results)
            active = len(self._active)
        in_q, out_q = self.runner.get_queue_sizes()
        st = self.staleness_manager.get_stats()
        cap = self.staleness_manager.get_capacity()
        limit = max(1, self.staleness_manager.get_pending_limit())
        max_conc = max(1, int(getattr(self.staleness_manager, "max_concurrent_rollouts", 1)))
        return {
            "pending_inputs": pending_inputs, "pending_results": pending_results, "active_tasks": active,
            "runner_input_queue": in_q, "runner_output_queue": out_q, "runner_max_queue": self.runner.max_queue_size,
            "staleness_enqueued": st.enqueued, "staleness_running": st.running, "staleness_accepted": st.accepted,
            "staleness_rejected": st.rejected, "staleness_capacity": cap, "staleness_pending_limit": limit,
            "queue_pressure": min(1.0, (pending_inputs + in_q) / float(limit)),
            "active_rollout_pressure": min(1.0, st.running / float(max_conc)),
            "paused": self.is_paused(),
        }
