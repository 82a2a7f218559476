"""Background asyncio runner for rollout coroutines.

Behaviour matches the reference ``infra/execution/async_runner.py``: a daemon
thread owns an event loop; ``submit`` hands a coroutine factory over a bounded
input queue, finished tasks land on a bounded output queue as ``TaskResult``;
``pause`` stops new starts while already accepted tasks still run (so a
weight update can drain the pipeline); ``reset_runtime_state`` restarts the
loop and bumps a generation counter so late results from the old loop are
dropped.

Implementation: the loop thread is woken through ``call_soon_threadsafe``; each
accepted task is wrapped in a coroutine that publishes its own result, so the
loop needs no polling over the running set.
"""

from __future__ import annotations

import asyncio
import queue
import threading
import time
from dataclasses import dataclass
from typing import Any, Awaitable, Callable, Generic, List, Optional, TypeVar

T = TypeVar("T")


@dataclass
class TaskResult(Generic[T]):
    data: T
    task_id: int
    create_time: float
    complete_time: float


class AsyncTaskRunner(Generic[T]):
    def __init__(self, max_queue_size: int = 100, enable_tracing: bool = False):
        self.max_queue_size = max_queue_size
        self.enable_tracing = enable_tracing
        self.exiting = threading.Event()
        self.paused = threading.Event()
        self.input_queue: queue.Queue = queue.Queue(maxsize=max_queue_size)
        self.output_queue: queue.Queue = queue.Queue(maxsize=max_queue_size)
        self._generation = 0
        self._active: set = set()
        self._active_lock = threading.Lock()
        self._error: Optional[BaseException] = None
        self._loop: Optional[asyncio.AbstractEventLoop] = None
        self._wake: Optional[asyncio.Event] = None
        self.thread: Optional[threading.Thread] = None

    # -------------------------------------------------------------- lifecycle
    def initialize(self) -> None:
        self.exiting.clear()
        ready = threading.Event()
        gen = self._generation
        self.thread = threading.Thread(target=self._thread_main, args=(gen, ready, self.exiting, self.input_queue,
                                                                        self.output_queue), daemon=True,
                                       name=f"async-runner-g{gen}")
        self.thread.start()
        ready.wait()
        if self._error is not None:
            raise RuntimeError(f"AsyncTaskRunner initialization failed: {self._error}")

    def destroy(self, timeout: float = 10.0) -> None:
        self.exiting.set()
        self.paused.clear()
        self._poke()
        if self.thread is not None:
            self.thread.join(timeout=timeout)
            if self.thread.is_alive():
                print("WARNING: AsyncTaskRunner thread did not exit before the timeout")

    def reset_runtime_state(self, timeout: float = 10.0) -> None:
        """Cancel everything in flight and restart with empty queues (pause state kept)."""
        was_paused = self.paused.is_set()
        self._generation += 1
        self.destroy(timeout=timeout)
        self.exiting = threading.Event()
        self.paused = threading.Event()
        self.input_queue = queue.Queue(maxsize=self.max_queue_size)
        self.output_queue = queue.Queue(maxsize=self.max_queue_size)
        with self._active_lock:
            self._active.clear()
        self._error = None
        self._loop = None
        self._wake = None
        self.initialize()
        if was_paused:
            self.pause()

    # -------------------------------------------------------------- loop thread
    def _thread_main(self, gen, ready, exiting, inq, outq):
        loop = asyncio.new_event_loop()
        asyncio.set_event_loop(loop)
        try:
            if gen == self._generation:
                self._loop = loop
                self._wake = asyncio.Event()
            wake = self._wake if gen == self._generation else asyncio.Event()
            ready.set()
            loop.run_until_complete(self._serve(gen, exiting, inq, outq, wake))
        except BaseException as exc:  # noqa: BLE001 - reported through submit/wait
            if gen == self._generation:
                self._error = exc
            print(f"ERROR: AsyncTaskRunner thread error: {exc}")
        finally:
            exiting.set()
            ready.set()
            loop.close()

    async def _serve(self, gen, exiting, inq, outq, wake: asyncio.Event):
        tasks: set = set()

        async def run_one(item):
            try:
                data = await item["fn"](*item["args"], **item["kwargs"])
            except asyncio.CancelledError:
                data = None
            except Exception as exc:  # noqa: BLE001 - a failed rollout yields None
                print(f"ERROR: task {item['task_id']} execution failed: {exc}")
                data = None
            with self._active_lock:
                self._active.discard(item["task_id"])
            if gen != self._generation:
                return
            outq.put_nowait(TaskResult(data=data, task_id=item["task_id"], create_time=item["create_time"],
                                       complete_time=time.monotonic_ns()))
            wake.set()

        try:
            while not exiting.is_set():
                # Accepted inputs always start, even while paused (drain semantics).
                while True:
                    try:
                        item = inq.get_nowait()
                    except queue.Empty:
                        break
                    task = asyncio.ensure_future(run_one(item))
                    tasks.add(task)
                    task.add_done_callback(tasks.discard)
                wake.clear()
                if inq.qsize() or exiting.is_set():
                    continue
                try:
                    await asyncio.wait_for(wake.wait(), timeout=0.05)
                except asyncio.TimeoutError:
                    pass
        finally:
            for task in list(tasks):
                task.cancel()
            if tasks:
                await asyncio.gather(*tasks, return_exceptions=True)

    def _poke(self) -> None:
        loop, wake = self._loop, self._wake
        if loop is None or wake is None:
            return
        try:
            loop.call_soon_threadsafe(wake.set)
        except RuntimeError:
            pass

    # -------------------------------------------------------------- API
    def submit(self, async_fn: Callable[..., Awaitable[T]], *args, task_id: int, **kwargs) -> int:
        if self._error is not None:
            raise RuntimeError(f"AsyncTaskRunner is unusable: {self._error}")
        with self._active_lock:
            if task_id in self._active:
                raise ValueError(f"duplicate task ID: {task_id}")
            self._active.add(task_id)
        item = {"fn": async_fn, "args": args, "kwargs": kwargs, "task_id": task_id, "create_time": time.monotonic_ns()}
        try:
            self.input_queue.put_nowait(item)
        except queue.Full:
            with self._active_lock:
                self._active.discard(task_id)
            raise queue.Full("input queue is full")
        self._poke()
        return task_id

    def wait(self, count: int, timeout: Optional[float] = None) -> List[TaskResult]:
        deadline = time.monotonic() + (3600.0 if timeout is None else timeout)
        out: List[TaskResult] = []
        while len(out) < count:
            if self._error is not None:
                raise RuntimeError(f"AsyncTaskRunner error: {self._error}")
            if self.exiting.is_set():
                raise RuntimeError("AsyncTaskRunner is shutting down")
            left = deadline - time.monotonic()
            if left <= 0:
                raise TimeoutError(f"waited for {count} tasks; received only {len(out)} results")
            try:
                out.append(self.output_queue.get(timeout=min(0.1, left)))
            except queue.Empty:
                pass
        return out

    def pause(self) -> None:
        self.paused.set()

    def resume(self) -> None:
        self.paused.clear()
        self._poke()

    def wait_until_idle(self, timeout: float = 3600.0) -> None:
        deadline = time.monotonic() + timeout
        while True:
            if self._error is not None:
                raise RuntimeError(f"AsyncTaskRunner error: {self._error}")
            with self._active_lock:
                active = len(self._active)
            if active == 0 and self.input_queue.empty():
                return
            if time.monotonic() >= deadline:
                raise TimeoutError("Timed out draining rollout tasks before weight reload: "
                                   f"active={active}, queued={self.input_queue.qsize()}")
            time.sleep(0.02)

    def get_queue_sizes(self):
        return self.input_queue.qsize(), self.output_queue.qsize()

    def active_count(self) -> int:
        with self._active_lock:
            return len(self._active)
