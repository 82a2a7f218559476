"""Heterogeneous rollout pool: TP-bucket instances behind one scheduler.

API of the reference (``engine/heterogeneous_engine.py``): ``generate`` routes
a request through the scheduler (an active C-MLFQ ``request_id`` keeps its
current instance; LA-MLFQ ``pending`` results wait for the scout), calls the
chosen instance and reports completion; ``begin / route_tool_return / finish /
cancel`` drive the C-MLFQ request lifecycle of multi-turn workflows;
``reconfigure_from_plan`` swaps the instance set after a planner decision;
``wait_until_idle`` drains before weight updates.

On one B200 box the instances are ``LocalRolloutEngine`` objects (in-process
engines pinned to their GPUs), ``HTTPRolloutEngine`` clients of separate server
processes, or mocks - the routing logic is the same for all three.
"""

from __future__ import annotations

import asyncio
import logging
import os
import threading
import time
import uuid
from typing import Any, Dict, List, Optional

from libra_b200.infra.scheduling import SchedulerFactory
from libra_b200.infra.scheduling.base import BaseScheduler, SchedulingResult

log = logging.getLogger(__name__)


class HeterogeneousRolloutEngine:
    def __init__(self, engines: List[Any], instance_configs: List[Dict[str, Any]], scheduler: BaseScheduler):
        if len(engines) != len(instance_configs):
            raise ValueError("engines and instance_configs must have the same length")
        self.engines = list(engines)
        self.instance_configs = [dict(c) for c in instance_configs]
        self.scheduler = scheduler
        self._lock = threading.Lock()
        self._rr = 0
        self._inflight = 0
        self._inflight_lock = threading.Lock()
        # C-MLFQ requests: token context after their last turn (prompt + output), for KV migration
        self._contexts: Dict[str, List[int]] = {}
        self.kv_migrations = {"count": 0, "tokens": 0, "seconds": 0.0}
        for i, c in enumerate(self.instance_configs):
            scheduler.register_instance(i, c["instance_id"], int(c["tp_degree"]))

    @property
    def num_instances(self) -> int:
        return len(self.engines)

    # -------------------------------------------------------------- generation
    async def generate(self, prompt, max_new_tokens: int = 1024, temperature: float = 1.0, top_p: float = 1.0,
                       n: int = 1, input_tokens: int = 0, prompt_id: str = "", n_samples: int = 1, epoch: int = -1,
                       request_id: str = "", **kwargs) -> Dict[str, Any]:
        if input_tokens <= 0:
            input_tokens = len(prompt) if not isinstance(prompt, str) else max(1, len(prompt) // 3)
        with self._lock:
            route = self.scheduler.get_request_route(request_id) if (
                request_id and hasattr(self.scheduler, "get_request_route")) else None
            managed = route is not None
            if route is None:
                route = self.scheduler.schedule(input_tokens=input_tokens, prompt_id=prompt_id, n_samples=n_samples,
                                                epoch=epoch)
        if route.pending:
            route = await self._wait_for_scout(prompt_id, input_tokens, n_samples, epoch)
        with self._lock:
            if route.instance_index < 0:
                idx = self._rr % max(1, self.num_instances)
                self._rr += 1
                log.warning("scheduling failed (%s); falling back to instance %d", route.reason, idx)
            else:
                idx = route.instance_index
            engine, cfg = self.engines[idx], self.instance_configs[idx]
        out_tokens = 0
        with self._inflight_lock:
            self._inflight += 1
        try:
            res = await engine.generate(prompt, max_new_tokens=max_new_tokens, temperature=temperature, top_p=top_p,
                                        n=n, input_tokens=input_tokens, **kwargs)
            out_tokens = len(res.get("token_ids") or res.get("tokens") or [])
            if managed and request_id and res.get("token_ids") is not None:
                ids = res.get("prompt_token_ids") if isinstance(prompt, str) else prompt
                if ids is not None:
                    self._contexts[request_id] = list(ids) + list(res["token_ids"])
            res["_schedule_info"] = {"instance_index": idx, "instance_id": cfg["instance_id"],
                                     "tp_degree": cfg["tp_degree"], "category": route.category,
                                     "is_fallback": route.is_fallback, "reason": route.reason, "prompt_id": prompt_id,
                                     "request_id": request_id or route.request_id}
            return res
        finally:
            with self._inflight_lock:
                self._inflight -= 1
            if not managed:
                with self._lock:
                    if route.request_id and hasattr(self.scheduler, "finish_request"):
                        self.scheduler.finish_request(route.request_id, out_tokens)
                    else:
                        self.scheduler.on_request_done(instance_index=idx, prompt_id=prompt_id,
                                                       final_bucket=route.category, output_tokens=out_tokens)

    async def _wait_for_scout(self, prompt_id: str, input_tokens: int, n_samples: int, epoch: int,
                              timeout: float = 60.0) -> SchedulingResult:
        mgr = getattr(self.scheduler, "scout_manager", None)
        if mgr is None:
            return self.scheduler.schedule(input_tokens, prompt_id, 1, epoch)
        from libra_b200.infra.scheduling.baselines import WaitingRequest

        fut = asyncio.get_running_loop().create_future()
        with self._lock:
            mgr.add_waiting(WaitingRequest(prompt_id, input_tokens, n_samples, epoch, 0, future=fut))
        try:
            return await asyncio.wait_for(fut, timeout)
        except asyncio.TimeoutError:
            with self._lock:
                for w in mgr.force_release(prompt_id):
                    if w.future is not None and not w.future.done():
                        w.future.set_result(self.scheduler.schedule(w.input_tokens, w.prompt_id, 1, w.epoch))
                return self.scheduler.schedule(input_tokens, prompt_id, 1, epoch)

    # -------------------------------------------------------------- C-MLFQ lifecycle
    def begin_cmlfq_request(self, prompt_id: str, input_tokens: int, epoch: int = -1) -> str:
        if not hasattr(self.scheduler, "get_request_route"):
            return ""
        with self._lock:
            return self.scheduler.schedule(input_tokens=input_tokens, prompt_id=prompt_id, n_samples=1,
                                           epoch=epoch).request_id

    def on_tool_return(self, request_id: str, tool_result: Any, generated_tokens: int = 0):
        if hasattr(self.scheduler, "on_tool_return"):
            with self._lock:
                return self.scheduler.on_tool_return(request_id, tool_result, generated_tokens)
        return None

    def execute_cmlfq_migration(self, request_id: str, decision: Any):
        """Move a C-MLFQ request to the bucket the decision names and, when both
        instances are in-process engines, bring its KV prefix along: the
        cached blocks of its context are copied GPU to GPU into the target's
        prefix cache, so its next turn there prefills only the new tokens."""
        if not hasattr(self.scheduler, "execute_migration"):
            return None
        with self._lock:
            old = self.scheduler.get_request_route(request_id) if hasattr(self.scheduler, "get_request_route") else None
            res = self.scheduler.execute_migration(request_id, decision)
        ctx = self._contexts.get(request_id)
        if old is not None and res is not None and res.instance_index >= 0 and ctx and \
                old.instance_index != res.instance_index:
            src = getattr(self.engines[old.instance_index], "engine", None)
            target = self.engines[res.instance_index]
            dst = getattr(target, "engine", None)
            t0, n = time.perf_counter(), 0
            if src is not None and dst is not None and hasattr(src, "migrate_prefix_to"):
                n = src.migrate_prefix_to(dst, ctx)
            elif src is not None and hasattr(src, "export_prefix") and hasattr(target, "import_prefix"):
                n = self._migrate_to_server(src, target, ctx)
            self.kv_migrations["count"] += 1 if n else 0
            self.kv_migrations["tokens"] += n
            self.kv_migrations["seconds"] += time.perf_counter() - t0
        return res

    def _migrate_to_server(self, src, target, ctx) -> int:
        """In-process engine -> server instance (e.g. a TP-k process group): the
        prefix's KV goes through a file in shared memory, which every server
        rank reads for its own KV heads.  Failures leave the request to
        recompute its prefix on the target."""
        import shutil
        import tempfile

        kv = src.kv
        need = 2 * len(ctx) * kv.num_layers * kv.kv_heads * kv.head_dim * kv.k.element_size()
        root = tempfile.gettempdir()
        try:  # shared memory when it has room (container /dev/shm is often small), else the temp dir
            if os.access("/dev/shm", os.W_OK) and shutil.disk_usage("/dev/shm").free > 2 * need:
                root = "/dev/shm"
        except OSError:
            pass
        path = os.path.join(root, f"libra_kv_{os.getpid()}_{uuid.uuid4().hex}.safetensors")
        try:
            payload = src.export_prefix(ctx, path)
            return target.import_prefix(payload) if payload["tokens"] else 0
        except (OSError, ValueError, RuntimeError) as exc:
            log.warning("KV migration to %s failed (%s); the request recomputes its prefix",
                        getattr(target, "instance_id", "?"), exc)
            return 0
        finally:
            if os.path.exists(path):
                os.unlink(path)

    def route_cmlfq_tool_return(self, request_id: str, tool_result: Any, generated_tokens: int):
        decision = self.on_tool_return(request_id, tool_result, generated_tokens)
        if decision is not None and decision.should_migrate:
            self.execute_cmlfq_migration(request_id, decision)
        return decision

    def finish_cmlfq_request(self, request_id: str, total_output_tokens: int) -> None:
        self._contexts.pop(request_id, None)
        if request_id and hasattr(self.scheduler, "finish_request"):
            with self._lock:
                self.scheduler.finish_request(request_id, total_output_tokens)

    def cancel_cmlfq_request(self, request_id: str) -> None:
        self._contexts.pop(request_id, None)
        if request_id and hasattr(self.scheduler, "cancel_request"):
            with self._lock:
                self.scheduler.cancel_request(request_id)

    def on_epoch_start(self, epoch: int) -> None:
        self.scheduler.on_epoch_start(epoch)

    def on_epoch_end(self, epoch: int) -> None:
        self.scheduler.on_epoch_end(epoch)

    # -------------------------------------------------------------- pool management
    def wait_until_idle(self, timeout: float = 3600.0) -> None:
        deadline = time.monotonic() + timeout
        while True:
            with self._inflight_lock:
                busy = self._inflight
            if busy == 0:
                return
            if time.monotonic() > deadline:
                raise TimeoutError(f"rollout pool still has {busy} requests in flight")
            time.sleep(0.01)

    def wait_for_ready(self, timeout: float = 300.0) -> bool:
        return all(getattr(e, "wait_for_ready", lambda t: True)(timeout) for e in self.engines)

    def reconfigure_from_plan(self, engines: List[Any], instance_configs: List[Dict[str, Any]],
                              scheduler: Optional[BaseScheduler] = None) -> None:
        """Swap to a new instance set (call after draining)."""
        self.wait_until_idle()
        with self._lock:
            if scheduler is None:
                scheduler = type(self.scheduler).__new__(type(self.scheduler))
                scheduler.__dict__.update(self.scheduler.__dict__)
                scheduler._instances, scheduler._instances_by_tp = [], type(self.scheduler._instances_by_tp)(list)
            self.scheduler = scheduler
            self.engines = list(engines)
            self.instance_configs = [dict(c) for c in instance_configs]
            for i, c in enumerate(self.instance_configs):
                self.scheduler.register_instance(i, c["instance_id"], int(c["tp_degree"]))

    def instance_loads(self) -> List[Dict[str, Any]]:
        out = []
        for e, c in zip(self.engines, self.instance_configs):
            inner = getattr(e, "engine", None)
            out.append({"instance_id": c["instance_id"], "tp": c["tp_degree"],
                        **(inner.load() if inner is not None and hasattr(inner, "load") else {})})
        return out

    # -------------------------------------------------------------- construction
    @classmethod
    def from_config(cls, config, engine_factory=None) -> "HeterogeneousRolloutEngine":
        """Build the pool from ``heterogeneous_rollout``.

        ``rollout_backend``: ``mock`` -> mocks; ``native`` -> in-process engines
        created by ``engine_factory(instance_config)`` (the trainer passes one
        that places weights on the instance's GPUs); anything else -> HTTP
        clients of ``host:port`` (``HETERO_INSTANCE_HOSTS`` may override hosts,
        comma separated, one per instance).
        """
        from libra_b200.engine.rollout_engine import HTTPRolloutEngine, MockRolloutEngine

        h = config.heterogeneous_rollout
        stype = h.scheduling.scheduler_type
        scheduler = SchedulerFactory.create(stype, h)
        hosts = [x.strip() for x in os.environ.get("HETERO_INSTANCE_HOSTS", "").split(",") if x.strip()]
        engines, cfgs = [], []
        for i, inst in enumerate(h.instances):
            host = hosts[i] if i < len(hosts) else (inst.host or h.vllm_host)
            port = inst.port or h.vllm_base_port + i
            cfgs.append({"instance_id": inst.instance_id, "tp_degree": inst.tp, "gpus": list(inst.gpus),
                         "host": host, "port": port})
            if config.rollout_backend == "mock":
                engines.append(MockRolloutEngine())
            elif config.rollout_backend in ("native", "local"):
                if engine_factory is None:
                    raise ValueError("native rollout backend needs an engine_factory")
                engines.append(engine_factory(inst))
            else:
                engines.append(HTTPRolloutEngine(host, port, config.model_path, instance_id=inst.instance_id))
        return cls(engines, cfgs, scheduler)
