"""Asynchronous GRPO trainer (the orchestrator).

Step structure follows the reference (``trainer/async_rl_trainer.py:741-1022``):
collect complete GRPO groups through the staleness-bounded dispatcher ->
distribute to data-parallel ranks -> group-normalised advantages -> logprob
recompute -> ``grpo_update`` -> (every ``sync_interval`` steps) drain rollouts,
sync weights, bump the policy version, resume -> history / phase trace ->
Global Resource Planner -> periodic checkpoint.

Single-box process model:

* one trainer process per training GPU (torchrun); NCCL between training GPUs,
  gloo on CPU;
* rollout instances are either in-process engines on the rollout GPUs owned by
  rank 0 (``rollout_backend: native``), one engine per training GPU sharing it
  with that rank's trainer (``rollout_backend: colocated``: every rank
  generates its own data-parallel slice and the weight sync is one device copy
  of the flat parameter buffer), HTTP servers (``vllm`` / ``http``), or mocks.
  With ``native`` engines rank 0 is the only batch source: it collects the
  global batch and scatters the data-parallel slices;
* weight sync for in-process engines is a device-to-device copy of the
  trainer's parameters into each instance's buffers (NVLink peer copies); for
  HTTP instances the trainer writes a versioned HF export and calls
  ``/reload_weights`` on every instance.
"""

from __future__ import annotations

import copy
import datetime
import itertools
import json
import os
import threading
import time
from collections import defaultdict
from concurrent.futures import Future, ThreadPoolExecutor
from pathlib import Path
from typing import Any, Dict, List, Optional

import torch
import torch.distributed as dist

from libra_b200.config import AsyncRLConfig
from libra_b200.infra.execution.async_runner import AsyncTaskRunner
from libra_b200.infra.execution.batch_dispatcher import BatchTaskDispatcher, TaskInput
from libra_b200.infra.observability.history_collector import HistoryDataCollector
from libra_b200.infra.observability.phase_tracer import PhaseTracer
from libra_b200.infra.sync.staleness import StalenessManager
from libra_b200.utils.snapshot import snapshot
from libra_b200.utils import nvtx


def compute_group_advantages(trajectories: List[Dict[str, Any]]) -> Dict[str, float]:
    """(r - mean) / (std + 1e-6) within each GRPO group; zero-variance groups -> 0;
    singleton groups keep the raw reward (reference ``trainer/async_rl_trainer.py:557-598``)."""
    groups: Dict[str, List[int]] = defaultdict(list)
    for i, t in enumerate(trajectories):
        r = t["rewards"].reshape(-1)
        if r.numel() != 1:
            raise ValueError("The current GRPO implementation requires exactly one outcome reward per trajectory")
        groups[str(t.get("grpo_group_id", f"singleton:{i}"))].append(i)
    zero_var = singles = 0
    for idx in groups.values():
        scores = torch.stack([trajectories[i]["rewards"].reshape(-1).float()[0] for i in idx])
        if len(idx) == 1:
            adv = scores
            singles += 1
        else:
            std = scores.std()
            if not torch.isfinite(std) or std <= 1e-6:
                adv = torch.zeros_like(scores)
                zero_var += 1
            else:
                adv = (scores - scores.mean()) / (std + 1e-6)
        for i, a in zip(idx, adv):
            trajectories[i]["advantages"] = a.reshape(1)
    return {"grpo_num_groups": len(groups), "grpo_mean_group_size": len(trajectories) / max(len(groups), 1),
            "grpo_singleton_groups": singles, "grpo_zero_variance_groups": zero_var}


class AsyncRLTrainer:
    def __init__(self, config: AsyncRLConfig, train_engine=None, rollout_engine=None, process_launcher=None):
        self.config = config
        self.rank = int(os.environ.get("RANK", "0"))
        self.local_rank = int(os.environ.get("LOCAL_RANK", "0"))
        self.world_size = int(os.environ.get("WORLD_SIZE", "1"))
        self.is_main_process = self.rank == 0
        self.train_engine = train_engine
        self.rollout_engine = rollout_engine
        self._local_engines: List[Any] = []
        self._tp_groups: List[Any] = []  # TP-k rollout buckets running as server process groups
        self.last_hybrid_dispatch: Optional[Dict[str, Any]] = None  # the latest batch share given to hybrids
        self.staleness_manager: Optional[StalenessManager] = None
        self.async_runner: Optional[AsyncTaskRunner] = None
        self.dispatcher: Optional[BatchTaskDispatcher] = None
        self.workflow = None
        self.global_step = 0
        self.stats: Dict[str, Any] = {}
        self._tracker = None
        self.start_step = int(os.environ.get("RL_TRAIN_START_STEP", "0") or 0)
        self.resumed_from: Optional[int] = None
        self.initial_model_version = int(os.environ.get("RL_INITIAL_MODEL_VERSION", str(self.start_step))
                                         or self.start_step)
        self._task_counter = itertools.count()
        self._pending_groups: Dict[str, List[Dict[str, Any]]] = {}
        self._advantage_stats: Dict[str, float] = {}
        self.history_collector: Optional[HistoryDataCollector] = None
        self.global_resource_planner = None
        self.runtime_elastic_executor = None
        self.process_launcher = process_launcher  # the executor's launcher (tests inject a fake one)
        self.calibrator = None
        self.reconfigurations: List[Dict[str, Any]] = []
        self._pending_decision = None
        self._grp_pool: Optional[ThreadPoolExecutor] = None
        self._grp_future: Optional[Future] = None
        trace = os.environ.get("RL_TRAIN_PHASE_TRACE", "0") == "1" or bool(config.phase_trace_enabled)
        trace_dir = (os.environ.get("RL_TRAIN_PHASE_TRACE_DIR", "") or config.phase_trace_dir
                     or os.path.join(config.log_dir, "phase_trace"))
        self._tracer = PhaseTracer(Path(trace_dir) / f"phase_trace_rank{self.rank}.jsonl", rank=self.rank,
                                   world_size=self.world_size) if trace else None
        self._single_batch_source = False
        self._nvtx_open: Dict[Any, Optional[int]] = {}
        # optional hook called at the end of every step: (step, stats, batch) on every rank
        self.step_callback = None

    # ================================================================== setup
    def _trace(self, step: int, name: str, **details) -> None:
        if nvtx.enabled():
            if name.endswith("_start"):
                self._nvtx_open[(step, name[:-6])] = nvtx.range_start(f"{name[:-6]}[{step}]")
            elif name.endswith("_done"):
                nvtx.range_end(self._nvtx_open.pop((step, name[:-5]), None))
        if self._tracer is None:
            return
        if name.endswith("_start"):
            self._tracer.start(step, name[:-6], details)
        elif name.endswith("_done"):
            self._tracer.end(step, name[:-5], details)

    def _init_distributed(self) -> None:
        if self.world_size <= 1 or (dist.is_available() and dist.is_initialized()):
            return
        timeout = datetime.timedelta(seconds=float(os.environ.get("TORCH_DISTRIBUTED_TIMEOUT", "1800")))
        use_cuda = torch.cuda.is_available() and os.environ.get("DIST_BACKEND", "") != "gloo"
        if use_cuda:
            torch.cuda.set_device(self.local_rank)
        dist.init_process_group("nccl" if use_cuda else "gloo", timeout=timeout)

    def _check_preflight(self) -> None:
        p = self.config.global_resource_planner
        if p.enabled and p.initial_allocation_strategy == "grp" and not p.initial_allocation_applied:
            raise RuntimeError("global_resource_planner.initial_allocation_strategy='grp' requires the GRP "
                               "preflight plan (PreflightPlanner) to be applied before training starts")

    def _make_tp_bucket(self, inst) -> Any:
        """A TP-k bucket (k > 1) as k server processes, one per GPU of ``inst.gpus``
        (``engine/tp_bucket.py``), reached through the HTTP client; the trainer
        syncs weights into it over NVLink (or from a checkpoint on CPU ranks)."""
        from libra_b200.engine.tp_bucket import TPServerGroup

        c = self.config
        eng = self.train_engine
        cuda = torch.cuda.is_available() and eng.device.type == "cuda"
        log_dir = os.path.join(c.log_dir, "rollout_servers")
        os.makedirs(log_dir, exist_ok=True)
        name = getattr(inst, "instance_id", "") or f"tp{inst.tp}-" + "-".join(str(g) for g in inst.gpus)
        group = TPServerGroup(os.path.basename(str(c.model_path)) or "qwen3-4b", int(inst.tp), list(inst.gpus),
                              kv_memory_fraction=float(c.heterogeneous_rollout.gpu_memory_utilization) * 0.5,
                              device="cuda" if cuda else "cpu", log_path=os.path.join(log_dir, f"{name}.log"),
                              startup_timeout=float(c.heterogeneous_rollout.startup_timeout))
        self._tp_groups.append(group)
        return group.client(instance_id=name)

    def _hetero_tp_buckets(self) -> bool:
        """Whether the config starts TP-k server groups (same answer on every rank)."""
        c = self.config
        return (c.rollout_backend in ("native", "local") and bool(c.heterogeneous_rollout.enabled)
                and any(int(getattr(i, "tp", 1) or 1) > 1 for i in c.heterogeneous_rollout.instances)
                and os.environ.get("LIBRA_TP_BUCKET_PROCESSES", "1") != "0")

    def _sync_tp_groups(self, version: int) -> None:
        """Weight sync into the TP-k server groups.  Collective over the trainer
        ranks (the peer request gathers every trainer TP rank's buffer handle;
        the disk path writes a distributed checkpoint); rank 0, which owns the
        rollout pool, posts it."""
        if not self._hetero_tp_buckets():
            return
        eng = self.train_engine
        timeout = float(self.config.rollout_weight_sync_timeout_s)
        if eng.flat_param.is_cuda:
            from libra_b200.infra.sync.peer_weight_sync import publish

            req = publish(eng)
            req["version"] = int(version)
            for group in self._tp_groups:  # each server rank pulls its own TP slice over NVLink
                group.reload_peer(req, timeout=timeout)
        else:
            from libra_b200.engine.checkpointing import DistributedCheckpointManager

            vdir = DistributedCheckpointManager(self.config.sync_path).save(
                eng, int(version), export_for_rollout=True, include_optimizer=False, export_only=True)
            for group in self._tp_groups:
                group.reload_disk(str(vdir), int(version), timeout=timeout)

    def _make_local_engine(self, inst) -> Any:
        """In-process rollout instance on the first GPU of ``inst.gpus`` with its own weight copy;
        TP-k instances (k > 1) become server groups (``_make_tp_bucket``)."""
        from libra_b200.engine.rollout.llm_engine import LLMEngine
        from libra_b200.engine.rollout_engine import LocalRolloutEngine
        from libra_b200.engine.tokenizer import load_tokenizer

        if int(getattr(inst, "tp", 1) or 1) > 1 and os.environ.get("LIBRA_TP_BUCKET_PROCESSES", "1") != "0":
            return self._make_tp_bucket(inst)
        eng = self.train_engine
        if torch.cuda.is_available() and getattr(inst, "gpus", None):
            dev = torch.device("cuda", int(inst.gpus[0]) % torch.cuda.device_count())
        else:
            dev = eng.device
        src = getattr(self, "_full_export", None) or {k: v.detach() for k, v in eng.params.items()}
        params = {k: v.to(dev, copy=True) for k, v in src.items()}
        tok = load_tokenizer(self.config.tokenizer_path, eng.cfg.vocab_size)
        llm = LLMEngine(eng.cfg, params, instance_id=getattr(inst, "instance_id", "") or f"local-{dev}",
                        kv_memory_fraction=float(self.config.heterogeneous_rollout.gpu_memory_utilization) * 0.5,
                        eos_token_id=None, max_model_len=int(self.config.max_seq_length) or 0)
        llm.version = eng.get_version()
        self._local_engines.append(llm)
        return LocalRolloutEngine(llm, tok)

    def _make_colocated_engine(self) -> Any:
        """Rollout engine on this rank's own GPU with its own copy of the trainer's
        flat bf16 weights (same layout, so a weight sync is one device copy)."""
        from libra_b200.engine.rollout.llm_engine import LLMEngine
        from libra_b200.engine.rollout.kv_cache import PagedKVCache
        from libra_b200.engine.rollout_engine import LocalRolloutEngine
        from libra_b200.engine.tokenizer import load_tokenizer

        eng = self.train_engine
        if int(getattr(eng, "tp_size", 1)) != 1 or int(getattr(eng, "pp_size", 1)) != 1:
            raise ValueError("rollout_backend='colocated' runs a full model per GPU: use train_tp_size=1 and "
                             "train_pp_size=1")
        c = self.config
        flat = eng.flat_param.detach().clone()
        cfg = eng.cfg
        max_len = int(c.max_seq_length)
        kv_blocks = 0
        if flat.is_cuda:
            free, _ = torch.cuda.mem_get_info(flat.device)
            # the trainer shares this GPU: the KV cache takes at most ~45 % of what initialisation left free
            frac = min(0.45, float(c.heterogeneous_rollout.gpu_memory_utilization) or 0.45)
            budget = PagedKVCache.blocks_for_budget(free * frac, cfg.num_hidden_layers, 16, cfg.num_key_value_heads,
                                                    cfg.head_dim)
            need = int(c.max_concurrent_rollouts or 256) * -(-max_len // 16) + 64
            kv_blocks = max(64, min(budget, need))
        tok = load_tokenizer(c.tokenizer_path, cfg.vocab_size)
        llm = LLMEngine(cfg, eng.layout.views(flat), kv_blocks=kv_blocks, block_size=16, max_model_len=max_len,
                        max_running=max(1, min(512, int(c.max_concurrent_rollouts or 256))),
                        instance_id=f"colocated-{self.rank}", flat=flat)
        llm.version = eng.get_version()
        self._local_engines.append(llm)
        return LocalRolloutEngine(llm, tok)

    def _build_rollout_engine(self) -> None:
        from libra_b200.engine.heterogeneous_engine import HeterogeneousRolloutEngine
        from libra_b200.engine.rollout_engine import HTTPRolloutEngine, MockRolloutEngine, MultiInstanceRolloutEngine

        c = self.config
        if c.rollout_backend == "colocated":
            self.rollout_engine = self._make_colocated_engine()
            return
        native = c.rollout_backend in ("native", "local")
        self._single_batch_source = native and self.world_size > 1
        if native and not self.is_main_process:
            return  # rank 0 owns the in-process rollout pool
        if c.heterogeneous_rollout.enabled and c.heterogeneous_rollout.instances:
            self.rollout_engine = HeterogeneousRolloutEngine.from_config(c, engine_factory=self._make_local_engine)
        elif c.rollout_backend == "mock":
            self.rollout_engine = MockRolloutEngine()
        elif native:
            from types import SimpleNamespace

            gpus = [int(x) for x in c.rollout_gpu_ids.split(",") if x.strip()] if c.rollout_gpu_ids else []
            self.rollout_engine = self._make_local_engine(SimpleNamespace(gpus=gpus, instance_id="native-0"))
        else:
            n = max(1, c.vllm_num_instances)
            eps = [e.strip() for e in c.vllm_endpoints.split(",") if e.strip()] or \
                  [f"{c.vllm_host}:{c.vllm_port + i}" for i in range(n)]
            self.rollout_engine = MultiInstanceRolloutEngine(
                [HTTPRolloutEngine(e.split(":")[0], int(e.split(":")[1]), c.model_path) for e in eps])

    def setup(self, workflow) -> None:
        self._check_preflight()
        self._init_distributed()
        self.workflow = workflow
        if self.train_engine is None:
            from libra_b200.engine.train_engine import create_train_engine

            self.train_engine = create_train_engine(self.config)
            self.train_engine.initialize(max_seq_length=self.config.max_seq_length)
        self._resume_from_checkpoint()
        self.train_engine.set_version(self.initial_model_version)
        if self.rollout_engine is None:
            # a TP- or pipeline-sharded trainer hands in-process rollout engines the full model (collective)
            self._full_export = self._export_full_params() if self.config.rollout_backend in ("native", "local") \
                else None
            self._build_rollout_engine()
            self._full_export = None
            # TP-k server groups start from their own initialisation: give them the trainer's weights
            self._sync_tp_groups(self.initial_model_version)
        else:
            from libra_b200.engine.rollout_engine import LocalRolloutEngine

            if isinstance(self.rollout_engine, LocalRolloutEngine) and self.rollout_engine.engine not in \
                    self._local_engines:
                self._local_engines.append(self.rollout_engine.engine)  # weight sync targets it directly
        if self.rollout_engine is not None and hasattr(self.rollout_engine, "wait_for_ready"):
            self.rollout_engine.wait_for_ready(float(self.config.heterogeneous_rollout.startup_timeout))
        if self._is_batch_source():
            local = self._collect_size()
            self.staleness_manager = StalenessManager(self.train_engine, self.config.max_concurrent_rollouts, local,
                                                      self.config.max_head_offpolicyness)
            self.async_runner = AsyncTaskRunner(max_queue_size=self.config.queue_size,
                                                enable_tracing=self.config.enable_rollout_tracing)
            self.async_runner.initialize()
            self.dispatcher = BatchTaskDispatcher(self.async_runner, self.staleness_manager,
                                                  self._create_rollout_task, self.config.enable_rollout_tracing)
            self.dispatcher.initialize()
        if self.is_main_process and self.config.enable_history_collection:
            out = self.config.history_output_dir or os.path.join(self.config.log_dir, "history")
            p = self.config.global_resource_planner
            self.history_collector = HistoryDataCollector(
                out, self.config.history_save_raw_lengths, self.config.history_flush_interval,
                self.config.history_experiment_name,
                (p.runtime_length_profile_jsonl or os.path.join(out, "runtime_length_profile.jsonl"))
                if p.runtime_length_profile_enabled else "")
            self.history_collector.initialize()
        if self.is_main_process and self.config.global_resource_planner.enabled:
            from libra_b200.infra.cost_model.global_resource_planner import GlobalResourcePlanner

            self.global_resource_planner = GlobalResourcePlanner.from_config(self.config)
            if self.config.global_resource_planner.runtime_async_planning:
                self._grp_pool = ThreadPoolExecutor(max_workers=1, thread_name_prefix="grp")
            if self.config.global_resource_planner.runtime_dynamic_reconfiguration_enabled:
                # online replanning: rank 0 applies the planner's decisions between steps
                from libra_b200.infra.elastic.runtime_executor import RuntimeElasticExecutor

                self.runtime_elastic_executor = RuntimeElasticExecutor(
                    config=self.config, planner=self.global_resource_planner, train_engine=self.train_engine,
                    rollout_engine=self.rollout_engine, dispatcher=self.dispatcher, launcher=self.process_launcher)
            from libra_b200.infra.cost_model.calibrator import ShadowCalibrator

            self.calibrator = ShadowCalibrator()

    def _is_batch_source(self) -> bool:
        if self._single_batch_source:
            return self.is_main_process
        return self.train_engine.is_batch_source()

    def _collect_size(self) -> int:
        if self._single_batch_source:
            return int(self.config.batch_size)
        return self.train_engine.get_local_batch_size(self.config.batch_size)

    # ================================================================== rollout tasks
    def _create_rollout_task(self, task_input: TaskInput):
        workflow, sm, eng = self.workflow, self.staleness_manager, self.train_engine
        max_stale = self.config.max_head_offpolicyness

        async def _execute():
            try:
                traj = await workflow.run_episode(self.rollout_engine, task_input.data, version=task_input.version,
                                                  rollout_index=task_input.rollout_index)
                traj["grpo_group_id"] = task_input.group_id or f"task:{task_input.task_id}"
                traj["grpo_rollout_index"] = task_input.rollout_index
                v = int(traj.get("versions", torch.tensor([task_input.version])).min())
                if eng.get_version() - v <= max_stale:
                    sm.on_rollout_accepted()
                    return traj
                sm.on_rollout_rejected()
                return None
            except Exception as exc:  # noqa: BLE001 - a failed rollout is a rejected rollout
                sm.on_rollout_rejected()
                if self.is_main_process:
                    print(f"ERROR: Rollout task_id={task_input.task_id} failed: {exc}")
                return None

        return _execute

    def _data_generator(self, dataset):
        n = int(self.config.n_samples)
        if n < 1:
            raise ValueError(f"n_samples must be positive; got {n}")
        dp_rank = 0 if self._single_batch_source else self.train_engine.get_data_parallel_rank()
        dp_size = 1 if self._single_batch_source else self.train_engine.get_data_parallel_world_size()
        g = torch.Generator().manual_seed(int(self.config.seed))
        for epoch in itertools.count():
            order = torch.randperm(len(dataset), generator=g).tolist()[dp_rank::dp_size]
            for sample_index, idx in enumerate(order):
                item = dataset[idx]
                if not isinstance(item, dict):
                    raise TypeError("GRPO items must be dictionaries so that a stable group ID can be attached")
                gid = f"dp{dp_rank}:epoch{epoch}:sample{sample_index}"
                for r in range(n):
                    yield TaskInput(task_id=next(self._task_counter), data=item, version=self.train_engine.get_version(),
                                    group_id=gid, rollout_index=r)

    def _collect_complete_grpo_batch(self, data_gen, batch_size: int) -> List[Dict[str, Any]]:
        n = int(self.config.n_samples)
        p = self.config.global_resource_planner
        timeout = float(p.runtime_batch_collection_timeout_s)
        retries_left = int(p.runtime_batch_collection_max_retries)
        chosen: List[Dict[str, Any]] = []
        while len(chosen) < batch_size:
            try:
                raw = self.dispatcher.active_submit_and_wait(data_gen, batch_size, timeout if timeout > 0 else None)
            except TimeoutError:
                self.dispatcher.reset_after_reconfigure()
                if retries_left <= 0:
                    raise
                retries_left -= 1
                continue
            self.staleness_manager.on_batch_consumed(len(raw))
            for t in raw:
                self._pending_groups.setdefault(str(t["grpo_group_id"]), []).append(t)
            for gid in list(self._pending_groups):
                members = self._pending_groups[gid]
                if len(members) < n:
                    continue
                if batch_size - len(chosen) < n:
                    break
                chosen.extend(members[:n])
                del self._pending_groups[gid]
            while len(self._pending_groups) > max(64, batch_size * 8):
                del self._pending_groups[next(iter(self._pending_groups))]
        return chosen

    def _distribute(self, batch):
        """Scatter data-parallel slices (whole groups) when rank 0 is the only
        batch source: one slice per data-parallel replica, so the tensor-parallel
        ranks and pipeline stages of a replica all receive the same trajectories."""
        if not self._single_batch_source:
            return self.train_engine.distribute_trajectories(batch)
        dp = max(1, int(self.train_engine.get_data_parallel_world_size()))
        payload = [None]
        if self.is_main_process:
            per = len(batch) // dp
            payload = [[batch[d * per:(d + 1) * per] for d in range(dp)]]
        dist.broadcast_object_list(payload, src=0)
        return payload[0][int(self.train_engine.get_data_parallel_rank())]

    # ================================================================== elastic hybrid replicas
    def _dispatch_hybrid(self, batch, step: int):
        """Share this replica's batch with its active hybrid replicas (Elastic
        Hybrid Pool): whole GRPO groups are dealt round-robin between the core
        and each hybrid, every hybrid gets its share as a task file, and the
        core trains the rest; before the optimizer step the engine waits
        (bounded) for the hybrids' gradients and averages them with its own.
        Returns the core's share (the whole batch when no hybrid is active)."""
        eng = self.train_engine
        dom = getattr(eng, "elastic_gradient_domain", None)
        if dom is None or not batch:
            return batch
        hybrids = list(dom.active_hybrid_ids_for_core(f"dp{eng.get_data_parallel_rank()}"))
        if not hybrids:
            eng.elastic_payload_wait_s, eng.elastic_average_merged = 0.0, False
            return batch
        from libra_b200.infra.elastic.worker import write_task

        groups: Dict[Any, List[Any]] = {}
        for t in batch:
            groups.setdefault(t.get("grpo_group_id", id(t)), []).append(t)
        shares: List[List[Any]] = [[] for _ in range(len(hybrids) + 1)]
        for i, g in enumerate(groups.values()):
            shares[i % len(shares)].extend(g)
        p = self.config.global_resource_planner
        task_dir = p.hybrid_worker_task_dir
        nxt = int(eng.step_count) + 1
        sent = 0
        for rid, part in zip(hybrids, shares[1:]):
            if part:
                write_task(task_dir, rid, nxt, part, state_version=int(eng.get_version()),
                           membership_epoch=dom.membership_epoch(rid))
                sent += len(part)
        eng.elastic_payload_wait_s = float(p.hybrid_active_gradient_timeout_s)
        eng.elastic_average_merged = True
        self.last_hybrid_dispatch = {"step": step, "hybrids": hybrids, "core": len(shares[0]),
                                     "hybrid_trajectories": sent}
        return shares[0] or batch

    # ================================================================== weight sync
    def _export_full_params(self):
        """Full-model parameters when the trainer is TP- or pipeline-sharded (collective over the first
        replica; rank 0 gets the model), else None."""
        eng = self.train_engine
        if int(getattr(eng, "tp_size", 1)) > 1 or int(getattr(eng, "pp_size", 1)) > 1 or \
                int(getattr(eng, "ep_size", 1)) > 1:
            return eng.export_params()
        return None

    def _sync_weights(self, target_version: int) -> float:
        """Push the trainer's weights to every rollout instance; returns seconds."""
        t0 = time.perf_counter()
        full = self._export_full_params() if self.config.rollout_backend in ("native", "local") else None
        if full is not None and self._local_engines:
            for llm in self._local_engines:
                llm.update_weights(full, version=target_version)
        elif self._local_engines:
            # in-process instances: one copy of the flat buffer when the layouts match, else per tensor
            # (device-to-device; NVLink peer copies across GPUs)
            src_flat = getattr(self.train_engine, "flat_param", None)
            src = None
            for llm in self._local_engines:
                if llm.flat is not None and src_flat is not None and llm.flat.numel() == src_flat.numel():
                    llm.load_flat_weights(src_flat, version=target_version)
                else:
                    src = src or {k: v.detach() for k, v in self.train_engine.params.items()}
                    llm.update_weights(src, version=target_version)
        elif self.config.rollout_backend not in ("mock",) and not self._hetero_tp_buckets() and (
                self.config.rollout_weight_sync_mode != "none" or self.config.require_rollout_weight_sync):
            self._sync_weights_disk(target_version)
        self._sync_tp_groups(target_version)
        return time.perf_counter() - t0

    def _sync_weights_disk(self, version: int) -> None:
        from libra_b200.engine.checkpointing import DistributedCheckpointManager

        mgr = DistributedCheckpointManager(self.config.sync_path)
        vdir = mgr.save(self.train_engine, version, export_for_rollout=True,
                        include_optimizer=False, export_only=self.config.rollout_weight_sync_export_only)
        if self.is_main_process and self.rollout_engine is not None:
            from libra_b200.infra.sync.weight_sync import reload_http_instances

            reload_http_instances(self.rollout_engine, str(vdir), version,
                                  timeout=self.config.rollout_weight_sync_timeout_s)

    # ================================================================== main loop
    def train(self, workflow, dataset=None) -> Dict[str, Any]:
        self.setup(workflow)
        if dataset is None:
            raise ValueError("dataset cannot be None")
        c = self.config
        if not 0 <= self.start_step < c.total_steps:
            raise ValueError(f"RL_TRAIN_START_STEP must be in [0, total_steps): start_step={self.start_step}, "
                             f"total_steps={c.total_steps}")
        gen = self._data_generator(dataset) if self._is_batch_source() else None
        local = self.train_engine.get_local_batch_size(c.batch_size)
        if local % int(c.n_samples):
            raise ValueError(f"Each data-parallel replica's local batch size must be divisible by n_samples: "
                             f"local_batch_size={local}, n_samples={c.n_samples}")
        t_start = time.time()
        for step in range(self.start_step, c.total_steps):
            self.global_step = step
            t_step = time.time()
            self._trace(step, "step_start")
            if hasattr(self.rollout_engine, "on_epoch_start"):
                self.rollout_engine.on_epoch_start(step)
            batch = None
            if self._is_batch_source():
                self._trace(step, "collect_batch_start")
                batch = self._collect_complete_grpo_batch(gen, self._collect_size())
                self._trace(step, "collect_batch_done", batch_size=len(batch))
            if batch is not None:
                self._advantage_stats = compute_group_advantages(batch)
            self._trace(step, "distribute_start")
            batch = self._distribute(batch)
            self._trace(step, "distribute_done", batch_size=len(batch or []))
            if not batch:
                continue
            batch = self.train_engine.align_distributed_trajectories(batch)
            batch = self._dispatch_hybrid(batch, step)
            rollout_time = time.time() - t_step
            t_adv = time.time()
            if not self._advantage_stats:
                self._advantage_stats = compute_group_advantages(batch)
            advantage_time = time.time() - t_adv
            recompute_time = 0.0
            if c.recompute_logprobs:
                t_r = time.time()
                self._trace(step, "recompute_logprobs_start")
                self.train_engine.recompute_logprobs(batch)
                recompute_time = time.time() - t_r
                self._trace(step, "recompute_logprobs_done", seconds=f"{recompute_time:.3f}")
            t_train = time.time()
            self._trace(step, "grpo_update_start")
            stats = self.train_engine.grpo_update(batch, ppo_epochs=c.ppo_epochs)
            rewards = torch.cat([t["rewards"].reshape(-1).float() for t in batch])
            stats.update({"reward_mean": float(rewards.mean()), "reward_std": float(rewards.std(unbiased=False)),
                          "reward_min": float(rewards.min()), "reward_max": float(rewards.max())})
            train_time = time.time() - t_train
            self._trace(step, "grpo_update_done", seconds=f"{train_time:.3f}")
            sync_time = 0.0
            if c.sync_interval > 0 and (step + 1) % c.sync_interval == 0:
                self._trace(step, "weight_sync_start")
                if self.dispatcher is not None:
                    self.dispatcher.pause()
                    self.dispatcher.wait_until_idle(timeout=float(c.rollout_weight_sync_timeout_s))
                if self.world_size > 1:
                    dist.barrier()
                sync_time = self._sync_weights(step + 1)
                self.train_engine.set_version(step + 1)
                if self.dispatcher is not None:
                    self.dispatcher.resume()
                self._trace(step, "weight_sync_done", seconds=f"{sync_time:.3f}")
            step_time = time.time() - t_step
            stats.update({"n_trajectories": len(batch), "rollout_time": rollout_time, "train_time": train_time,
                          "weight_sync_time": sync_time, "advantage_time": advantage_time,
                          "recompute_logprob_time": recompute_time, "step_time": step_time,
                          "version": self.train_engine.get_version(), **self._advantage_stats})
            self._advantage_stats = {}
            if self.resumed_from is not None:
                stats["resumed_from"] = self.resumed_from
            self.stats = stats
            if self.is_main_process:
                self._record_history(step, batch, stats)
                if self._tracker is None:
                    from libra_b200.utils.tracking import Tracker

                    self._tracker = Tracker.create(self.config, self.rank)
                self._tracker.log(stats, step)
                self._run_planner(step, batch, stats)
                if hasattr(self.rollout_engine, "on_epoch_end"):
                    self.rollout_engine.on_epoch_end(step)
                if step % 10 == 0 or c.total_steps <= 10 or step == c.total_steps - 1:
                    print(f"Step {step}/{c.total_steps}: {time.time() - t_start:.1f}s loss={stats.get('loss', 0):.4f} "
                          f"kl={stats.get('kl', 0):.4f} reward={stats['reward_mean']:.3f} "
                          f"n={len(batch)} rollout={rollout_time:.2f}s train={train_time:.2f}s", flush=True)
            self._apply_pending_reconfiguration(step)
            if self.step_callback is not None:
                self.step_callback(step, stats, batch)
            self._run_periodic_evaluation(workflow, dataset, step)
            if c.save_interval > 0 and (step + 1) % c.save_interval == 0:
                self._save_checkpoint(step)
        self.shutdown()
        return self.stats

    # ================================================================== evaluation
    def _run_periodic_evaluation(self, workflow, dataset, step: int) -> None:
        """Greedy evaluation on rank 0 every ``eval_interval`` steps (not step 0).

        Behaviour of the reference's ``trainer/async_rl_trainer.py:1034-1131``:
        rollout dispatch is paused; rank 0 runs ``workflow.evaluate`` with the
        ``EVAL_*`` environment settings, appends the summary to
        ``<log_dir>/eval/$EVAL_METRICS_FILE``, writes up to a few sample records
        to ``$EVAL_SAMPLES_FILE`` and drops ``eval_step_<step>.done`` (or
        ``.error`` with the message).  The other ranks poll for those files
        instead of sitting in a collective, so an evaluation longer than the
        process-group timeout does not kill the job.
        """
        interval = int(getattr(self.config, "eval_interval", 0) or 0)
        if interval <= 0 or step <= 0 or step % interval or not hasattr(workflow, "evaluate"):
            return
        if self.rollout_engine is None:
            return
        env = os.environ.get
        eval_dir = os.path.join(self.config.log_dir, "eval")
        done, error = (os.path.join(eval_dir, f"eval_step_{step}.{ext}") for ext in ("done", "error"))
        if self.dispatcher is not None:
            self.dispatcher.pause()
        try:
            if self.is_main_process:
                os.makedirs(eval_dir, exist_ok=True)
                for path in (done, error):
                    if os.path.exists(path):
                        os.remove(path)
                kw = dict(max_samples=int(env("EVAL_MAX_SAMPLES", "0")), concurrency=int(env("EVAL_CONCURRENCY", "16")),
                          accuracy_threshold=float(env("EVAL_ACCURACY_THRESHOLD", "0.5")),
                          max_new_tokens=int(env("EVAL_MAX_NEW_TOKENS", str(self.config.max_new_tokens))))
                try:
                    import asyncio

                    stats = asyncio.run(workflow.evaluate(self.rollout_engine, dataset, **kw))
                    stats["step"] = step
                    records = stats.pop("eval_records", [])
                    self.stats.update(stats)
                    print(f"[eval] step={step} accuracy={stats['eval_accuracy']:.4f} "
                          f"reward_mean={stats['eval_reward_mean']:.4f} failures={stats['eval_failures']} "
                          f"samples={stats['eval_samples']}", flush=True)
                    with open(os.path.join(eval_dir, env("EVAL_METRICS_FILE", "eval_metrics.jsonl")), "a",
                              encoding="utf-8") as f:
                        f.write(json.dumps(stats, ensure_ascii=False) + "\n")
                    if records:
                        with open(os.path.join(eval_dir, env("EVAL_SAMPLES_FILE", f"eval_samples_step_{step}.jsonl")),
                                  "w", encoding="utf-8") as f:
                            for r in records:
                                f.write(json.dumps(r, ensure_ascii=False) + "\n")
                    if self._tracker is not None:
                        self._tracker.log({k: v for k, v in stats.items() if isinstance(v, (int, float))}, step)
                    Path(done).write_text("ok\n", encoding="utf-8")
                except Exception as exc:
                    Path(error).write_text(f"{type(exc).__name__}: {exc}", encoding="utf-8")
                    raise
            else:
                limit = float(env("EVAL_WAIT_TIMEOUT", "86400"))
                poll = float(env("EVAL_WAIT_POLL_S", "2.0"))
                t0 = time.monotonic()
                while not os.path.exists(done) and not os.path.exists(error):
                    if time.monotonic() - t0 > limit:
                        raise TimeoutError(f"timed out waiting for the evaluation of step {step}")
                    time.sleep(poll)
                if os.path.exists(error):
                    raise RuntimeError(Path(error).read_text(encoding="utf-8"))
        finally:
            if self.dispatcher is not None:
                self.dispatcher.resume()

    # ================================================================== bookkeeping
    def _record_history(self, step: int, batch, stats) -> None:
        if self.history_collector is None:
            return
        seqs = [{"input_len": int(t.get("prompt_len", 0)), "output_len": int(t.get("output_len", 0)),
                 "prompt_id": str(t.get("prompt_id", "")), "total_output_tokens": int(t.get("total_output_tokens",
                                                                                            t.get("output_len", 0))),
                 "tool_returns": t.get("tool_events", [])} for t in batch]
        sm = self.staleness_manager.get_stats() if self.staleness_manager else None
        self.history_collector.record_step(
            step, sequence_records=seqs, rollout_time=stats["rollout_time"], train_time=stats["train_time"],
            weight_sync_time=stats["weight_sync_time"], advantage_time=stats["advantage_time"],
            recompute_logprob_time=stats["recompute_logprob_time"], step_total_time=stats["step_time"],
            training_stats=stats, pipeline_running=getattr(sm, "running", 0),
            pipeline_accepted=getattr(sm, "accepted", 0), pipeline_rejected=getattr(sm, "rejected", 0),
            model_version=self.train_engine.get_version(),
            resource_config=HistoryDataCollector.snapshot_resource_config(self.config))

    def _run_planner(self, step: int, batch, stats) -> None:
        grp = self.global_resource_planner
        if grp is None:
            return
        if self._grp_future is not None and self._grp_future.done():
            decision = self._grp_future.result()
            self._grp_future = None
            self._apply_decision(decision)
        grp.observe_batch([{"input_len": t.get("prompt_len", 0), "output_len": t.get("output_len", 0)} for t in batch])
        plan = grp.active_plan
        if self.calibrator is not None and plan is not None:
            # measured vs modelled phase times of the active plan: the calibrator's efficiencies rescale the
            # planner's B200 model before it is asked for the next decision
            from libra_b200.infra.cost_model.calibrator import EpochRunData

            self.calibrator.update(EpochRunData(
                t_train_real=float(stats["train_time"]) + float(stats.get("recompute_logprob_time", 0.0)),
                t_rollout_real=float(stats["rollout_time"]), t_train_predicted=float(plan.t_train),
                t_rollout_predicted=float(plan.t_rollout),
                gen_lengths=[float(t.get("output_len", 0)) for t in batch],
                prompt_lengths=[float(t.get("prompt_len", 0)) for t in batch], epoch_id=step))
            cm = getattr(getattr(grp, "evaluator", None), "analytic", None)
            if cm is not None:
                if not hasattr(self, "_calib_base"):
                    self._calib_base = (cm.training_model.train_mfu, cm.rollout_model.decode_bw_util)
                self.calibrator.apply_to_cost_model(cm, *self._calib_base)
        metrics = grp.observe_runtime(step=step, dispatcher_metrics=self.dispatcher.get_runtime_metrics()
                                      if self.dispatcher else {},
                                      step_stats={"rollout_time": stats["rollout_time"],
                                                  "train_time": stats["train_time"], "step_time": stats["step_time"],
                                                  "max_concurrent_rollouts": self.config.max_concurrent_rollouts})
        cfg = copy.deepcopy(self.config)
        if self._grp_pool is not None:
            if self._grp_future is None:
                self._grp_future = self._grp_pool.submit(grp.plan_if_needed, step, cfg, None, metrics)
        else:
            self._apply_decision(grp.plan_if_needed(step, cfg, None, metrics))

    def _apply_decision(self, decision) -> None:
        """Rank 0: log the planner's decision; a reconfiguration is applied at the
        end of the step by ``_apply_pending_reconfiguration`` with every rank."""
        self.last_planner_decision = decision
        log = os.path.join(self.config.log_dir, "global_resource_planner_decisions.jsonl")
        os.makedirs(self.config.log_dir, exist_ok=True)
        with open(log, "a", encoding="utf-8") as fh:
            fh.write(json.dumps(decision.to_dict(), default=str) + "\n")
        if self.runtime_elastic_executor is not None and (
                decision.should_reconfigure or getattr(decision, "elastic_hybrid_signal", None) is not None):
            self._pending_decision = decision

    def _apply_pending_reconfiguration(self, step: int) -> None:
        """Collective (every rank, end of step, outside any other collective).

        Rank 0 broadcasts whether the planner asked for a reconfiguration.  If
        so, rank 0 runs ``RuntimeElasticExecutor.execute`` — which, for
        strategies that move GPUs (cluster swap), posts a drain request and
        waits for the peer ranks' ready files — while the other ranks poll
        the coordination directory and answer requests
        (``follow_reconfiguration_request``) until rank 0 reaches the closing
        barrier.  The applied layout lands in the shared config object, so the
        next history record shows it."""
        flag = 1 if (self.is_main_process and self._pending_decision is not None) else 0
        if self.world_size > 1 and dist.is_initialized():
            dev = self.train_engine.device if getattr(self.train_engine, "device", None) is not None and \
                dist.get_backend() == "nccl" else torch.device("cpu")
            t = torch.tensor([flag], dtype=torch.int32, device=dev)
            dist.broadcast(t, src=0)
            flag = int(t.item())
        if not flag:
            return
        if self.is_main_process:
            decision, self._pending_decision = self._pending_decision, None
            try:
                result = self.runtime_elastic_executor.execute(decision)
                record = {"step": step, **result.to_dict(),
                          "layout": {"train_gpus": self.config.train_gpus, "rollout_gpus": self.config.rollout_gpus,
                                     "rollout_tp_list": list(self.config.heterogeneous_rollout.tp_list)}}
            except Exception as exc:  # noqa: BLE001 - a failed reconfiguration keeps the current layout
                record = {"step": step, "applied": False, "reason": f"error: {type(exc).__name__}: {exc}"}
            self.reconfigurations.append(record)
            self.stats["reconfiguration"] = record
            pool = getattr(self.runtime_elastic_executor, "elastic_pool", None)
            if pool is not None and getattr(self.train_engine, "elastic_gradient_domain", None) is None:
                self.train_engine.elastic_gradient_domain = pool.gradient_domain
            with open(os.path.join(self.config.log_dir, "runtime_reconfigurations.jsonl"), "a",
                      encoding="utf-8") as fh:
                fh.write(json.dumps(record, default=str) + "\n")
            if self.world_size > 1 and dist.is_initialized():
                dist.barrier()
            return
        from libra_b200.infra.elastic.runtime_executor import follow_reconfiguration_request

        p = self.config.global_resource_planner
        coord = getattr(p, "runtime_reconfiguration_coord_dir", "") or os.path.join(self.config.log_dir,
                                                                                    "runtime_reconfiguration")
        drain = None
        if self.dispatcher is not None:
            def drain(timeout=float(p.runtime_drain_timeout_s)):
                self.dispatcher.pause()
                self.dispatcher.wait_until_idle(timeout=timeout)
        work = dist.barrier(async_op=True)
        answered = set()
        while not work.is_completed():
            cid = None
            req = Path(coord) / "request.json"
            if req.exists():
                try:
                    cid = json.loads(req.read_text(encoding="utf-8")).get("coord_id")
                except (OSError, ValueError):
                    cid = None
            if cid and cid not in answered:
                follow_reconfiguration_request(coord, self.rank, drain=drain)
                answered.add(cid)
            time.sleep(0.02)
        work.wait()
        if drain is not None and answered:
            self.dispatcher.resume()

    def _resume_from_checkpoint(self) -> None:
        """Resume (collective): with ``RL_TRAIN_START_STEP=S > 0`` and a checkpoint
        version ``S`` under ``<log_dir>/checkpoints`` (written after step ``S - 1``),
        every rank loads its weights and optimizer state from it, whatever the
        parallel layout that wrote it.  Without one, the engine keeps the
        weights it was initialised with (``model_path``)."""
        if self.start_step <= 0:
            return
        from libra_b200.engine.checkpointing import DistributedCheckpointManager, all_versions

        root = os.path.join(self.config.log_dir, "checkpoints")
        if self.start_step not in all_versions(root):
            if self.is_main_process:
                print(f"RL_TRAIN_START_STEP={self.start_step}: no checkpoint v{self.start_step} under {root}; "
                      "starting from the initial weights")
            return
        DistributedCheckpointManager(root).load(self.train_engine, self.start_step)
        self.resumed_from = self.start_step
        if self.is_main_process:
            print(f"resumed from {root}/v{self.start_step}")

    def _save_checkpoint(self, step: int) -> None:
        from libra_b200.engine.checkpointing import DistributedCheckpointManager

        mgr = DistributedCheckpointManager(os.path.join(self.config.log_dir, "checkpoints"))
        mgr.save(self.train_engine, step + 1, export_for_rollout=False)
        if self.is_main_process:
            light = {"step": step, "version": self.train_engine.get_version(),
                     "stats": snapshot(self.stats),
                     "config": self.config.to_dict()}
            torch.save(light, os.path.join(self.config.log_dir, "checkpoints", f"step_{step}.pt"))
            mgr.prune(self.config.keep_latest_checkpoints, protect=self.start_step or None)

    def shutdown(self) -> None:
        if self.dispatcher is not None:
            self.dispatcher.destroy()
            self.dispatcher = None
        for llm in self._local_engines:
            llm.shutdown()
        for group in self._tp_groups:
            group.close()
        self._tp_groups = []
        if self._grp_pool is not None:
            self._grp_pool.shutdown(wait=False)
        if self.history_collector is not None:
            self.history_collector.close()
        if self._tracer is not None:
            self._tracer.close()
        if self._tracker is not None:
            self._tracker.finish()
