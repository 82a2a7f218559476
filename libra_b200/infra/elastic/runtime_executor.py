"""Runtime executor for Global Resource Planner decisions.

Behaviour of the reference's ``infra/elastic/runtime_executor.py``
(``execute:144-420``): accept the planner's elastic signal, pause/drain the
dispatcher, coordinate peer ranks through ``request.json`` / ``ready/`` /
``applied.json`` files, apply the plan to the runtime config, reconfigure the
rollout processes with one of the strategies

* ``diff`` / ``blue_green`` - start changed instances first (spare ports when
  the port is taken), cut the rollout engine over, then stop the old ones;
* ``restart_all`` - stop everything, start the new set;
* ``prewarm`` - start the new set on spare ports *before* pausing traffic,
  finish the cutover inside the short paused window; falls back to
  ``runtime_prewarm_no_spare_fallback_strategy`` when the GPUs do not fit;
* ``cluster_swap`` - no spare GPUs: stop surplus rollout instances and hand
  their GPUs to training slots (Elastic Hybrid Pool replicas);

and grow/shrink the training side in whole DP replicas through the
``ElasticHybridPool`` (or record the plan only).  Rollout instances are our
own ``libra_b200.engine.server`` processes bound to GPU subsets through
``CUDA_VISIBLE_DEVICES``; processes are started in their own session and
stopped by exact pid / process group, never by name.
"""

from __future__ import annotations

import copy
import json
import os
import shlex
import signal
import subprocess
import sys
import threading
import time
import urllib.request
from dataclasses import dataclass, field
from pathlib import Path
from typing import Any, Dict, List, Optional, Tuple


@dataclass
class ManagedRolloutProcess:
    instance_id: str
    command: str
    pid: int
    gpus: List[int]
    port: int
    host: str = "127.0.0.1"
    tp: int = 1
    adopted: bool = False
    log_path: str = ""


@dataclass
class ManagedHybridWorkerProcess:
    worker_id: str
    target_core_id: str
    command: str
    pid: int
    snapshot_path: str
    host: str = ""
    gpus: List[int] = field(default_factory=list)
    replica_id: str = ""
    replica_rank: int = 0
    replica_world_size: int = 1


@dataclass
class RuntimeReconfigurationResult:
    applied: bool
    reason: str
    actions: List[str] = field(default_factory=list)
    started_processes: List[ManagedRolloutProcess] = field(default_factory=list)
    stopped_processes: List[ManagedRolloutProcess] = field(default_factory=list)
    started_hybrid_workers: List[ManagedHybridWorkerProcess] = field(default_factory=list)
    training_actions: List[str] = field(default_factory=list)
    errors: List[str] = field(default_factory=list)

    def to_dict(self) -> Dict[str, Any]:
        return {"applied": self.applied, "reason": self.reason, "actions": list(self.actions),
                "started_processes": [vars(p) for p in self.started_processes],
                "stopped_processes": [vars(p) for p in self.stopped_processes],
                "started_hybrid_workers": [vars(p) for p in self.started_hybrid_workers],
                "training_actions": list(self.training_actions), "errors": list(self.errors)}


def write_json_atomic(path: Path, payload: Dict[str, Any]) -> None:
    path.parent.mkdir(parents=True, exist_ok=True)
    tmp = path.with_name(f".{path.name}.tmp")
    tmp.write_text(json.dumps(payload, sort_keys=True, indent=1), encoding="utf-8")
    os.replace(tmp, path)


# ============================================================================ process control
class ProcessLauncher:
    """Starts/stops rollout and hybrid-worker processes (replaceable in tests)."""

    def start(self, command: str, env: Dict[str, str], log_path: str = "") -> subprocess.Popen:
        out = None
        if log_path:
            Path(log_path).parent.mkdir(parents=True, exist_ok=True)
            out = open(log_path, "a", encoding="utf-8")
            out.write(f"\n[{time.strftime('%Y-%m-%d %H:%M:%S')}] {command}\n")
            out.flush()
        try:
            return subprocess.Popen(command, shell=True, env=env, stdout=out,
                                    stderr=subprocess.STDOUT if out else None, start_new_session=True)
        finally:
            if out is not None:
                out.close()

    def stop(self, proc: subprocess.Popen, timeout: float) -> None:
        """SIGTERM the process group the launcher created, SIGKILL after ``timeout``."""
        if proc.poll() is not None:
            return
        try:
            os.killpg(proc.pid, signal.SIGTERM)  # its own session: pgid == pid
        except ProcessLookupError:
            return
        try:
            proc.wait(timeout=timeout)
        except subprocess.TimeoutExpired:
            try:
                os.killpg(proc.pid, signal.SIGKILL)
            except ProcessLookupError:
                pass
            proc.wait(timeout=5)

    def stop_pid(self, pid: int, timeout: float) -> None:
        """Stop an adopted external process by its exact pid."""
        if pid <= 0:
            return
        try:
            os.kill(pid, signal.SIGTERM)
        except ProcessLookupError:
            return
        deadline = time.monotonic() + timeout
        while time.monotonic() < deadline:
            try:
                os.kill(pid, 0)
            except ProcessLookupError:
                return
            time.sleep(0.1)
        try:
            os.kill(pid, signal.SIGKILL)
        except ProcessLookupError:
            pass

    def run(self, command: str, timeout: float) -> int:
        return subprocess.run(command, shell=True, timeout=timeout).returncode

    def wait_ready(self, host: str, port: int, timeout: float) -> None:
        deadline = time.monotonic() + timeout
        url = f"http://{host}:{port}/health"
        while time.monotonic() < deadline:
            try:
                with urllib.request.urlopen(url, timeout=2) as r:
                    if r.status == 200:
                        return
            except OSError:
                pass
            time.sleep(0.5)
        raise TimeoutError(f"rollout endpoint {url} not ready after {timeout:.0f}s")


# ============================================================================ executor
class RuntimeElasticExecutor:
    _DIST_ENV = ("RANK", "WORLD_SIZE", "LOCAL_RANK", "LOCAL_WORLD_SIZE", "GROUP_RANK", "ROLE_RANK",
                 "ROLE_WORLD_SIZE", "MASTER_ADDR", "MASTER_PORT", "TORCHELASTIC_ERROR_FILE",
                 "TORCHELASTIC_MAX_RESTARTS", "TORCHELASTIC_RESTART_COUNT", "TORCHELASTIC_RUN_ID",
                 "TORCHELASTIC_USE_AGENT_STORE")

    def __init__(self, *, config, planner, train_engine=None, rollout_engine=None, dispatcher=None,
                 elastic_pool=None, launcher: Optional[ProcessLauncher] = None):
        self.config, self.planner = config, planner
        self.train_engine, self.rollout_engine, self.dispatcher = train_engine, rollout_engine, dispatcher
        self.elastic_pool = elastic_pool
        self.launcher = launcher or ProcessLauncher()
        self._procs: Dict[str, subprocess.Popen] = {}
        self._meta: Dict[str, ManagedRolloutProcess] = {}
        self._replaced: List[Tuple[ManagedRolloutProcess, Optional[subprocess.Popen]]] = []
        self._prewarm_stop: List[str] = []
        self._hybrid_procs: Dict[str, subprocess.Popen] = {}
        self._hybrid_meta: Dict[str, ManagedHybridWorkerProcess] = {}
        self._pending: Dict[str, Any] = {}
        self._pending_started: Dict[str, float] = {}
        self._plock = threading.RLock()
        self._signal: Optional[Dict[str, Any]] = None
        self._slots: Dict[str, Dict[str, Any]] = {}
        self._coord_id = ""
        self.gradient_server = None

    # ------------------------------------------------------------------ config helpers
    @property
    def _pc(self):
        return self.config.global_resource_planner

    def _opt(self, name: str, default=None):
        return getattr(self._pc, name, default)

    def _cluster_swap(self, strategy: Optional[str] = None) -> bool:
        return bool(self._opt("runtime_cluster_swap_enabled", False)
                    or (strategy or self._opt("runtime_rollout_reconfigure_strategy", "")) == "cluster_swap")

    def _replica_size(self) -> int:
        width = 1
        for key in ("train_tp_size", "train_pp_size", "train_cp_size"):
            width *= max(1, int(getattr(self.config, key, 1) or 1))
        configured = int(self._opt("elastic_hybrid_replica_size_gpus", 0) or 0)
        if configured > 0 and configured != width:
            raise ValueError(f"elastic_hybrid_replica_size_gpus must equal one complete DP replica "
                             f"topology width ({width}); got {configured}")
        return configured or width

    def _replica_capacity(self) -> int:
        reserve = max(0, int(self._opt("elastic_hybrid_min_rollout_gpus", 0) or 0))
        return max(0, (int(getattr(self.config, "rollout_gpus", 0) or 0) - reserve) // self._replica_size())

    def _current_step(self) -> int:
        m = getattr(self.planner, "latest_runtime_metrics", None)
        return int(getattr(m, "step", 0) or 0)

    def _desired_hybrid_gpus(self, current_train_gpus: int, plan=None) -> int:
        """GRP-commanded elastic GPU count, in whole-replica units."""
        size = self._replica_size()
        sig = self._signal
        if sig is not None:
            exp = int(sig.get("expires_step", 0) or 0)
            if not exp or self._current_step() <= exp:
                want = max(0, int(sig.get("desired_replicas", sig.get("desired_workers", 0)) or 0))
                return min(want, self._replica_capacity()) * size
        if self._opt("elastic_hybrid_require_planner_signal", False):
            return 0
        target = int(self._opt("runtime_training_pool_target_gpus", 0) or 0)
        if target <= 0 and plan is not None:
            target = int(getattr(plan, "train_gpus", 0) or 0)
        return min(max(0, target - int(current_train_gpus)) // size, self._replica_capacity()) * size

    @staticmethod
    def _groups(candidates: List[str], size: int) -> List[Tuple[str, Tuple[str, ...]]]:
        out = []
        for i in range(0, len(candidates) - size + 1, size):
            members = tuple(candidates[i:i + size])
            out.append((f"ehp_replica_{members[0]}", members))
        return out

    @staticmethod
    def _role(role) -> str:
        return str(getattr(role, "value", role))

    # ------------------------------------------------------------------ main entry
    def execute(self, decision) -> RuntimeReconfigurationResult:
        result = RuntimeReconfigurationResult(applied=False, reason=decision.reason)
        self._reconcile_pending(result)
        self.accept_planner_signal(getattr(decision, "elastic_hybrid_signal", None), result=result)
        if not decision.should_reconfigure or decision.candidate_plan is None:
            return result
        plan = decision.candidate_plan
        if not self._opt("runtime_dynamic_reconfiguration_enabled", True):
            return RuntimeReconfigurationResult(applied=False, reason="runtime_dynamic_reconfiguration_disabled")
        manage = bool(self._opt("runtime_manage_rollout_processes", False))
        rollout_runtime = bool(self._opt("apply_to_runtime", True) or manage)
        cur_train = int(self.config.train_gpus)
        strategy = self._opt("runtime_rollout_reconfigure_strategy", "diff")
        swap = self._cluster_swap(strategy)
        drain = bool(self._opt("runtime_drain_before_reconfigure", True))
        if manage:
            self._adopt_existing()
            if self._already_applied(plan, cur_train):
                self._write_manifest(plan, "applied")
                self._write_peer_state(plan, "applied")
                return RuntimeReconfigurationResult(False, "runtime_plan_already_applied",
                                                    actions=["runtime_plan_already_applied"])
        config_applied = prewarmed = coordinated = False
        pre_started: List[ManagedRolloutProcess] = []
        if manage and strategy == "prewarm" and not swap:
            self._apply_config(plan)
            config_applied = True
            result.actions.append("apply_config")
            issue = self._prewarm_capacity_issue(plan)
            if issue:
                strategy = self._opt("runtime_prewarm_no_spare_fallback_strategy", "restart_all")
                result.actions.append(f"prewarm_unavailable:{issue}:fallback_{strategy}")
            else:
                pre_started = self._prewarm(plan)
                prewarmed = True
                result.actions.append("prewarm_rollout_processes")
        if swap and manage and not config_applied:
            self._apply_config(plan)
            config_applied = True
            result.actions.append("apply_config")
            self._write_manifest(plan, "planned")
        if swap and config_applied and self._opt("runtime_coordinate_reconfiguration_ranks", True):
            self._coordinate_peers(plan, result)
            coordinated = True
        paused = False
        if not (swap and not drain) and self.dispatcher is not None and hasattr(self.dispatcher, "pause"):
            self.dispatcher.pause()
            paused = True
            result.actions.append("dispatcher_pause")
            if manage and config_applied and not coordinated:
                self._coordinate_peers(plan, result)
                coordinated = True
            if drain and hasattr(self.dispatcher, "wait_until_idle"):
                self.dispatcher.wait_until_idle(timeout=float(self._opt("runtime_drain_timeout_s", 3600.0)))
                result.actions.append("dispatcher_drain")
        if drain and self.rollout_engine is not None and hasattr(self.rollout_engine, "wait_until_idle"):
            self.rollout_engine.wait_until_idle(timeout=float(self._opt("runtime_drain_timeout_s", 3600.0)))
            result.actions.append("rollout_engine_drain")
        try:
            engine_done = False
            if swap:
                if not config_applied:
                    self._apply_config(plan)
                    config_applied = True
                    result.actions.append("apply_config")
                    self._write_manifest(plan, "planned")
                if not coordinated:
                    self._coordinate_peers(plan, result)
                    coordinated = True
                engine_done = self._cluster_swap_pools(cur_train, plan, result)
            elif self._opt("runtime_reconfigure_training", False):
                if self._opt("runtime_training_pool_plan_only", True):
                    result.training_actions.extend(self._plan_training_pool(cur_train, plan))
                else:
                    self._ensure_pool()
                    result.training_actions.extend(self._reconfigure_training_pool(cur_train, plan, result))
            if not prewarmed and not config_applied:
                if rollout_runtime:
                    self._apply_config(plan)
                    result.actions.append("apply_config")
                else:  # externally managed endpoints stay exactly as launched
                    result.actions.append("preserve_external_rollout_config")
            self._write_manifest(plan, "planned")
            if not coordinated:
                self._coordinate_peers(plan, result)
            if prewarmed:
                stopped = self._finish_prewarm(plan)
                engine_done = True
                result.stopped_processes.extend(stopped)
                result.started_processes.extend(pre_started)
                result.actions.append("reconfigure_rollout_processes:prewarm")
            elif not swap and manage:
                stopped, started = self._reconfigure_processes(plan, strategy)
                engine_done = True
                result.stopped_processes.extend(stopped)
                result.started_processes.extend(started)
                result.actions.append(f"reconfigure_rollout_processes:{strategy}")
            if (not engine_done and not swap and self._opt("apply_to_runtime", True)
                    and self.rollout_engine is not None and hasattr(self.rollout_engine, "reconfigure_from_plan")):
                self._reconfigure_engine(plan, wait_ready=manage)
                result.actions.append("reconfigure_rollout_engine")
            self._write_manifest(plan, "applied")
            self._write_peer_state(plan, "applied")
            result.applied = True
            return result
        except Exception as exc:
            result.errors.append(str(exc))
            self._write_peer_state(plan, "aborted", error=str(exc))
            raise
        finally:
            if paused and hasattr(self.dispatcher, "resume"):
                self.dispatcher.resume()
                result.actions.append("dispatcher_resume")

    # ------------------------------------------------------------------ planner signal
    def accept_planner_signal(self, sig, *, result: Optional[RuntimeReconfigurationResult] = None) -> None:
        """Record a versioned GRP command; releases take effect immediately."""
        if sig is None:
            return
        payload = sig.to_dict() if hasattr(sig, "to_dict") else dict(sig)
        if int(payload.get("step", -1)) < int((self._signal or {}).get("step", -1)):
            return
        self._signal = payload
        want = int(payload.get("desired_replicas", payload.get("desired_workers", 0)) or 0)
        if want <= 0:
            self._release_all(reason=f"grp_{payload.get('reason', 'release')}", result=result)

    def _expire_signal(self) -> None:
        sig = self._signal
        if not sig:
            return
        exp = int(sig.get("expires_step", 0) or 0)
        if exp and self._current_step() > exp:
            self._release_all(reason="planner_signal_expired")
            self._signal = None

    def hybrid_runtime_state(self) -> Dict[str, Any]:
        """EHP state for the planner (copies only)."""
        self._reconcile_pending()
        self._expire_signal()
        active = joining = 0
        domain: Dict[str, Any] = {}
        if self.elastic_pool is not None:
            reps = self.elastic_pool.replica_snapshot()
            membership = self.elastic_pool.gradient_domain.membership_state()
            targets = membership.get("hybrid_targets") or {}
            active_ids = set(membership.get("active_replica_ids") or ())
            mdir = Path(self._opt("hybrid_worker_task_dir", "./logs/elastic_training_tasks")) / "membership"
            for rid, members in reps.items():
                roles = {self._role(w.role) for w in members}
                write_json_atomic(mdir / f"{rid}.json", {
                    "worker_id": rid, "target_core_id": str(targets.get(rid, "")),
                    "role": "hybrid_training" if rid in active_ids else "hybrid_joining",
                    "membership_epoch": int(membership.get("membership_epoch", 0)),
                    "members": [w.worker_id for w in members], "replica_world_size": len(members)})
                if roles == {"hybrid_training"}:
                    active += 1
                elif "hybrid_joining" in roles:
                    joining += 1
            domain = dict(membership)
        with self._plock:
            pending = len(self._pending)
        return {"active_hybrid_replicas": active, "joining_hybrid_replicas": joining,
                "pending_hybrid_replica_joins": pending, "active_hybrid_workers": active,
                "joining_hybrid_workers": joining, "pending_hybrid_joins": pending,
                "replica_size_gpus": self._replica_size(), "communication_domain": domain,
                "planner_signal": dict(self._signal or {})}

    # ------------------------------------------------------------------ training pool
    def _ensure_gradient_server(self) -> None:
        if self.gradient_server is not None or self.train_engine is None:
            return
        if not hasattr(self.train_engine, "enqueue_hybrid_gradient_payload"):
            return
        from libra_b200.infra.elastic.worker import attach_gradient_server, write_endpoint

        import secrets

        self.gradient_server = attach_gradient_server(
            self.train_engine, host=self._opt("gradient_server_host", "") or "127.0.0.1",
            authkey=secrets.token_hex(16))
        self.train_engine.elastic_payload_wait_s = float(self._opt("elastic_hybrid_payload_wait_s", 0.0) or 0.0)
        write_endpoint(self._opt("hybrid_worker_task_dir", "./logs/elastic_training_tasks"),
                       int(os.environ.get("RANK", "0")), self.gradient_server.endpoint,
                       data_parallel_rank=int(getattr(self.train_engine, "dp_rank", 0)))

    def _ensure_pool(self) -> None:
        self._ensure_gradient_server()
        if self.elastic_pool is not None or self.train_engine is None:
            return
        from libra_b200.infra.elastic.hybrid_pool import ElasticHybridPool

        core = list(self.train_engine.get_elastic_core_replica_ids())
        domain = getattr(self.train_engine, "elastic_gradient_domain", None) or \
            self.train_engine.configure_elastic_training(core)
        rollout = [f"rollout{i}" for i in range(int(getattr(self.config, "rollout_gpus", 0) or 0))]
        self.elastic_pool = ElasticHybridPool(core_train_workers=core, core_rollout_workers=rollout,
                                              gradient_domain=domain, snapshot_fetcher=self._fetch_snapshot,
                                              zero_sync_steps=1)

    def _fetch_snapshot(self, worker_id: str, target_core_id: str) -> int:
        if self.train_engine is not None and hasattr(self.train_engine, "capture_elastic_state_snapshot"):
            return int(self.train_engine.capture_elastic_state_snapshot(worker_id, target_core_id))
        return int(getattr(self.train_engine, "current_version", 0) or 0)

    def _targets(self, cur_train: int, plan) -> Tuple[List[str], List[str]]:
        if self.elastic_pool is not None:
            snap = self.elastic_pool.snapshot()
            core = [w for w, x in snap.items() if self._role(x.role) == "core_training"]
            cand = [w for w, x in snap.items() if self._role(x.role) in ("core_rollout", "hybrid_rollout")]
            return core, cand
        dp = max(1, int(getattr(self.config, "train_dp_size", 1) or 1))
        n = max(self._desired_hybrid_gpus(cur_train, plan), int(getattr(self.config, "rollout_gpus", 0) or 0))
        return [f"dp{i}" for i in range(dp)], [f"rollout{i}" for i in range(n)]

    def _plan_training_pool(self, cur_train: int, plan) -> List[str]:
        """Record the training-pool decision without touching live process groups."""
        delta = self._desired_hybrid_gpus(cur_train, plan)
        if delta == 0:
            return [f"plan_training_gpus_unchanged:{cur_train}"]
        size = self._replica_size()
        core, cand = self._targets(cur_train, plan)
        groups = self._groups(cand, size)
        want = delta // size
        acts = ["training_pool_plan_only"]
        for i, (rid, members) in enumerate(groups[:want]):
            acts.append(f"plan_join_replica:{rid}[{','.join(members)}]->{core[i % len(core)]}")
        if want > len(groups):
            acts.append(f"plan_join_replica_shortfall:{want - len(groups)}")
        return acts

    def _reconfigure_training_pool(self, cur_train: int, plan, result) -> List[str]:
        if self.elastic_pool is None:
            return ["training_resize_requested_without_elastic_pool"]
        size = self._replica_size()
        want = self._desired_hybrid_gpus(cur_train, plan) // size
        core, cand = self._targets(cur_train, plan)
        reps = self.elastic_pool.replica_snapshot()
        live = [rid for rid, ms in reps.items()
                if ms and all(self._role(w.role) in ("hybrid_training", "hybrid_joining") for w in ms)]
        delta = want - len(live)
        acts: List[str] = []
        if delta > 0:
            groups = self._groups(cand, size)
            for k, (rid, members) in enumerate(groups[:delta]):
                target = core[(len(live) + k) % len(core)]
                barrier = self._activate_replica if self._opt("hybrid_worker_launch_enabled", False) else None
                h = self.elastic_pool.join_replica(rid, members, target, replica_activation_barrier=barrier,
                                                   timeout_s=float(self._opt("elastic_hybrid_join_timeout_s", 180.0)))
                with self._plock:
                    self._pending[rid] = h
                    self._pending_started[rid] = time.time()
                acts.append(f"join_replica_submitted:{rid}[{','.join(members)}]->{target}:generation={h.generation}")
            if delta > len(groups):
                acts.append(f"join_replica_capacity_shortfall:{delta - len(groups)}")
        elif delta < 0:
            for rid in live[:-delta]:
                with self._plock:
                    pend = self._pending.pop(rid, None)
                    self._pending_started.pop(rid, None)
                if pend is not None:
                    pend.cancel()
                members = tuple(w.worker_id for w in reps[rid])
                try:
                    self.elastic_pool.release_replica_to_rollout(rid)
                except (KeyError, RuntimeError):
                    pass  # a cancellation already rolled it back
                for w in members:
                    self._stop_hybrid(w, result)
                acts.append(f"release_replica_to_rollout:{rid}[{','.join(members)}]")
        else:
            acts.append(f"training_gpus_unchanged:{cur_train + want * size}:active_hybrid_replicas={len(live)}")
        return acts

    def _activate_replica(self, rid: str, members: Tuple[str, ...], target: str, version: int) -> None:
        """Activation barrier: launch the replica's worker process and wait for it."""
        slots = [self._slots.get(w, {}) for w in members]
        hosts = {str(s.get("host", "")) for s in slots}
        if len(hosts) > 1:
            raise RuntimeError(f"a DP replica must launch on one host; replica={rid}, hosts={sorted(hosts)}")
        gpus = [int(g) for s in slots for g in s.get("gpus", [])]
        snap = self.train_engine.get_elastic_state_snapshot_path(version) if self.train_engine is not None else ""
        cmd = self._hybrid_command(rid, target, snap, gpus, len(members))
        env = {k: v for k, v in os.environ.items() if k not in self._DIST_ENV}
        proc = self.launcher.start(cmd, env)
        self._hybrid_procs[rid] = proc
        for rank, w in enumerate(members):
            self._hybrid_procs[w] = proc
            self._hybrid_meta[w] = ManagedHybridWorkerProcess(w, target, cmd, proc.pid, snap, next(iter(hosts), ""),
                                                              gpus, rid, rank, len(members))
        self._wait_hybrid_ready(rid)

    def _hybrid_command(self, rid: str, target: str, snapshot: str, gpus: List[int], world: int) -> str:
        endpoint = getattr(self.gradient_server, "endpoint", None)
        values = {"python": shlex.quote(self._opt("hybrid_worker_python", "") or sys.executable),
                  "worker_id": shlex.quote(rid), "replica_id": shlex.quote(rid), "replica_rank": 0,
                  "replica_world_size": world, "target_core_id": shlex.quote(target),
                  "snapshot_path": shlex.quote(snapshot), "gpus": ",".join(map(str, gpus)),
                  "cuda_visible_devices": shlex.quote(",".join(map(str, gpus))),
                  "gradient_host": shlex.quote(getattr(endpoint, "host", "127.0.0.1")),
                  "gradient_port": int(getattr(endpoint, "port", 0)),
                  "authkey": shlex.quote(getattr(endpoint, "authkey", "")),
                  "task_dir": shlex.quote(self._opt("hybrid_worker_task_dir", "./logs/elastic_training_tasks")),
                  "worker_config": shlex.quote(self._opt("hybrid_worker_config_path", "")
                                               or os.environ.get("RUNTIME_CONFIG", ""))}
        template = self._opt("hybrid_worker_command_template", "")
        if template:
            return template.format(**values)
        prefix = f"CUDA_VISIBLE_DEVICES={values['cuda_visible_devices']} " if gpus else ""
        launch = (f"{values['python']} -m torch.distributed.run --standalone --nproc-per-node {world} -m"
                  if world > 1 else f"{values['python']} -m")
        return (f"{prefix}{launch} libra_b200.infra.elastic.worker --replica-id {values['replica_id']} "
                f"--target-core-id {values['target_core_id']} --snapshot-path {values['snapshot_path']} "
                f"--gradient-host {values['gradient_host']} --gradient-port {values['gradient_port']} "
                f"--authkey {values['authkey']} --task-dir {values['task_dir']} --config {values['worker_config']}")

    def _wait_hybrid_ready(self, rid: str) -> None:
        ready = Path(self._opt("hybrid_worker_task_dir", "./logs/elastic_training_tasks")) / "ready" / f"{rid}.json"
        deadline = time.monotonic() + float(self._opt("hybrid_worker_ready_timeout_s", 60.0))
        proc = self._hybrid_procs.get(rid)
        while time.monotonic() < deadline:
            if ready.exists():
                return
            if proc is not None and proc.poll() is not None:
                raise RuntimeError(f"hybrid worker {rid} exited with {proc.returncode} before becoming ready")
            time.sleep(0.1)
        raise TimeoutError(f"hybrid worker {rid} not ready")

    def _stop_hybrid(self, worker_id: str, result=None) -> None:
        proc = self._hybrid_procs.pop(worker_id, None)
        self._hybrid_meta.pop(worker_id, None)
        if proc is not None and all(p is not proc for p in self._hybrid_procs.values()):
            self.launcher.stop(proc, timeout=float(self._opt("vllm_stop_timeout_s", 30.0)))
            if result is not None:
                result.training_actions.append(f"stop_hybrid_worker:{worker_id}")

    def _release_all(self, *, reason: str, result=None) -> None:
        with self._plock:
            pend = list(self._pending.items())
            self._pending.clear()
            self._pending_started.clear()
        for rid, h in pend:
            h.cancel()
            for w in getattr(h, "member_worker_ids", (rid,)):
                self._stop_hybrid(w, result)
            if result is not None:
                result.training_actions.append(f"join_replica_cancelled:{rid}:{reason}")
        if self.elastic_pool is None:
            return
        for rid, members in self.elastic_pool.replica_snapshot().items():
            if not any(self._role(w.role) in ("hybrid_training", "hybrid_joining") for w in members):
                continue
            try:
                self.elastic_pool.release_replica_to_rollout(rid)
            except (KeyError, RuntimeError):
                continue
            for w in members:
                self._stop_hybrid(w.worker_id, result)
            if result is not None:
                result.training_actions.append(f"release_replica_to_rollout:{rid}:{reason}")

    def _reconcile_pending(self, result=None) -> None:
        """Collect finished background joins without blocking the train loop."""
        timeout = float(self._opt("elastic_hybrid_join_timeout_s", 180.0))
        with self._plock:
            items = list(self._pending.items())
        for rid, h in items:
            if not h.done():
                if time.time() - self._pending_started.get(rid, time.time()) > timeout:
                    h.cancel()
                    with self._plock:
                        self._pending.pop(rid, None)
                        self._pending_started.pop(rid, None)
                    for w in getattr(h, "member_worker_ids", (rid,)):
                        self._stop_hybrid(w, result)
                    if result is not None:
                        result.training_actions.append(f"join_replica_timeout_cancelled:{rid}")
                continue
            try:
                joined = h.result(timeout=0)
                ws = joined if isinstance(joined, tuple) else (joined,)
                if result is not None:
                    result.training_actions.append(f"join_replica_active:{rid}:members="
                                                   f"{','.join(w.worker_id for w in ws)}:generation={h.generation}")
            except Exception as exc:  # noqa: BLE001 - surfaced in the result
                for w in getattr(h, "member_worker_ids", (rid,)):
                    self._stop_hybrid(w, result)
                if result is not None:
                    result.errors.append(f"hybrid_replica_join_failed:{rid}:{exc}")
            finally:
                with self._plock:
                    self._pending.pop(rid, None)
                    self._pending_started.pop(rid, None)

    # ------------------------------------------------------------------ cluster swap
    def _cluster_swap_pools(self, cur_train: int, plan, result) -> bool:
        """Swap GPUs between rollout and training without spare GPUs; returns
        whether the rollout engine was reconfigured."""
        retrain = bool(self._opt("runtime_reconfigure_training", False))
        plan_only = bool(self._opt("runtime_training_pool_plan_only", True))
        if retrain and not plan_only:
            self._ensure_pool()
        planned = int(getattr(plan, "train_gpus", cur_train))
        target = planned if planned < cur_train else cur_train + self._desired_hybrid_gpus(cur_train, plan)
        delta = target - cur_train
        result.actions.append(f"cluster_swap_begin:train_delta={delta}:target_train_gpus={target}")
        if retrain and plan_only:
            result.training_actions.extend(self._plan_training_pool(cur_train, plan))
        elif retrain and delta <= 0:
            result.training_actions.extend(self._reconfigure_training_pool(cur_train, plan, result))
        engine_done = False
        if self._opt("runtime_manage_rollout_processes", False):
            stopped, started = self._swap_processes(plan)
            engine_done = True
            result.stopped_processes.extend(stopped)
            result.started_processes.extend(started)
            result.actions.append("reconfigure_rollout_processes:cluster_swap")
            if delta > 0:
                slots = self._assign_slots(stopped, cur_train, plan)
                if slots:
                    result.training_actions.append("cluster_swap_training_slots:" + ",".join(
                        f"{w}@{s['host']}:{s['gpus']}" for w, s in slots.items()))
        elif self._opt("apply_to_runtime", True) and hasattr(self.rollout_engine, "reconfigure_from_plan"):
            self._reconfigure_engine(plan, wait_ready=False)
            engine_done = True
            result.actions.append("reconfigure_rollout_engine:cluster_swap")
        if retrain and not plan_only and delta > 0:
            result.training_actions.extend(self._reconfigure_training_pool(cur_train, plan, result))
        result.actions.append("cluster_swap_complete")
        return engine_done

    def _assign_slots(self, stopped: List[ManagedRolloutProcess], cur_train: int, plan) -> Dict[str, Dict[str, Any]]:
        delta = self._desired_hybrid_gpus(cur_train, plan)
        if delta <= 0 or not stopped:
            self._slots = {}
            return {}
        _, cand = self._targets(cur_train, plan)
        keep = {(m.host, int(g)) for m in self._desired(plan) for g in m.gpus}
        free = [{"host": m.host, "gpus": [int(g)]} for m in stopped for g in m.gpus if (m.host, int(g)) not in keep]
        self._slots = {str(w): s for w, s in zip(cand[:delta], free[:delta])}
        return dict(self._slots)

    def _swap_processes(self, plan) -> Tuple[List[ManagedRolloutProcess], List[ManagedRolloutProcess]]:
        desired = {m.instance_id: m for m in self._desired(plan)}
        done_cur, done_want = set(), set()
        for iid, cur in list(self._meta.items()):
            if iid in desired and self._same(cur, desired[iid]):
                done_cur.add(iid)
                done_want.add(iid)
        for wid, want in desired.items():  # same slot under a new id: adopt, do not restart
            if wid in done_want:
                continue
            match = next((c for c, m in self._meta.items() if c not in done_cur and self._same(m, want)), None)
            if match is not None:
                m = self._meta.pop(match)
                p = self._procs.pop(match, None)
                self._meta[wid] = ManagedRolloutProcess(wid, want.command or m.command, m.pid, list(m.gpus), m.port,
                                                        m.host, m.tp, m.adopted, m.log_path or want.log_path)
                if p is not None:
                    self._procs[wid] = p
                done_cur.add(wid)
                done_want.add(wid)
        stopped = []
        for iid in list(self._meta):
            if iid not in done_want:
                stopped.extend(self._stop(iid))
        self._grace_after_stop(stopped)
        started = []
        for wid, want in desired.items():
            cur = self._meta.get(wid)
            if cur is None or not self._same(cur, want):
                started.append(self._start(want))
                self._wait_started(started[-1])
        self._reconfigure_engine(plan, wait_ready=bool(started))
        return stopped, started

    # ------------------------------------------------------------------ rollout processes
    @staticmethod
    def _same(a: ManagedRolloutProcess, b: ManagedRolloutProcess) -> bool:
        return a.host == b.host and a.port == b.port and a.tp == b.tp and list(a.gpus) == list(b.gpus)

    def _host(self, inst) -> str:
        h = inst.host or self.config.heterogeneous_rollout.vllm_host
        return "127.0.0.1" if h == "0.0.0.0" else h

    def _log_path(self, iid: str) -> str:
        d = self._opt("runtime_rollout_log_dir", "") or os.path.join(self.config.log_dir, "runtime_rollout")
        return str(Path(d) / f"{iid}.log")

    def _desired(self, plan=None) -> List[ManagedRolloutProcess]:
        """Rollout processes the plan produces (applied to a copy of the config)."""
        h = self.config.heterogeneous_rollout
        if plan is not None:
            probe = copy.deepcopy(self.config)
            self.planner.apply_plan_to_config(plan, probe)
            if any(getattr(i, "port", 0) for i in h.instances):  # keep ports already moved to spares
                ports = {i.instance_id: i.port for i in h.instances if i.instance_id}
                for inst in probe.heterogeneous_rollout.instances:
                    if inst.instance_id in ports and self._same_slot(inst, h.instances, inst.instance_id):
                        inst.port = ports[inst.instance_id]
            h = probe.heterogeneous_rollout
        out = []
        for i, inst in enumerate(h.instances):
            port = int(inst.port) if getattr(inst, "port", 0) else int(h.vllm_base_port) + i
            iid = inst.instance_id or f"grp_tp{inst.tp}_{i}"
            out.append(ManagedRolloutProcess(iid, self._rollout_command(inst, port), 0, list(inst.gpus), port,
                                             self._host(inst), int(inst.tp), False, self._log_path(iid)))
        return out

    @staticmethod
    def _same_slot(inst, current, iid: str) -> bool:
        for c in current:
            if c.instance_id == iid:
                return list(c.gpus) == list(inst.gpus) and int(c.tp) == int(inst.tp)
        return False

    def _rollout_command(self, inst, port: int) -> str:
        h = self.config.heterogeneous_rollout
        host = inst.host or h.vllm_host
        iid = inst.instance_id or f"tp{inst.tp}_{port}"
        values = {"python": shlex.quote(sys.executable), "instance_id": shlex.quote(str(iid)),
                  "model_path": shlex.quote(getattr(self.config, "model_path", "") or ""),
                  "model": shlex.quote(self._preset()),
                  "host": shlex.quote(host), "public_host": shlex.quote("127.0.0.1" if host == "0.0.0.0" else host),
                  "port": port, "tp": inst.tp, "gpus": ",".join(map(str, inst.gpus)),
                  "devices": ",".join(map(str, inst.gpus)),
                  "max_model_len": h.max_model_len or getattr(self.config, "max_seq_length", 0),
                  "gpu_memory_utilization": h.gpu_memory_utilization,
                  "log_path": shlex.quote(self._log_path(str(iid)))}
        template = self._opt("vllm_launch_command_template", "")
        if template:
            return template.format(**values)
        prefix = f"CUDA_VISIBLE_DEVICES={shlex.quote(values['devices'])} " if values["devices"] else ""
        launch = (f"{values['python']} -m torch.distributed.run --standalone --nproc-per-node {inst.tp} -m"
                  if int(inst.tp) > 1 else f"{values['python']} -m")
        mp = getattr(self.config, "model_path", "") or ""
        ckpt = f"--checkpoint {values['model_path']} " if mp and os.path.isdir(mp) else ""
        return (f"{prefix}{launch} libra_b200.engine.server --model {values['model']} {ckpt}--host {values['host']} "
                f"--port {port} --tp {inst.tp} --kv-memory-fraction {values['gpu_memory_utilization']}")

    def _preset(self) -> str:
        from libra_b200.models.qwen3 import PRESETS

        name = os.path.basename(str(getattr(self.config, "model_path", "") or "")).lower()
        return name if name in PRESETS else "qwen3-4b"

    def _env(self, meta: ManagedRolloutProcess) -> Dict[str, str]:
        env = {k: v for k, v in os.environ.items() if k not in self._DIST_ENV}
        env["PLANNED_CUDA_VISIBLE_DEVICES"] = ",".join(map(str, meta.gpus))
        env["LIBRA_ROLE"] = "runtime_rollout"
        return env

    def _start(self, meta: ManagedRolloutProcess) -> ManagedRolloutProcess:
        old = self._meta.get(meta.instance_id)
        if old is not None and not self._same(old, meta):
            self._replaced.append((old, self._procs.get(meta.instance_id)))
        proc = self.launcher.start(meta.command, self._env(meta), meta.log_path)
        started = ManagedRolloutProcess(meta.instance_id, meta.command, proc.pid, list(meta.gpus), meta.port,
                                        meta.host, meta.tp, False, meta.log_path)
        self._procs[meta.instance_id] = proc
        self._meta[meta.instance_id] = started
        return started

    def _stop_meta(self, meta: ManagedRolloutProcess, proc) -> List[ManagedRolloutProcess]:
        timeout = float(self._opt("vllm_stop_timeout_s", 30.0))
        if meta.adopted or proc is None:
            self.launcher.stop_pid(meta.pid, timeout)
            tmpl = self._opt("vllm_stop_command_template", "")
            if tmpl:
                self.launcher.run(tmpl.format(instance_id=shlex.quote(meta.instance_id), host=shlex.quote(meta.host),
                                              port=meta.port, pid=meta.pid, gpus=",".join(map(str, meta.gpus))),
                                  timeout=timeout)
        else:
            self.launcher.stop(proc, timeout)
        return [meta]

    def _stop(self, iid: str) -> List[ManagedRolloutProcess]:
        meta = self._meta.pop(iid, None)
        proc = self._procs.pop(iid, None)
        return [] if meta is None else self._stop_meta(meta, proc)

    def _stop_replaced(self) -> List[ManagedRolloutProcess]:
        out = []
        for meta, proc in self._replaced:
            out.extend(self._stop_meta(meta, proc))
        self._replaced = []
        return out

    def _wait_started(self, meta: ManagedRolloutProcess) -> None:
        if self._opt("runtime_wait_rollout_process_start_ready", False):
            self.launcher.wait_ready(meta.host, meta.port, float(self._opt("vllm_ready_timeout_s", 300.0)))

    def _grace_after_stop(self, stopped) -> None:
        grace = float(self._opt("runtime_post_rollout_stop_grace_s", 0.0) or 0.0)
        if stopped and grace > 0:
            time.sleep(grace)

    def _set_port(self, iid: str, port: int) -> None:
        for inst in self.config.heterogeneous_rollout.instances:
            if (inst.instance_id or "") == iid:
                inst.port = int(port)

    def _adopt_existing(self) -> None:
        """Track already-running endpoints as external processes (never signalled
        unless a registry gives their exact pid)."""
        cfgs = getattr(self.rollout_engine, "instance_configs", None)
        if not cfgs or self._meta or not self._opt("runtime_adopt_existing_rollout_processes", True):
            return
        reg = self._registry()
        h = self.config.heterogeneous_rollout
        for i, c in enumerate(cfgs):
            iid = str(c.get("instance_id") or f"adopted_{i}")
            r = reg.get(iid, {})
            host = str(r.get("host") or c.get("host") or h.vllm_host)
            self._meta[iid] = ManagedRolloutProcess(
                iid, "", int(r.get("pid", -1)), list(r.get("gpus") or c.get("gpu_ids") or []),
                int(r.get("port", c.get("port", int(h.vllm_base_port) + i))),
                "127.0.0.1" if host == "0.0.0.0" else host, int(r.get("tp", c.get("tp_degree", 1))), True,
                str(r.get("log_path") or ""))

    def _registry(self) -> Dict[str, Dict[str, Any]]:
        path = self._opt("runtime_rollout_pid_registry_path", "") or os.environ.get("GRP_ROLLOUT_PID_REGISTRY_PATH", "")
        if not path or not Path(path).exists():
            return {}
        out = {}
        for line in Path(path).read_text(encoding="utf-8").splitlines():
            try:
                rec = json.loads(line)
            except json.JSONDecodeError:
                continue
            if rec.get("instance_id"):
                out[str(rec["instance_id"])] = rec
        return out

    def _already_applied(self, plan, cur_train: int) -> bool:
        if self._opt("runtime_reconfigure_training", False):
            if int(getattr(plan, "train_gpus", cur_train)) != cur_train:
                return False
            if self._desired_hybrid_gpus(cur_train, plan):
                return False
        want = {m.instance_id: m for m in self._desired(plan)}
        return set(want) == set(self._meta) and all(self._same(self._meta[i], m) for i, m in want.items())

    def _reconfigure_processes(self, plan, strategy: str):
        if strategy == "restart_all":
            stopped = []
            for iid in list(self._meta):
                stopped.extend(self._stop(iid))
            self._grace_after_stop(stopped)
            started = [self._start(m) for m in self._desired(plan)]
            for m in started:
                self._wait_started(m)
            self._reconfigure_engine(plan, wait_ready=True)
            return stopped, started
        if strategy == "cluster_swap":
            return self._swap_processes(plan)
        return self._blue_green(plan)  # "diff" keeps blue-green ordering: in-flight requests finish

    def _blue_green(self, plan):
        desired = {m.instance_id: m for m in self._desired(plan)}
        used = {m.port for m in self._meta.values()}
        spare = max(used | {int(self.config.heterogeneous_rollout.vllm_base_port)}) + 1
        owners = {m.port: iid for iid, m in self._meta.items()}
        to_stop, started = [], []
        for iid, cur in list(self._meta.items()):
            want = desired.get(iid)
            if want is None:
                to_stop.append(iid)
            elif not self._same(cur, want):
                to_stop.append(iid)
        for iid, want in desired.items():
            cur = self._meta.get(iid)
            if cur is not None and self._same(cur, want):
                continue
            if want.port in used and (owners.get(want.port) not in (None, iid) or cur is not None):
                want.port = spare
                spare += 1
                self._set_port(iid, want.port)
                want.command = self._rollout_command(self._inst(iid), want.port)
                used.add(want.port)
            started.append(self._start(want))
            self._wait_started(started[-1])
        self._reconfigure_engine(plan, wait_ready=True)
        stopped = []
        for iid in to_stop:
            if any(s.instance_id == iid for s in started):
                continue  # its old process sits in the replaced list
            stopped.extend(self._stop(iid))
        stopped.extend(self._stop_replaced())
        return stopped, started

    def _inst(self, iid: str):
        for inst in self.config.heterogeneous_rollout.instances:
            if (inst.instance_id or "") == iid:
                return inst
        raise KeyError(iid)

    def _prewarm_capacity_issue(self, plan) -> str:
        desired = self._desired(plan)
        starting = [w for w in desired if w.instance_id not in self._meta or not self._same(self._meta[w.instance_id], w)]
        if not starting:
            return ""
        cap: Dict[str, int] = {}
        for m in list(self._meta.values()) + desired:
            if m.gpus:
                cap[m.host] = max(cap.get(m.host, 0), max(int(g) for g in m.gpus) + 1, len(m.gpus))
        h = self.config.heterogeneous_rollout
        if h.available_gpus:  # the rollout pool is exactly these GPUs (training owns the rest of the box)
            host = "127.0.0.1" if h.vllm_host == "0.0.0.0" else h.vllm_host
            cap[host] = len(set(int(g) for g in h.available_gpus))
        demand: Dict[str, int] = {}
        for m in list(self._meta.values()) + starting:
            demand[m.host] = demand.get(m.host, 0) + max(int(m.tp), len(m.gpus))
        for host, d in demand.items():
            if cap.get(host, 0) and d > cap[host]:
                return f"no_spare_gpu_capacity:{host}:{d}>{cap[host]}"
        return ""

    def _prewarm(self, plan) -> List[ManagedRolloutProcess]:
        desired = self._desired(plan)
        ports = {m.port for m in self._meta.values()} | {m.port for m in desired}
        spare = max(ports | {int(self.config.heterogeneous_rollout.vllm_base_port)}) + 1
        self._prewarm_stop = [iid for iid, m in self._meta.items()
                              if not any(w.instance_id == iid and self._same(m, w) for w in desired)]
        started = []
        for want in desired:
            cur = self._meta.get(want.instance_id)
            if cur is not None and self._same(cur, want):
                continue
            want.port = spare
            spare += 1
            self._set_port(want.instance_id, want.port)
            want.command = self._rollout_command(self._inst(want.instance_id), want.port)
            started.append(self._start(want))
            self._wait_started(started[-1])
        return started

    def _finish_prewarm(self, plan) -> List[ManagedRolloutProcess]:
        """Cut traffic over to the prewarmed set, then stop what it replaced."""
        self._reconfigure_engine(plan, wait_ready=True)
        replaced = {m.instance_id for m, _ in self._replaced}
        stopped = []
        for iid in self._prewarm_stop:
            if iid not in replaced:  # a restarted id's old process is in the replaced list
                stopped.extend(self._stop(iid))
        stopped.extend(self._stop_replaced())
        self._prewarm_stop = []
        return stopped

    def _reconfigure_engine(self, plan, wait_ready: bool) -> None:
        if self.rollout_engine is None or not hasattr(self.rollout_engine, "reconfigure_from_plan"):
            return
        self.rollout_engine.reconfigure_from_plan(plan, self.config)
        if wait_ready and hasattr(self.rollout_engine, "wait_for_ready"):
            self.rollout_engine.wait_for_ready(timeout=float(self._opt("vllm_ready_timeout_s", 300.0)))

    def _apply_config(self, plan) -> None:
        """Apply the plan; a fixed training topology survives when the
        training pool is managed elastically."""
        keep = bool(self._opt("runtime_training_pool_only", True) and self._opt("runtime_reconfigure_training", False))
        saved = {k: getattr(self.config, k) for k in ("n_total_gpus", "train_gpus", "train_tp_size", "tp_size",
                                                      "train_pp_size", "train_dp_size", "micro_batch_size")} if keep else {}
        self.planner.apply_plan_to_config(plan, self.config)
        for k, v in saved.items():
            setattr(self.config, k, v)

    # ------------------------------------------------------------------ manifests / peers
    def _write_manifest(self, plan, phase: str) -> None:
        path = self._opt("runtime_rollout_manifest_path", "") or os.path.join(self.config.log_dir,
                                                                               "runtime_rollout_manifest.json")
        write_json_atomic(Path(path), {"phase": phase, "updated_at": time.time(),
                                       "plan": plan.to_dict() if hasattr(plan, "to_dict") else {},
                                       "processes": [vars(m) for m in self._meta.values()]})

    def _coord_dir(self) -> Path:
        d = self._opt("runtime_reconfiguration_coord_dir", "")
        return Path(d) if d else Path(self.config.log_dir) / "runtime_reconfiguration"

    def _peer_training_state(self, plan) -> Dict[str, Any]:
        if not self._opt("runtime_reconfigure_training", False):
            return {"enabled": False}
        cur = int(getattr(self.config, "train_gpus", 0) or 0)
        extra = self._desired_hybrid_gpus(cur, plan)
        core, cand = self._targets(cur, plan)
        targets = {rid: core[i % len(core)] for i, (rid, _) in
                   enumerate(self._groups(cand, self._replica_size())[:extra // self._replica_size()])}
        active: List[str] = []
        if self.elastic_pool is not None:
            m = self.elastic_pool.gradient_domain.membership_state()
            if m.get("hybrid_targets"):
                targets = {str(k): str(v) for k, v in m["hybrid_targets"].items()}
            active = [str(r) for r in m.get("active_replica_ids", ()) if str(r) in targets]
        return {"enabled": True, "plan_only": bool(self._opt("runtime_training_pool_plan_only", True)),
                "target_train_gpus": cur + extra, "current_train_gpus": cur, "core_replica_ids": core,
                "hybrid_targets": targets, "active_hybrid_ids": active, "replica_size_gpus": self._replica_size(),
                "elastic_hybrid_signal": dict(self._signal or {}), "activate_hybrids": bool(active)}

    def _write_peer_state(self, plan, phase: str, error: str = "") -> Path:
        h = self.config.heterogeneous_rollout
        payload = {"coord_id": self._coord_id, "phase": phase, "job_id": os.environ.get("JOB_ID", ""),
                   "updated_at": time.time(), "plan": plan.to_dict() if hasattr(plan, "to_dict") else {},
                   "instances": [{"instance_id": inst.instance_id, "tp": int(inst.tp), "gpus": list(inst.gpus),
                                  "host": inst.host or h.vllm_host, "port": int(inst.port or (h.vllm_base_port + i))}
                                 for i, inst in enumerate(h.instances)],
                   "training": self._peer_training_state(plan), "error": error}
        path = self._coord_dir() / f"{phase}.json"
        write_json_atomic(path, payload)
        return path

    def _expected_ready_ranks(self) -> List[int]:
        world = int(os.environ.get("WORLD_SIZE", "1") or 1)
        if world <= 1:
            return []
        if not self._opt("runtime_coordinate_batch_source_only", True):
            return list(range(1, world))
        mp = max(1, int(getattr(self.config, "train_tp_size", 1) or 1)) * \
            max(1, int(getattr(self.config, "train_pp_size", 1) or 1))
        return [r for r in range(1, world) if r % mp == 0]

    def _coordinate_peers(self, plan, result) -> None:
        """Rank 0 asks the batch-source ranks to drain and waits for each
        ``ready/rank_R.json`` carrying this request's coordination id."""
        if int(os.environ.get("WORLD_SIZE", "1") or 1) <= 1 or int(os.environ.get("RANK", "0") or 0) != 0:
            return
        if not self._opt("runtime_coordinate_reconfiguration_ranks", True):
            return
        if not self._opt("runtime_drain_before_reconfigure", True):
            result.actions.append("peer_reconfig_drain_skipped")
            return
        self._coord_id = f"rollout_{time.time_ns()}_{'_'.join(map(str, getattr(plan, 'rollout_tp_list', [])))}"
        cdir = self._coord_dir()
        ready = cdir / "ready"
        ready.mkdir(parents=True, exist_ok=True)
        for old in ready.glob("rank_*.json"):
            old.unlink(missing_ok=True)
        for name in ("request.json", "applied.json", "aborted.json"):
            (cdir / name).unlink(missing_ok=True)
        self._write_peer_state(plan, "request")
        result.actions.append("peer_reconfig_request")
        ranks = self._expected_ready_ranks()
        deadline = time.monotonic() + float(self._opt("runtime_drain_timeout_s", 3600.0))

        def ok(r: int) -> bool:
            p = ready / f"rank_{r}.json"
            try:
                return json.loads(p.read_text(encoding="utf-8")).get("coord_id") == self._coord_id
            except (OSError, ValueError):
                return False

        while time.monotonic() < deadline:
            if all(ok(r) for r in ranks):
                result.actions.append("peer_reconfig_drain:" + ",".join(map(str, ranks)))
                return
            time.sleep(0.1)
        raise TimeoutError("peer ranks did not drain before runtime reconfiguration: "
                           + ", ".join(str(r) for r in ranks if not ok(r)))

    # ------------------------------------------------------------------ shutdown
    def close(self) -> None:
        for iid in list(self._meta):
            if not self._meta[iid].adopted:
                self._stop(iid)
        for w in list(self._hybrid_procs):
            self._stop_hybrid(w)
        if self.gradient_server is not None and hasattr(self.gradient_server, "close"):
            self.gradient_server.close()
        self.gradient_server = None
        if self.elastic_pool is not None:
            self.elastic_pool.close()
        self.elastic_pool = None


def follow_reconfiguration_request(coord_dir: str, rank: int, drain=None, timeout_s: float = 0.0) -> Optional[str]:
    """Peer-rank side: if rank 0 posted ``request.json``, drain (callable) and
    answer ``ready/rank_R.json`` with the request's coordination id."""
    req = Path(coord_dir) / "request.json"
    if not req.exists():
        return None
    try:
        coord_id = json.loads(req.read_text(encoding="utf-8")).get("coord_id", "")
    except (OSError, ValueError):
        return None
    if drain is not None:
        drain(timeout_s) if timeout_s else drain()
    write_json_atomic(Path(coord_dir) / "ready" / f"rank_{rank}.json",
                      {"coord_id": coord_id, "rank": rank, "job_id": os.environ.get("JOB_ID", ""),
                       "ready_at": time.time()})
    return coord_id
