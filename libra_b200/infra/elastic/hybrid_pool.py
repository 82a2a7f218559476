"""Elastic Hybrid Pool (EHP) and the inter-replica gradient domain.

Contract (reference ``infra/elastic/hybrid_pool.py``):

* the core training topology never changes; borrowed rollout GPUs join only
  the *inter-replica gradient domain* as whole data-parallel replicas;
* a join is non-blocking: ``join_replica`` returns a handle immediately and a
  background thread walks REQUESTED -> FETCHING_STATE -> ZERO_SYNC ->
  ACTIVATING -> ACTIVE; while joining, the replica only counts as a zero
  placeholder, so core steps never wait for it;
* every join carries a generation number; cancelling (or a planner reversal)
  bumps it, and the background thread rolls every member back as soon as it
  notices (CANCELLED), a member failure rolls the whole replica back (FAILED);
* hybrid gradients are added to their *target core replica's* gradient before
  the core DP reduction, and only when the payload's membership epoch, step
  and state version match; the elastic collective must never use the core DP
  process group (decoupled communication domains).

Implementation notes: a single-worker join is a one-member replica join; the
gradient transports are a chunked torch.distributed all-reduce on a separate
group (``TorchDistributedTransport``) and the single-box peer-memory lane
(``PeerMemoryTransport``) where the hybrid replica's gradient is read from its
exported device buffer and added on the target's GPU.
"""

from __future__ import annotations

import enum
import threading
import time
from concurrent.futures import Future, ThreadPoolExecutor
from dataclasses import dataclass, field
from typing import Callable, Dict, Iterable, List, Mapping, Optional, Protocol, Tuple

import torch

try:
    import torch.distributed as dist
except ModuleNotFoundError:  # pragma: no cover
    dist = None

DEFAULT_CHUNK_BYTES = 16 * 1024 * 1024


class ReplicaRole(str, enum.Enum):
    CORE_TRAINING = "core_training"
    CORE_ROLLOUT = "core_rollout"
    HYBRID_ROLLOUT = "hybrid_rollout"
    HYBRID_JOINING = "hybrid_joining"
    HYBRID_TRAINING = "hybrid_training"


class JoinState(str, enum.Enum):
    REQUESTED = "requested"
    FETCHING_STATE = "fetching_state"
    ZERO_SYNC = "zero_sync"
    ACTIVATING = "activating"
    ACTIVE = "active"
    CANCELLED = "cancelled"
    FAILED = "failed"


class JoinCancelledError(RuntimeError):
    """Raised inside a stale background join after the target changed."""


@dataclass(frozen=True)
class GradientPayload:
    replica_id: str
    target_core_id: str
    tensors: Tuple[torch.Tensor, ...]
    zero_placeholder: bool = False
    replica_rank: int = 0
    replica_world_size: int = 1
    step: int = -1
    state_version: int = -1
    membership_epoch: int = 0

    @staticmethod
    def zeros_like(*, replica_id: str, target_core_id: str, reference: Iterable[torch.Tensor]) -> "GradientPayload":
        return GradientPayload(replica_id, target_core_id, tuple(torch.zeros_like(t) for t in reference), True)


@dataclass
class ElasticWorker:
    worker_id: str
    role: ReplicaRole
    target_core_id: Optional[str] = None
    join_state: Optional[JoinState] = None
    state_version: int = 0
    membership_epoch: int = 0
    transition_generation: int = 0
    last_transition_ts: float = field(default_factory=time.time)

    def transition(self, role: ReplicaRole, *, target_core_id: Optional[str] = None,
                   join_state: Optional[JoinState] = None, state_version: Optional[int] = None,
                   membership_epoch: Optional[int] = None, transition_generation: Optional[int] = None) -> None:
        self.role, self.target_core_id, self.join_state = role, target_core_id, join_state
        if state_version is not None:
            self.state_version = state_version
        if membership_epoch is not None:
            self.membership_epoch = int(membership_epoch)
        if transition_generation is not None:
            self.transition_generation = transition_generation
        self.last_transition_ts = time.time()


@dataclass
class ReplicaJoinHandle:
    replica_id: str
    member_worker_ids: Tuple[str, ...]
    target_core_id: str
    future: Future
    generation: int = 0
    cancel_callback: Optional[Callable[[str, int], None]] = None

    def done(self) -> bool:
        return self.future.done()

    def result(self, timeout: Optional[float] = None):
        return self.future.result(timeout=timeout)

    def cancel(self) -> None:
        if self.cancel_callback is not None:
            self.cancel_callback(self.replica_id, self.generation)


@dataclass
class JoinHandle(ReplicaJoinHandle):
    """Single-worker join handle (``result()`` returns the worker)."""

    @property
    def worker_id(self) -> str:
        return self.replica_id

    def result(self, timeout: Optional[float] = None):
        return self.future.result(timeout=timeout)[0]


# =============================================================================== transports
class GradientTransport(Protocol):
    def exchange(self, local: torch.Tensor, *, group, average: bool) -> torch.Tensor: ...


class TorchDistributedTransport:
    """Chunked all-reduce on the elastic process group (NCCL on GPUs, gloo on CPU)."""

    def __init__(self, chunk_bytes: int = DEFAULT_CHUNK_BYTES):
        if chunk_bytes <= 0:
            raise ValueError("chunk_bytes must be positive")
        self.chunk_bytes = chunk_bytes

    def exchange(self, local: torch.Tensor, *, group=None, average: bool) -> torch.Tensor:
        out = local.clone()
        if dist is None or not dist.is_available() or not dist.is_initialized():
            return out
        flat = out.view(-1)
        step = max(self.chunk_bytes // max(out.element_size(), 1), 1)
        for s in range(0, flat.numel(), step):
            dist.all_reduce(flat[s:s + step], op=dist.ReduceOp.SUM, group=group)
        if average:
            n = dist.get_world_size(group=group)
            if n > 1:
                out.div_(n)
        return out


# the reference's class name for the same role
TorchDistributedRDMATransport = TorchDistributedTransport


class PeerMemoryTransport:
    """Single-box lane: peers publish device tensors (same process, or mapped via
    CUDA IPC); ``exchange`` sums every published peer tensor for this round
    onto the local device (peer reads over NVLink) and optionally averages."""

    def __init__(self):
        self._round: Dict[str, torch.Tensor] = {}
        self._lock = threading.Lock()

    def publish(self, replica_id: str, tensor: torch.Tensor) -> None:
        with self._lock:
            self._round[replica_id] = tensor

    def exchange(self, local: torch.Tensor, *, group=None, average: bool) -> torch.Tensor:
        with self._lock:
            peers = list(self._round.values())
        out = local.clone()
        for t in peers:
            if t is not local:
                out.add_(t.to(out.device, non_blocking=True))
        if average:
            out.div_(1 + sum(1 for t in peers if t is not local))
        return out

    def clear(self) -> None:
        with self._lock:
            self._round.clear()


@dataclass
class GradientCommunicationDomains:
    core_process_group: object = None
    hybrid_process_group: object = None
    decoupled: bool = True

    @property
    def gradient_process_group(self):
        if self.decoupled:
            return self.hybrid_process_group
        return self.hybrid_process_group or self.core_process_group


# =============================================================================== gradient domain
class InterReplicaGradientDomain:
    def __init__(self, *, core_replica_ids: Iterable[str], transport: Optional[GradientTransport] = None,
                 process_group=None, communication_domains: Optional[GradientCommunicationDomains] = None,
                 decouple_communication_domains: bool = True, average_core_replicas: bool = True,
                 require_isolated_process_group: bool = False, local_replica_rank: int = 0,
                 replica_world_size: int = 1):
        ids = list(core_replica_ids)
        if not ids:
            raise ValueError("core_replica_ids cannot be empty")
        if len(ids) != len(set(ids)):
            raise ValueError("core_replica_ids must be unique")
        self.core_replica_ids = tuple(ids)
        self.transport = transport or TorchDistributedTransport()
        self.communication_domains = communication_domains or GradientCommunicationDomains(
            core_process_group=process_group,
            hybrid_process_group=None if decouple_communication_domains else process_group,
            decoupled=decouple_communication_domains)
        self.average_core_replicas = average_core_replicas
        self.require_isolated_process_group = bool(require_isolated_process_group)
        self.replica_world_size = max(1, int(replica_world_size))
        self.local_replica_rank = int(local_replica_rank)
        if not 0 <= self.local_replica_rank < self.replica_world_size:
            raise ValueError("local_replica_rank must be inside replica_world_size")
        self._targets: Dict[str, str] = {}
        self._epochs: Dict[str, int] = {}
        self._joining: set = set()
        self._epoch = 0
        self._lock = threading.RLock()

    # -------------------------------------------------------------- communication groups
    @property
    def process_group(self):
        return self.communication_domains.gradient_process_group

    @process_group.setter
    def process_group(self, value) -> None:
        if self.communication_domains.decoupled:
            self.communication_domains.hybrid_process_group = value
        else:
            self.communication_domains.core_process_group = value
            self.communication_domains.hybrid_process_group = value

    @property
    def decoupled_communication_domains(self) -> bool:
        return bool(self.communication_domains.decoupled)

    def communication_state(self) -> Dict[str, bool]:
        c = self.communication_domains
        return {"decoupled": c.decoupled, "has_core_process_group": c.core_process_group is not None,
                "has_hybrid_process_group": c.hybrid_process_group is not None,
                "uses_core_group_for_elastic_reduce": (not c.decoupled and c.gradient_process_group is
                                                       c.core_process_group),
                "isolated_group_verified": (c.hybrid_process_group is not None and
                                            c.hybrid_process_group is not c.core_process_group)}

    def validate_communication_isolation(self) -> None:
        c = self.communication_domains
        if not c.decoupled:
            return
        if c.hybrid_process_group is not None and c.hybrid_process_group is c.core_process_group:
            raise RuntimeError("elastic gradient process group aliases the core training group")
        if self.require_isolated_process_group and c.hybrid_process_group is None:
            raise RuntimeError("isolated elastic collective group is required but not initialized")

    def bind_hybrid_process_group(self, process_group) -> None:
        c = self.communication_domains
        if c.decoupled and process_group is not None and process_group is c.core_process_group:
            raise ValueError("decoupled elastic gradients cannot reuse the core process group")
        c.hybrid_process_group = process_group

    # -------------------------------------------------------------- membership
    def _check_core(self, core_id: str) -> None:
        if core_id not in self.core_replica_ids:
            raise KeyError(f"unknown core replica: {core_id}")

    def request_join(self, replica_id: str, target_core_id: str, *, membership_epoch: Optional[int] = None) -> None:
        self._check_core(target_core_id)
        with self._lock:
            self._targets[replica_id] = target_core_id
            self._joining.add(replica_id)
            if membership_epoch is None:
                self._epoch += 1
                membership_epoch = self._epoch
            else:
                self._epoch = max(self._epoch, int(membership_epoch))
            self._epochs[replica_id] = int(membership_epoch)

    def mark_active(self, replica_id: str) -> None:
        with self._lock:
            if replica_id not in self._targets:
                raise KeyError(f"unknown hybrid replica: {replica_id}")
            self._joining.discard(replica_id)
            self._epoch += 1
            self._epochs[replica_id] = self._epoch

    def detach(self, replica_id: str) -> None:
        with self._lock:
            self._joining.discard(replica_id)
            if self._targets.pop(replica_id, None) is not None:
                self._epoch += 1
                self._epochs.pop(replica_id, None)

    def is_joining(self, replica_id: str) -> bool:
        with self._lock:
            return replica_id in self._joining

    def active_hybrid_ids(self) -> Tuple[str, ...]:
        with self._lock:
            return tuple(r for r in self._targets if r not in self._joining)

    def attached_hybrid_ids(self) -> Tuple[str, ...]:
        with self._lock:
            return tuple(self._targets)

    def active_hybrid_ids_for_core(self, core_replica_id: str) -> Tuple[str, ...]:
        self._check_core(core_replica_id)
        with self._lock:
            return tuple(r for r, t in self._targets.items() if t == core_replica_id and r not in self._joining)

    def membership_epoch(self, replica_id: str) -> int:
        with self._lock:
            return int(self._epochs.get(replica_id, 0))

    def membership_state(self) -> Dict[str, object]:
        with self._lock:
            return {"membership_epoch": self._epoch, "core_replica_ids": self.core_replica_ids,
                    "hybrid_targets": dict(self._targets), "joining_replica_ids": tuple(sorted(self._joining)),
                    "active_replica_ids": tuple(sorted(r for r in self._targets if r not in self._joining)),
                    "decoupled": self.decoupled_communication_domains}

    def zero_payload_for(self, *, hybrid_replica_id: str, reference: Iterable[torch.Tensor]) -> GradientPayload:
        with self._lock:
            target = self._targets[hybrid_replica_id]
        return GradientPayload.zeros_like(replica_id=hybrid_replica_id, target_core_id=target, reference=reference)

    # -------------------------------------------------------------- aggregation
    def _usable(self, p: GradientPayload, core_id: str, targets, joining, epochs, step: int, version: int,
                check_epoch: bool) -> bool:
        if targets.get(p.replica_id) != core_id or p.replica_id in joining or p.zero_placeholder:
            return False
        if check_epoch and p.membership_epoch != epochs.get(p.replica_id, 0):
            return False
        if p.step >= 0 and step >= 0 and p.step != step:
            return False
        if p.state_version >= 0 and version >= 0 and p.state_version != version:
            return False
        if p.replica_world_size != self.replica_world_size:
            raise ValueError(f"payload replica world size mismatch for {p.replica_id}: "
                             f"{p.replica_world_size} != {self.replica_world_size}")
        return p.replica_rank == self.local_replica_rank

    def _snapshot(self):
        with self._lock:
            return dict(self._targets), set(self._joining), dict(self._epochs)

    def usable_payloads(self, core_replica_id: str, hybrid_payloads: Iterable[GradientPayload], *, step: int = -1,
                        state_version: int = -1) -> List[GradientPayload]:
        """The payloads that count for ``core_replica_id`` now: target matches,
        replica active (not joining), not a zero placeholder, membership epoch
        current, step/state version matching when both sides give one, and
        the payload's replica rank equal to this lane's rank."""
        self._check_core(core_replica_id)
        targets, joining, epochs = self._snapshot()
        return [p for p in hybrid_payloads
                if self._usable(p, core_replica_id, targets, joining, epochs, step, state_version, True)]

    def accumulate_local_gradients(self, *, core_replica_id: str, core_gradients: Iterable[torch.Tensor],
                                   hybrid_payloads: Iterable[GradientPayload] = (), step: int = -1,
                                   state_version: int = -1) -> Tuple[torch.Tensor, ...]:
        """core gradients + every matching hybrid payload for this core replica."""
        out = [t.clone() for t in core_gradients]
        for p in self.usable_payloads(core_replica_id, hybrid_payloads, step=step, state_version=state_version):
            if len(p.tensors) != len(out):
                raise ValueError("hybrid payload tensor count mismatch")
            for i, extra in enumerate(p.tensors):
                out[i].add_(extra.to(device=out[i].device, dtype=out[i].dtype))
        return tuple(out)

    def reduce_core_gradients(self, *, core_gradients: Mapping[str, Iterable[torch.Tensor]],
                              hybrid_payloads: Iterable[GradientPayload] = ()) -> Dict[str, Tuple[torch.Tensor, ...]]:
        distributed = dist is not None and dist.is_available() and dist.is_initialized()
        if distributed and self.decoupled_communication_domains:
            self.validate_communication_isolation()
        local_ids = tuple(r for r in self.core_replica_ids if r in core_gradients)
        missing = set(self.core_replica_ids) - set(core_gradients)
        if missing and not distributed:
            raise ValueError(f"missing core gradients for: {sorted(missing)}")
        if not local_ids:
            raise ValueError("no local core gradients were provided")
        eff = {r: [t.clone() for t in core_gradients[r]] for r in local_ids}
        shapes = {tuple(t.shape for t in v) for v in eff.values()}
        if len(shapes) > 1:
            raise ValueError("core gradient tensor shapes do not match")
        targets, joining, epochs = self._snapshot()
        for p in hybrid_payloads:
            tgt = targets.get(p.replica_id)
            if tgt is None or tgt not in eff:
                continue
            if tgt != p.target_core_id:
                raise ValueError(f"payload target mismatch for {p.replica_id}: {p.target_core_id} != {tgt}")
            if not self._usable(p, tgt, targets, joining, epochs, -1, -1, False):
                continue
            if len(p.tensors) != len(eff[tgt]):
                raise ValueError("hybrid payload tensor count mismatch")
            for i, extra in enumerate(p.tensors):
                eff[tgt][i].add_(extra.to(device=eff[tgt][i].device, dtype=eff[tgt][i].dtype))
        if distributed and self.process_group is not None:
            return {r: tuple(self.transport.exchange(t, group=self.process_group, average=self.average_core_replicas)
                             for t in ts) for r, ts in eff.items()}
        reduced = []
        for col in zip(*(eff[r] for r in local_ids)):
            s = torch.stack([t.to(col[0].device) for t in col]).sum(0)
            reduced.append(s / len(local_ids) if self.average_core_replicas else s)
        return {r: tuple(t.clone() for t in reduced) for r in local_ids}


# =============================================================================== pool
class ElasticHybridPool:
    """Role/state machine for lending rollout workers to training."""

    def __init__(self, *, core_train_workers: Iterable[str], core_rollout_workers: Iterable[str] = (),
                 hybrid_workers: Iterable[str] = (), gradient_domain: Optional[InterReplicaGradientDomain] = None,
                 snapshot_fetcher: Optional[Callable[[str, str], int]] = None, zero_sync_steps: int = 1,
                 max_background_workers: int = 0):
        if zero_sync_steps < 0:
            raise ValueError("zero_sync_steps cannot be negative")
        core_train, core_roll, hybrid = tuple(core_train_workers), tuple(core_rollout_workers), tuple(hybrid_workers)
        self.zero_sync_steps = zero_sync_steps
        self.snapshot_fetcher = snapshot_fetcher or (lambda worker_id, target: 0)
        self.gradient_domain = gradient_domain or InterReplicaGradientDomain(core_replica_ids=core_train)
        self._workers: Dict[str, ElasticWorker] = {}
        for ids, role in ((core_train, ReplicaRole.CORE_TRAINING), (core_roll, ReplicaRole.CORE_ROLLOUT),
                          (hybrid, ReplicaRole.HYBRID_ROLLOUT)):
            for w in ids:
                self._workers[w] = ElasticWorker(w, role)
        if not self._workers:
            raise ValueError("ElasticHybridPool requires at least one worker")
        cap = int(max_background_workers) if int(max_background_workers) > 0 else max(1, len(core_roll) + len(hybrid))
        self._executor = ThreadPoolExecutor(max_workers=cap, thread_name_prefix="ehp-join")
        self._lock = threading.RLock()
        self._closed = False
        self._generations: Dict[str, int] = {}
        self._members: Dict[str, Tuple[str, ...]] = {}

    # -------------------------------------------------------------- views
    def snapshot(self) -> Dict[str, ElasticWorker]:
        with self._lock:
            return {w: ElasticWorker(x.worker_id, x.role, x.target_core_id, x.join_state, x.state_version,
                                     x.membership_epoch, x.transition_generation, x.last_transition_ts)
                    for w, x in self._workers.items()}

    def replica_snapshot(self) -> Dict[str, Tuple[ElasticWorker, ...]]:
        ws = self.snapshot()
        with self._lock:
            members = dict(self._members)
        return {r: tuple(ws[w] for w in m) for r, m in members.items()}

    def _pick(self, worker_id: Optional[str], allowed) -> ElasticWorker:
        if worker_id is not None:
            if worker_id not in self._workers:
                raise KeyError(f"unknown worker: {worker_id}")
            w = self._workers[worker_id]
            if w.role not in allowed:
                raise RuntimeError(f"worker {worker_id} is {w.role}, expected one of {allowed}")
            return w
        for w in self._workers.values():
            if w.role in allowed:
                return w
        raise RuntimeError(f"no worker available in roles: {allowed}")

    # -------------------------------------------------------------- transitions
    _LENDABLE = {ReplicaRole.CORE_ROLLOUT, ReplicaRole.HYBRID_ROLLOUT}

    def borrow_rollout_worker(self, worker_id: Optional[str] = None) -> ElasticWorker:
        with self._lock:
            w = self._pick(worker_id, self._LENDABLE)
            w.transition(ReplicaRole.HYBRID_ROLLOUT)
            return w

    def join_replica(self, replica_id: str, member_worker_ids: Iterable[str], target_core_id: str, *,
                     activation_barrier: Optional[Callable[[str, str, int], None]] = None,
                     replica_activation_barrier: Optional[Callable[[str, Tuple[str, ...], str, int], None]] = None,
                     timeout_s: Optional[float] = None, _handle_cls=ReplicaJoinHandle) -> ReplicaJoinHandle:
        members = tuple(str(w) for w in member_worker_ids)
        if not members:
            raise ValueError("a DP replica must contain at least one worker")
        if len(members) != len(set(members)):
            raise ValueError("DP replica member_worker_ids must be unique")
        with self._lock:
            if self._closed:
                raise RuntimeError("ElasticHybridPool is closed")
            if replica_id in self._members:
                raise RuntimeError(f"replica is already registered: {replica_id}")
            workers = [self._pick(w, self._LENDABLE) for w in members]
            gen = self._generations.get(replica_id, 0) + 1
            self._generations[replica_id] = gen
            self._members[replica_id] = members
            for w in workers:
                w.transition(ReplicaRole.HYBRID_JOINING, target_core_id=target_core_id,
                             join_state=JoinState.REQUESTED, transition_generation=gen)
            self.gradient_domain.request_join(replica_id, target_core_id)
            fut = self._executor.submit(self._finish, replica_id, members, target_core_id, gen, activation_barrier,
                                        replica_activation_barrier, timeout_s)
            return _handle_cls(replica_id, members, target_core_id, fut, gen, self.cancel_replica_join)

    def join_training(self, worker_id: str, target_core_id: str, *,
                      activation_barrier: Optional[Callable[[str, str, int], None]] = None,
                      timeout_s: Optional[float] = None) -> JoinHandle:
        return self.join_replica(worker_id, [worker_id], target_core_id, activation_barrier=activation_barrier,
                                 timeout_s=timeout_s, _handle_cls=JoinHandle)

    def _rollback(self, replica_id: str, members: Tuple[str, ...], state: JoinState, generation: int) -> None:
        self.gradient_domain.detach(replica_id)
        for w in members:
            self._workers[w].transition(ReplicaRole.HYBRID_ROLLOUT, target_core_id=None, join_state=state,
                                        transition_generation=generation)

    def cancel_replica_join(self, replica_id: str, generation: int) -> None:
        with self._lock:
            if self._generations.get(replica_id) != generation:
                return
            self._generations[replica_id] = generation + 1
            self._rollback(replica_id, self._members.get(replica_id, ()), JoinState.CANCELLED, generation + 1)
            self._members.pop(replica_id, None)

    cancel_join = cancel_replica_join

    def release_replica_to_rollout(self, replica_id: str) -> None:
        with self._lock:
            members = self._members.get(replica_id)
            if not members:
                raise KeyError(f"unknown hybrid replica: {replica_id}")
            self._generations[replica_id] = self._generations.get(replica_id, 0) + 1
            self.gradient_domain.detach(replica_id)
            for w in members:
                if self._workers[w].role not in (ReplicaRole.HYBRID_TRAINING, ReplicaRole.HYBRID_JOINING):
                    raise RuntimeError(f"replica {replica_id} member {w} is {self._workers[w].role}")
                self._workers[w].transition(ReplicaRole.HYBRID_ROLLOUT)
            self._members.pop(replica_id, None)

    def release_to_rollout(self, worker_id: str) -> None:
        with self._lock:
            self._pick(worker_id, {ReplicaRole.HYBRID_TRAINING, ReplicaRole.HYBRID_JOINING})
            if worker_id in self._members:
                self.release_replica_to_rollout(worker_id)
            else:
                self._generations[worker_id] = self._generations.get(worker_id, 0) + 1
                self.gradient_domain.detach(worker_id)
                self._workers[worker_id].transition(ReplicaRole.HYBRID_ROLLOUT)

    def close(self) -> None:
        with self._lock:
            self._closed = True
        self._executor.shutdown(wait=False, cancel_futures=True)

    # -------------------------------------------------------------- background join
    def _check_current(self, replica_id: str, generation: int, deadline: Optional[float]) -> None:
        with self._lock:
            if self._closed:
                raise JoinCancelledError(f"join cancelled because pool is closed: {replica_id}")
            if self._generations.get(replica_id) != generation:
                raise JoinCancelledError(f"stale join generation for {replica_id}")
        if deadline is not None and time.monotonic() > deadline:
            raise TimeoutError(f"hybrid replica join timed out for {replica_id}")

    def _set_state(self, members, target, state: JoinState, **kw) -> None:
        with self._lock:
            for w in members:
                self._workers[w].transition(ReplicaRole.HYBRID_JOINING, target_core_id=target, join_state=state, **kw)

    def _finish(self, replica_id, members, target, generation, barrier, replica_barrier, timeout_s):
        deadline = time.monotonic() + max(float(timeout_s), 0.0) if timeout_s is not None else None
        try:
            self._check_current(replica_id, generation, deadline)
            self._set_state(members, target, JoinState.FETCHING_STATE)
            versions = tuple(int(self.snapshot_fetcher(w, target)) for w in members)
            self._check_current(replica_id, generation, deadline)
            if len(set(versions)) != 1:
                raise RuntimeError(f"DP replica {replica_id} fetched inconsistent state versions: {versions}")
            version = versions[0]
            self._set_state(members, target, JoinState.ZERO_SYNC, state_version=version)
            for _ in range(self.zero_sync_steps):
                time.sleep(0)
            self._check_current(replica_id, generation, deadline)
            if replica_barrier is not None or barrier is not None:
                self._set_state(members, target, JoinState.ACTIVATING, state_version=version,
                                transition_generation=generation)
                if replica_barrier is not None:
                    replica_barrier(replica_id, members, target, version)
                    self._check_current(replica_id, generation, deadline)
                else:
                    for w in members:
                        barrier(w, target, version)
                        self._check_current(replica_id, generation, deadline)
            self.gradient_domain.mark_active(replica_id)
            with self._lock:
                for w in members:
                    self._workers[w].transition(ReplicaRole.HYBRID_TRAINING, target_core_id=target,
                                                join_state=JoinState.ACTIVE, state_version=version,
                                                transition_generation=generation)
                return tuple(self._workers[w] for w in members)
        except JoinCancelledError:
            with self._lock:
                if self._generations.get(replica_id) == generation + 1:
                    self._rollback(replica_id, members, JoinState.CANCELLED, generation + 1)
            raise
        except Exception:
            with self._lock:
                if self._generations.get(replica_id) == generation:
                    self._rollback(replica_id, members, JoinState.FAILED, generation)
                    self._members.pop(replica_id, None)
            raise
