"""Elastic hybrid worker: one process per hybrid DP-replica rank.

Behaviour of the reference's ``scripts/elastic_hybrid_worker.py:121-198``:
load the training state snapshot of the target core replica, announce
readiness, then poll the task directory for ``<replica>.step_<N>.pt`` batches.
For each batch: recompute logprobs, compute the gradient payload (no
optimizer step), send it to the core's gradient endpoint and, in lockstep
mode, apply the post-reduce update that comes back so the replica's weights
stay identical to the core's.  Finished tasks are renamed ``.done``; failures
``.failed`` with the message in ``.error``.

Transports: ``tcp`` (``gradient_ipc``; lockstep capable) and ``peer``
(the native ``peer_xfer`` add into the core's registered buffer; one-way, so
lockstep then refreshes weights from the core's snapshot of the next task).

Core side helpers at the bottom: ``write_task`` (trainer -> worker batches)
and ``attach_gradient_server`` (payloads -> engine queue, reduced gradient ->
lockstep updates).

    python -m libra_b200.infra.elastic.worker --replica-id ehp_replica_rollout0 \\
        --target-core-id dp0 --snapshot-path logs/elastic_training_state/v3/rank_0.pt \\
        --gradient-host 127.0.0.1 --gradient-port 29600 --task-dir logs/elastic_training_tasks
"""

from __future__ import annotations

import argparse
import json
import os
import time
from pathlib import Path
from typing import Any, Dict, List, Optional

import torch


def parse_args(argv=None) -> argparse.Namespace:
    ap = argparse.ArgumentParser(description="libra_b200 elastic hybrid worker")
    ap.add_argument("--replica-id", required=True)
    ap.add_argument("--replica-rank", type=int, default=int(os.environ.get("RANK", "0")))
    ap.add_argument("--replica-world-size", type=int, default=int(os.environ.get("WORLD_SIZE", "1")))
    ap.add_argument("--target-core-id", required=True)
    ap.add_argument("--snapshot-path", default="")
    ap.add_argument("--gradient-host", default="127.0.0.1")
    ap.add_argument("--gradient-port", type=int, default=0)
    ap.add_argument("--authkey", default="")
    ap.add_argument("--gradient-transport", choices=["tcp", "peer"], default="tcp")
    ap.add_argument("--task-dir", required=True)
    ap.add_argument("--config", default="")
    ap.add_argument("--model", default="")
    ap.add_argument("--device", default="")
    ap.add_argument("--poll-interval", type=float, default=0.2)
    ap.add_argument("--no-lockstep", action="store_true")
    ap.add_argument("--initialize-only", action="store_true")
    ap.add_argument("--max-tasks", type=int, default=0, help="exit after this many tasks (0 = until shutdown)")
    return ap.parse_args(argv)


def _engine(args):
    from libra_b200.engine.train_engine import B200TrainEngine, create_train_engine

    if args.config:
        from libra_b200.config import AsyncRLConfig

        cfg = AsyncRLConfig.from_file(args.config)
        eng = create_train_engine(cfg)
        max_len = cfg.max_seq_length
    else:
        eng = B200TrainEngine(args.model or "qwen3-4b", use_distributed_optimizer=False)
        max_len = 2048
    if args.device:
        eng.device = torch.device(args.device)
    eng.initialize(max_seq_length=max_len)
    if args.snapshot_path and not args.initialize_only:
        eng.load_elastic_state_snapshot(args.snapshot_path)
    return eng


def _ready(task_dir: Path, args, snapshot: str) -> None:
    from libra_b200.infra.elastic.runtime_executor import write_json_atomic

    rank = int(os.environ.get("RANK", "0"))
    rec = {"replica_id": args.replica_id, "rank": rank, "pid": os.getpid(), "snapshot": snapshot,
           "ready_at": time.time()}
    write_json_atomic(task_dir / "ready" / f"{args.replica_id}.rank_{rank}.json", rec)
    if rank == 0:
        write_json_atomic(task_dir / "ready" / f"{args.replica_id}.json", rec)


def _send(args, payload, lockstep: bool):
    if args.gradient_transport == "peer":
        from libra_b200.infra.elastic.native_peer import NativePeerEndpoint, NativePeerGradientLane

        NativePeerGradientLane.send(NativePeerEndpoint(args.gradient_host, args.gradient_port, args.authkey), payload)
        return None
    from libra_b200.infra.elastic.gradient_ipc import ElasticGradientClient, GradientEndpoint

    client = ElasticGradientClient(GradientEndpoint(args.gradient_host, args.gradient_port, args.authkey))
    return client.send(payload, expect_update=lockstep)


def run_task(engine, args, task: Dict[str, Any], lockstep: bool, snapshot: str) -> str:
    snap = str(task.get("snapshot_path", "") or "")
    if snap and snap != snapshot:
        engine.load_elastic_state_snapshot(snap)
        snapshot = snap
    trajs = task["trajectories"]
    engine.recompute_logprobs(trajs)
    payload = engine.compute_gradient_payload(trajs, replica_id=args.replica_id, target_core_id=args.target_core_id,
                                              step=int(task["step"]), membership_epoch=int(task["membership_epoch"]),
                                              replica_rank=args.replica_rank,
                                              replica_world_size=args.replica_world_size)
    update = _send(args, payload, lockstep)
    if update is not None:
        if (update.replica_id, update.step, update.membership_epoch) != (payload.replica_id, payload.step,
                                                                        payload.membership_epoch):
            raise RuntimeError("received a post-reduce update for another replica, step or epoch")
        (grad,) = update.tensors
        engine.apply_gradient_update(grad)
        engine.set_version(int(update.state_version) + 1)
    return snapshot


def main(argv=None) -> int:
    args = parse_args(argv)
    task_dir = Path(args.task_dir)
    task_dir.mkdir(parents=True, exist_ok=True)
    if args.snapshot_path and not args.initialize_only and not os.path.exists(args.snapshot_path):
        raise FileNotFoundError(f"snapshot does not exist: {args.snapshot_path}")
    engine = _engine(args)
    _ready(task_dir, args, args.snapshot_path)
    if args.initialize_only:
        return 0
    lockstep = not args.no_lockstep and args.gradient_transport == "tcp"
    snapshot = args.snapshot_path
    done = 0
    while True:
        tasks = sorted(task_dir.glob(f"{args.replica_id}.step_*.pt"), key=lambda p: int(p.stem.rsplit("_", 1)[1]))
        if not tasks:
            time.sleep(args.poll_interval)
            continue
        for path in tasks:
            try:
                task = torch.load(path, map_location="cpu", weights_only=True)
                if task.get("shutdown"):
                    path.rename(path.with_suffix(".pt.done"))
                    return 0
                snapshot = run_task(engine, args, task, lockstep, snapshot)
                if torch.distributed.is_available() and torch.distributed.is_initialized():
                    torch.distributed.barrier()
                if int(os.environ.get("RANK", "0")) == 0:
                    path.rename(path.with_suffix(".pt.done"))
            except Exception as exc:  # noqa: BLE001 - recorded next to the task
                path.with_suffix(".pt.error").write_text(str(exc), encoding="utf-8")
                path.rename(path.with_suffix(".pt.failed"))
            done += 1
            if args.max_tasks and done >= args.max_tasks:
                return 0


# ============================================================================ core side
def write_task(task_dir: str, replica_id: str, step: int, trajectories: List[Dict[str, Any]], *, state_version: int,
               membership_epoch: int, snapshot_path: str = "") -> Path:
    """Hand one batch to a hybrid replica (atomic rename; tensors + primitives only)."""
    d = Path(task_dir)
    d.mkdir(parents=True, exist_ok=True)
    keep = [{k: v for k, v in t.items() if isinstance(v, (torch.Tensor, int, float, str, bool))} for t in trajectories]
    path = d / f"{replica_id}.step_{int(step)}.pt"
    tmp = d / f".{path.name}.tmp"
    torch.save({"trajectories": keep, "step": int(step), "state_version": int(state_version),
                "membership_epoch": int(membership_epoch), "snapshot_path": snapshot_path}, tmp)
    os.replace(tmp, path)
    return path


def write_shutdown(task_dir: str, replica_id: str, step: int = 1 << 30) -> Path:
    d = Path(task_dir)
    d.mkdir(parents=True, exist_ok=True)
    path = d / f"{replica_id}.step_{int(step)}.pt"
    torch.save({"shutdown": True}, path)
    return path


def attach_gradient_server(engine, *, host: str = "127.0.0.1", port: int = 0, authkey: str = ""):
    """Receive hybrid payloads into ``engine``'s queue and publish each step's
    reduced gradient as the lockstep update of every active hybrid replica."""
    from libra_b200.infra.elastic.gradient_ipc import ElasticGradientServer, GradientUpdate

    server = ElasticGradientServer(host=host, port=port, authkey=authkey,
                                   on_payload=engine.enqueue_hybrid_gradient_payload)
    server.start()

    def publish(full_grad: torch.Tensor, step: int, version: int) -> None:
        domain = engine.elastic_gradient_domain
        if domain is None:
            return
        cpu = full_grad.detach().to("cpu")
        for rid in domain.active_hybrid_ids():
            server.publish_update(GradientUpdate(rid, (cpu,), step, version, domain.membership_epoch(rid)))

    engine.elastic_update_publisher = publish
    return server


def write_endpoint(task_dir: str, rank: int, endpoint, **extra) -> Path:
    """Record a core rank's gradient endpoint for workers to discover."""
    from libra_b200.infra.elastic.runtime_executor import write_json_atomic

    path = Path(task_dir) / "core_endpoints" / f"rank_{rank}.json"
    write_json_atomic(path, {"host": endpoint.host, "port": endpoint.port, "authkey": endpoint.authkey, **extra})
    return path


if __name__ == "__main__":
    raise SystemExit(main())
