"""Peer-memory weight sync: trainer shards -> rollout instance buffers over NVLink.

Every trainer tensor-parallel rank keeps its parameters in one flat bf16
buffer.  ``publish`` (collective over the trainer's TP group) describes those
buffers as plain JSON — base64 CUDA IPC handle, byte offset, dtype, element
count, device — so the request can cross an HTTP hop without pickled objects.
A rollout rank maps the buffers into its own GPU context and runs the
``weight_reshard`` kernel with the copy plan for its (TP degree, rank): each
piece of its slice is read once from the trainer rank that owns it, over
NVLink, and written straight into its flat weight buffer (the reference
gathers full tensors on trainer rank 0 and broadcasts them through a separate
NCCL communicator, ``infra/sync/nccl_weight_sync.py:126-197``).

Plans and mappings are cached, so a steady-state sync is one kernel launch.
"""

from __future__ import annotations

import time
from typing import Any, Dict, List, Optional, Sequence, Tuple

import torch
import torch.distributed as dist

from libra_b200.infra.sync.reshard import DeviceReshard, apply_plan, build_plan, export_buffer, open_buffer
from libra_b200.models.qwen3 import Qwen3Config

_PLANS: Dict[Tuple, DeviceReshard] = {}


def publish(engine, group=None) -> Dict[str, Any]:
    """Trainer side (collective over the TP group): the JSON request every
    rollout rank needs to pull its slice of the current weights."""
    mine = export_buffer(engine.flat_param)
    tp = int(getattr(engine, "tp_size", 1))
    group = group if group is not None else getattr(engine, "tp_group", None)
    if tp > 1:
        sources: List[Any] = [None] * tp
        dist.all_gather_object(sources, mine, group=group)
    else:
        sources = [mine]
    return {"kind": "peer", "src_tp": tp, "sources": sources, "cfg": engine.cfg.to_dict(),
            "version": int(engine.get_version())}


def _validate(request: Dict[str, Any]) -> None:
    src = request.get("sources")
    if not isinstance(src, list) or not src or not isinstance(request.get("src_tp"), int) \
            or len(src) != request["src_tp"]:
        raise ValueError("peer weight request needs 'src_tp' and one source description per trainer TP rank")
    for d in src:
        if not isinstance(d, dict) or d.get("dtype") not in ("bfloat16", "float32"):
            raise ValueError("peer weight sources must be bf16 or fp32 buffer descriptions")


def receive_peer_weights(request: Dict[str, Any], dst_flat: torch.Tensor, cfg: Qwen3Config, tp: int = 1,
                         rank: int = 0) -> int:
    """Rollout side: reshard the published trainer buffers into ``dst_flat``
    (this rank's flat bf16 weights, TP degree ``tp``).  Returns bytes written."""
    _validate(request)
    dev = dst_flat.device
    addrs = [open_buffer(d, dev) for d in request["sources"]]
    esz = [4 if d["dtype"] == "float32" else 2 for d in request["sources"]]
    key = (tuple(addrs), int(dst_flat.data_ptr()), int(request["src_tp"]), int(tp), int(rank))
    plan = _PLANS.get(key)
    if plan is None:
        plan = DeviceReshard(cfg, int(request["src_tp"]), tp, rank, addrs, dst_flat, esz)
        _PLANS[key] = plan
    with torch.cuda.device(dev):
        moved = plan.run()
        torch.cuda.current_stream(dev).synchronize()
    return moved


class PeerWeightSync:
    """Trainer side of the peer path, plus the in-process variant for rollout
    engines that live in the trainer's processes."""

    def __init__(self, **_):
        self.last_seconds = 0.0
        self.last_bytes = 0

    def publish(self, engine) -> Dict[str, Any]:
        return publish(engine)

    def push_local(self, engine, targets: Sequence[Tuple[torch.Tensor, int, int]]) -> Tuple[float, int]:
        """Reshard this trainer rank's weights into in-process targets, given as
        (flat bf16 buffer, TP degree, TP rank); sources and targets must be
        reachable from the target's GPU (the same GPU, or peer access)."""
        t0 = time.perf_counter()
        moved = 0
        tp = int(getattr(engine, "tp_size", 1))
        if tp != 1:
            raise ValueError("push_local reads one trainer shard; use publish() for a TP-sharded trainer")
        for flat, dst_tp, dst_rank in targets:
            if flat.is_cuda:
                key = ((int(engine.flat_param.data_ptr()),), int(flat.data_ptr()), 1, int(dst_tp), int(dst_rank))
                plan = _PLANS.get(key)
                if plan is None:
                    plan = DeviceReshard(engine.cfg, 1, dst_tp, dst_rank, [int(engine.flat_param.data_ptr())], flat)
                    _PLANS[key] = plan
                moved += plan.run()
            else:
                rects = build_plan(engine.cfg, 1, dst_tp, dst_rank)
                apply_plan(rects, [engine.flat_param], flat)
                moved += sum(r.rows * r.row_elems for r in rects) * 2
        if engine.flat_param.is_cuda:
            torch.cuda.synchronize()
        self.last_seconds, self.last_bytes = time.perf_counter() - t0, moved
        return self.last_seconds, moved


def clear_plans() -> None:
    _PLANS.clear()
