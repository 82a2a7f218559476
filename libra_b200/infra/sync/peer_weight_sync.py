"""Peer-memory weight sync: trainer shards -> rollout instance buffers over NVLink.

The trainer keeps its parameters in one flat bf16 buffer; ``export_handle``
wraps it in a CUDA IPC handle (plus the parameter layout).  A rollout process
on the same box ``open_handle``s it - the mapping is a peer view of the
trainer GPU's memory - and ``copy_resharded`` copies, for every parameter, the
slice its tensor-parallel rank owns into its local buffers; the copies run on
the copy engines over NVLink, there is no host staging and no full-tensor
broadcast (the reference broadcasts whole HF tensors from trainer rank 0
through a separate NCCL communicator, ``infra/sync/nccl_weight_sync.py``).

TP slicing rules (column-parallel along output rows, row-parallel along input
columns, vocabulary split for the embedding / LM head) are the ones of
``models.qwen3.param_shapes``.
"""

from __future__ import annotations

import base64
import pickle
import time
from typing import Any, Dict, Optional, Tuple

import torch

from libra_b200.models.qwen3 import ParamLayout, Qwen3Config, param_shapes

COLUMN = ("qkv_proj", "gate_up_proj", "experts.w1", "embed_tokens", "lm_head", "router")
ROW = ("o_proj", "down_proj", "experts.w2")


def export_handle(flat: torch.Tensor, layout: ParamLayout, cfg: Qwen3Config, version: int) -> Dict[str, Any]:
    """Serialisable description of the trainer's flat buffer (CUDA IPC)."""
    from torch.multiprocessing.reductions import reduce_tensor

    fn, args = reduce_tensor(flat)
    blob = base64.b64encode(pickle.dumps((fn, args))).decode()
    return {"ipc": blob, "layout": {n: list(s) for n, s in layout.shapes.items()}, "order": layout.order,
            "offsets": layout.offsets, "cfg": cfg.to_dict(), "version": int(version), "numel": flat.numel()}


def open_handle(handle: Dict[str, Any]) -> torch.Tensor:
    fn, args = pickle.loads(base64.b64decode(handle["ipc"]))
    return fn(*args)


def tp_slice(name: str, full: torch.Tensor, cfg: Qwen3Config, tp: int, rank: int) -> torch.Tensor:
    """The part of a full (TP=1) parameter that rank ``rank`` of a TP group owns."""
    if tp == 1:
        return full
    base = name.split(".", 2)[-1] if name.startswith("layers.") else name
    if base == "qkv_proj":
        D, nq, nkv = cfg.head_dim, cfg.num_attention_heads, cfg.num_key_value_heads
        q, k, v = full[:nq * D], full[nq * D:(nq + nkv) * D], full[(nq + nkv) * D:]
        nq_l = nq // tp
        kv_l = max(1, nkv // tp)
        kv_rank = rank * nkv // tp if nkv >= tp else rank * nkv // tp
        return torch.cat([q[rank * nq_l * D:(rank + 1) * nq_l * D],
                          k[kv_rank * D:(kv_rank + kv_l) * D], v[kv_rank * D:(kv_rank + kv_l) * D]])
    if base in ("gate_up_proj",):
        F = full.shape[0] // 2
        Fl = F // tp
        return torch.cat([full[rank * Fl:(rank + 1) * Fl], full[F + rank * Fl:F + (rank + 1) * Fl]])
    if base == "experts.w1":
        F = full.shape[1] // 2
        Fl = F // tp
        return torch.cat([full[:, rank * Fl:(rank + 1) * Fl], full[:, F + rank * Fl:F + (rank + 1) * Fl]], dim=1)
    if base in ("embed_tokens", "lm_head"):
        Vl = full.shape[0] // tp
        return full[rank * Vl:(rank + 1) * Vl]
    if base in ("o_proj", "down_proj"):
        C = full.shape[1] // tp
        return full[:, rank * C:(rank + 1) * C]
    if base == "experts.w2":
        C = full.shape[2] // tp
        return full[:, :, rank * C:(rank + 1) * C]
    return full  # norms, router: replicated


def copy_resharded(src_flat: torch.Tensor, handle: Dict[str, Any], dst: Dict[str, torch.Tensor], tp: int = 1,
                   rank: int = 0) -> int:
    """Copy every parameter's TP slice from the trainer's flat buffer into ``dst``; returns bytes moved."""
    cfg = Qwen3Config(**handle["cfg"])
    moved = 0
    with torch.no_grad():
        for name in handle["order"]:
            if name not in dst:
                continue
            shape = tuple(handle["layout"][name])
            off = int(handle["offsets"][name])
            n = 1
            for s in shape:
                n *= s
            full = src_flat[off:off + n].view(shape)
            part = tp_slice(name, full, cfg, tp, rank)
            dst[name].copy_(part, non_blocking=True)
            moved += part.numel() * part.element_size()
    return moved


def receive_peer_weights(request: Dict[str, Any], holder_params: Dict[str, torch.Tensor],
                         tp: int = 1, rank: int = 0) -> Dict[str, torch.Tensor]:
    """Server-side entry: map the trainer's buffer and pull into a fresh copy of the holder's params."""
    src = open_handle(request["handle"])
    params = {k: torch.empty_like(v) for k, v in holder_params.items()}
    copy_resharded(src, request["handle"], params, tp, rank)
    torch.cuda.synchronize()
    return params


class PeerWeightSync:
    """Trainer side: publish the flat buffer handle; in-process consumers copy directly."""

    def __init__(self, **_):
        self.last_seconds = 0.0
        self.last_bytes = 0

    def publish(self, engine) -> Dict[str, Any]:
        return export_handle(engine.flat_param, engine.layout, engine.cfg, engine.get_version())

    def push_local(self, engine, targets, tp: int = 1) -> Tuple[float, int]:
        """Copy into in-process targets: list of (param dict, tp_rank)."""
        t0 = time.perf_counter()
        handle = {"layout": {n: list(s) for n, s in engine.layout.shapes.items()}, "order": engine.layout.order,
                  "offsets": engine.layout.offsets, "cfg": engine.cfg.to_dict()}
        moved = 0
        for params, r in targets:
            moved += copy_resharded(engine.flat_param, handle, params, tp, r)
        if engine.flat_param.is_cuda:
            torch.cuda.synchronize()
        self.last_seconds, self.last_bytes = time.perf_counter() - t0, moved
        return self.last_seconds, moved
