"""KV-cache migration between rollout instances of different TP degree.

When C-MLFQ moves a multi-turn request to another bucket its KV cache is either
migrated or recomputed by a prefill on the target (reference
``infra/scheduling/cmlfq_migration.py``: CPU offload -> head-dim reshard ->
reload, with a profiled/heuristic migrate-vs-recompute choice).

B200 design: every rollout instance lives on the same NVSwitch box, so the KV
slices go **GPU to GPU** (``Tensor.to(peer_device)`` is a copy-engine transfer
over NVLink) without a host round trip; the host-staged path is kept for
CPU-only runs and tests.  KV layout per layer: [tokens, kv_heads, head_dim]
(the reference's [batch, seq, heads, dim] is handled by ``dim``); resharding
splits/merges contiguous head groups (TP rank r owns heads
[r*H/tp, (r+1)*H/tp)).
"""

from __future__ import annotations

import json
import logging
import os
from dataclasses import asdict, dataclass
from typing import Dict, List, Optional, Tuple

import torch

log = logging.getLogger(__name__)

LayerKV = Dict[int, Tuple[torch.Tensor, torch.Tensor]]


@dataclass
class KVCacheShard:
    gpu_id: int
    tensor: torch.Tensor
    tp_rank: int


@dataclass
class MigrationLatencyProfile:
    source_tp: int
    target_tp: int
    seq_len: int
    offload_ms: float
    reshard_ms: float
    network_ms: float
    reload_ms: float
    total_migration_ms: float
    recompute_prefill_ms: float


def reshard_heads(shards: List[torch.Tensor], target_tp: int, dim: int) -> List[torch.Tensor]:
    """Re-split per-rank head shards (concatenated along ``dim``) for ``target_tp`` ranks."""
    source_tp = len(shards)
    if source_tp <= 0 or target_tp <= 0:
        raise ValueError("source_tp and target_tp must be positive")
    if source_tp % target_tp and target_tp % source_tp:
        raise ValueError("source_tp and target_tp must be integer multiples")
    total = sum(s.shape[dim] for s in shards)
    if total % target_tp or total % source_tp:
        raise ValueError(f"dimension size {total} must be divisible by source_tp={source_tp} and target_tp={target_tp}")
    if target_tp >= source_tp:
        ratio = target_tp // source_tp
        return [p.contiguous() for s in shards for p in torch.chunk(s, ratio, dim=dim)]
    ratio = source_tp // target_tp
    return [torch.cat(shards[t * ratio:(t + 1) * ratio], dim=dim).contiguous() for t in range(target_tp)]


class KVCacheManager:
    """Stages a request's KV, reshards it and places it on target devices."""

    def __init__(self):
        self._staged: Dict[str, LayerKV] = {}

    def offload(self, request_id: str, kv_cache: LayerKV, to_host: bool = True) -> LayerKV:
        staged = {}
        for layer, (k, v) in kv_cache.items():
            if to_host:
                k, v = k.detach().cpu(), v.detach().cpu()
                if torch.cuda.is_available():
                    k, v = k.pin_memory(), v.pin_memory()
            staged[layer] = (k.detach(), v.detach())
        self._staged[request_id] = staged
        return staged

    def reshard_kv_cache(self, request_id: str, source_tp: int, target_tp: int, dim: int = 1) -> Dict[int, Dict[int, Tuple]]:
        staged = self._staged.get(request_id)
        if staged is None:
            raise ValueError(f"Request {request_id} KV cache not found in staging memory")
        out = {}
        for layer, (k, v) in staged.items():
            ks = reshard_heads(list(torch.chunk(k, source_tp, dim=dim)), target_tp, dim)
            vs = reshard_heads(list(torch.chunk(v, source_tp, dim=dim)), target_tp, dim)
            out[layer] = {r: (ks[r], vs[r]) for r in range(target_tp)}
        return out

    def reload(self, request_id: str, target_device, layer_shards: Dict[int, Tuple]) -> LayerKV:
        dev = torch.device(target_device) if not isinstance(target_device, int) else torch.device("cuda", target_device)
        return {layer: (k.to(dev, non_blocking=True), v.to(dev, non_blocking=True))
                for layer, (k, v) in layer_shards.items()}

    def release(self, request_id: str) -> None:
        self._staged.pop(request_id, None)

    def clear(self) -> None:
        self._staged.clear()


class MigrationCostProfiler:
    """Measured (source_tp, target_tp, seq_len) costs with a nearest-length lookup;
    without a profile, an NVLink/compute model decides migrate vs recompute."""

    def __init__(self, profile_path: str = "", nvlink_bw: float = 7.7e11, kv_bytes_per_token: float = 0.0,
                 prefill_tokens_per_s: float = 0.0):
        self._profile: Dict[Tuple[int, int, int], MigrationLatencyProfile] = {}
        self._profile_path = profile_path
        self.nvlink_bw = nvlink_bw
        self.kv_bytes_per_token = kv_bytes_per_token
        self.prefill_tokens_per_s = prefill_tokens_per_s
        if profile_path and os.path.exists(profile_path):
            self.load_profile(profile_path)

    def record_measurement(self, source_tp: int, target_tp: int, seq_len: int, offload_ms: float, reshard_ms: float,
                           network_ms: float, reload_ms: float, recompute_prefill_ms: float) -> None:
        self._profile[(source_tp, target_tp, seq_len)] = MigrationLatencyProfile(
            source_tp, target_tp, seq_len, offload_ms, reshard_ms, network_ms, reload_ms,
            offload_ms + reshard_ms + network_ms + reload_ms, recompute_prefill_ms)

    def _lookup(self, source_tp: int, target_tp: int, seq_len: int) -> Optional[MigrationLatencyProfile]:
        hit = self._profile.get((source_tp, target_tp, seq_len))
        if hit is not None:
            return hit
        same_pair = [p for (s, t, _), p in self._profile.items() if s == source_tp and t == target_tp]
        return min(same_pair, key=lambda p: abs(p.seq_len - seq_len)) if same_pair else None

    def decide_migration_path(self, source_tp: int, target_tp: int, seq_len: int,
                              is_cross_node: bool = False) -> Tuple[str, float]:
        prof = self._lookup(source_tp, target_tp, seq_len)
        if prof is not None:
            move = prof.total_migration_ms if is_cross_node else prof.offload_ms + prof.reshard_ms + prof.reload_ms
            return ("migrate", move) if move <= prof.recompute_prefill_ms else ("recompute", prof.recompute_prefill_ms)
        if self.kv_bytes_per_token > 0 and self.prefill_tokens_per_s > 0:
            move_ms = 1e3 * seq_len * self.kv_bytes_per_token / self.nvlink_bw + 0.05
            redo_ms = 1e3 * seq_len / self.prefill_tokens_per_s
            return ("migrate", move_ms) if move_ms <= redo_ms else ("recompute", redo_ms)
        crossover = 2048 if is_cross_node else 4096
        return ("recompute", seq_len * 0.5) if seq_len <= crossover else ("migrate", seq_len * 0.3)

    def save_profile(self, path: str) -> None:
        with open(path, "w") as fh:
            json.dump([asdict(p) for p in self._profile.values()], fh, indent=2)

    def load_profile(self, path: str) -> None:
        with open(path) as fh:
            for e in json.load(fh):
                self._profile[(e["source_tp"], e["target_tp"], e["seq_len"])] = MigrationLatencyProfile(**e)


class CMLFQMigrationCoordinator:
    def __init__(self, kv_cache_manager: Optional[KVCacheManager] = None,
                 cost_profiler: Optional[MigrationCostProfiler] = None):
        self.kv_manager = kv_cache_manager or KVCacheManager()
        self.profiler = cost_profiler or MigrationCostProfiler()

    def execute_full_migration(self, request_id: str, source_instance_index: int, source_tp: int,
                               target_instance_index: int, target_tp: int, kv_cache: LayerKV, seq_len: int,
                               is_cross_node: bool = False, target_rank: Optional[int] = None,
                               target_device=None) -> LayerKV:
        on_gpu = any(k.is_cuda for k, _ in kv_cache.values())
        self.kv_manager.offload(request_id, kv_cache, to_host=is_cross_node or not on_gpu)
        resharded = self.kv_manager.reshard_kv_cache(request_id, source_tp, target_tp)
        rank = target_instance_index % max(target_tp, 1) if target_rank is None else target_rank
        shards = {layer: per_rank[rank] for layer, per_rank in resharded.items()}
        device = target_device if target_device is not None else (
            torch.device("cuda", target_instance_index) if on_gpu else torch.device("cpu"))
        out = self.kv_manager.reload(request_id, device, shards)
        self.kv_manager.release(request_id)
        return out

    def decide_and_execute(self, request_id: str, source_instance_index: int, source_tp: int,
                           target_instance_index: int, target_tp: int, kv_cache: Optional[LayerKV], seq_len: int,
                           is_cross_node: bool = False):
        path, cost = self.profiler.decide_migration_path(source_tp, target_tp, seq_len, is_cross_node)
        if path == "migrate" and kv_cache:
            return "migrate", self.execute_full_migration(request_id, source_instance_index, source_tp,
                                                          target_instance_index, target_tp, kv_cache, seq_len,
                                                          is_cross_node)
        return "recompute", None
