"""Megatron-Core ``torch_dist`` model-space layout of the engine's tensors.

A Megatron-Core distributed checkpoint stores every tensor once, in its global
(unsharded) shape, as a torch.distributed.checkpoint (DCP) tensor made of
chunks: each rank writes the chunks it holds at their global offsets and DCP
keeps one copy of chunks that several ranks hold (data-parallel replicas,
replicated norms).  The conventions this module follows (the reference saves
through Megatron-Core, ``engine/megatron_core_checkpointing.py:59-137``):

* transformer layers are stacked on a leading layer axis under one key per
  tensor kind, ``decoder.layers.self_attention.linear_qkv.weight`` of shape
  ``[num_layers, ...]``; a pipeline stage writes the rows of its layers;
* column-parallel weights (QKV, fc1, vocabulary rows) and row-parallel weights
  (proj, fc2) are split along the same axis as the tensor-parallel layer; the
  QKV rows are in per-query-group order ``[group][q heads, k, v]`` so that a
  rank's heads form contiguous row blocks, and fc1 is ``[all gate; all up]``,
  i.e. a rank holds two row blocks of it;
* experts are stacked on an expert axis after the layer axis,
  ``decoder.layers.mlp.experts.experts.linear_fc1.weight`` of shape
  ``[num_layers, num_experts, 2*ffn, hidden]``; an expert-parallel rank writes
  its experts' rows;
* the distributed optimizer's state uses the same global shapes under
  ``optimizer.state.{fp32_param,exp_avg,exp_avg_sq}.<model key>`` (the
  fully-sharded model-space format).

``param_chunks`` maps one local parameter to its chunks.  Every chunk is a view
of the local tensor (``narrow`` plus leading singleton axes), so loading writes
straight into the engine's buffers.  ``ChunkSavePlanner`` / ``ChunkLoadPlanner``
hand the chunks to DCP as write and read items.
"""

from __future__ import annotations

import dataclasses
import re
from dataclasses import dataclass
from typing import Dict, List, Sequence, Tuple

import torch
from torch.distributed.checkpoint.default_planner import DefaultLoadPlanner, DefaultSavePlanner
from torch.distributed.checkpoint.metadata import ChunkStorageMetadata, MetadataIndex, TensorProperties
from torch.distributed.checkpoint.planner import TensorWriteData, WriteItem, WriteItemType
from torch.distributed.checkpoint.planner_helpers import create_read_items_for_chunk_list

from libra_b200.models.qwen3 import Qwen3Config

OPTIM_KINDS = ("fp32_param", "exp_avg", "exp_avg_sq")

_LAYER_KEYS = {
    "input_layernorm": "input_layernorm.weight",
    "q_norm": "self_attention.q_layernorm.weight",
    "k_norm": "self_attention.k_layernorm.weight",
    "post_attention_layernorm": "pre_mlp_layernorm.weight",
    "qkv_proj": "self_attention.linear_qkv.weight",
    "o_proj": "self_attention.linear_proj.weight",
    "gate_up_proj": "mlp.linear_fc1.weight",
    "down_proj": "mlp.linear_fc2.weight",
    "router": "mlp.router.weight",
    "experts.w1": "mlp.experts.experts.linear_fc1.weight",
    "experts.w2": "mlp.experts.experts.linear_fc2.weight",
}
_TOP_KEYS = {
    "embed_tokens": "embedding.word_embeddings.weight",
    "lm_head": "output_layer.weight",
    "norm": "decoder.final_layernorm.weight",
}
_LAYER_RE = re.compile(r"^layers\.(\d+)\.(.+)$")


@dataclass(frozen=True)
class Chunk:
    """One chunk of a global tensor: ``key`` of global shape ``gshape``; the
    chunk starts at ``offsets`` and is the local tensor narrowed by ``narrows``
    (``(dim, start, length)`` each, in the local tensor's dims) with ``prepend``
    leading singleton axes (layer / expert axes)."""

    key: str
    gshape: Tuple[int, ...]
    offsets: Tuple[int, ...]
    narrows: Tuple[Tuple[int, int, int], ...]
    prepend: int

    def view(self, local: torch.Tensor) -> torch.Tensor:
        t = local
        for dim, start, length in self.narrows:
            t = t.narrow(dim, start, length)
        for _ in range(self.prepend):
            t = t.unsqueeze(0)
        return t


@dataclass(frozen=True)
class ShardInfo:
    """Which slice of the model a rank's parameters are."""

    tp_size: int = 1
    tp_rank: int = 0
    ep_size: int = 1
    ep_rank: int = 0


def mcore_key(name: str) -> str:
    """Model-space (stacked) key of an engine parameter name."""
    m = _LAYER_RE.match(name)
    if m:
        return "decoder.layers." + _LAYER_KEYS[m.group(2)]
    return _TOP_KEYS[name]


def _qkv_chunks(key, layer, L, cfg: Qwen3Config, info: ShardInfo, H) -> List[Chunk]:
    """QKV rows: the local tensor is [this rank's q heads | its k heads | its v heads];
    globally the rows are per query group [q heads of the group, k, v]."""
    D = cfg.head_dim
    nq, nkv = cfg.num_attention_heads, cfg.num_key_value_heads
    per = nq // nkv
    tp, r = info.tp_size, info.tp_rank
    nq_l, kv_l = nq // tp, max(1, nkv // tp)
    kv0 = r * nkv // tp
    rows_g = (nq + 2 * nkv) * D
    out = []
    # q heads: consecutive heads of one group are contiguous both locally and globally
    lq = 0
    while lq < nq_l:
        h = r * nq_l + lq
        g, j = divmod(h, per)
        n = min(nq_l - lq, per - j)
        out.append(Chunk(key, (L, rows_g, H), (layer, (g * (per + 2) + j) * D, 0), ((0, lq * D, n * D),), 1))
        lq += n
    for lk in range(kv_l):
        g = kv0 + lk
        out.append(Chunk(key, (L, rows_g, H), (layer, (g * (per + 2) + per) * D, 0), ((0, (nq_l + lk) * D, D),), 1))
        out.append(Chunk(key, (L, rows_g, H), (layer, (g * (per + 2) + per + 1) * D, 0),
                         ((0, (nq_l + kv_l + lk) * D, D),), 1))
    return out


def param_chunks(name: str, shape: Sequence[int], cfg: Qwen3Config, info: ShardInfo) -> List[Chunk]:
    """The model-space chunks that one local parameter (of local ``shape``) fills."""
    tp, r = info.tp_size, info.tp_rank
    key = mcore_key(name)
    m = _LAYER_RE.match(name)
    if not m:
        if name in ("embed_tokens", "lm_head"):
            V_l, H = shape
            return [Chunk(key, (V_l * tp, H), (r * V_l, 0), (), 0)]
        return [Chunk(key, tuple(shape), (0,) * len(shape), (), 0)]
    layer, kind = int(m.group(1)), m.group(2)
    L = cfg.num_hidden_layers
    if kind == "qkv_proj":
        return _qkv_chunks(key, layer, L, cfg, info, shape[1])
    if kind in ("o_proj", "down_proj"):
        H, cols = shape
        return [Chunk(key, (L, H, cols * tp), (layer, 0, r * cols), (), 1)]
    if kind == "gate_up_proj":
        F2, H = shape
        Fl = F2 // 2
        F = Fl * tp
        return [Chunk(key, (L, 2 * F, H), (layer, r * Fl, 0), ((0, 0, Fl),), 1),
                Chunk(key, (L, 2 * F, H), (layer, F + r * Fl, 0), ((0, Fl, Fl),), 1)]
    if kind == "experts.w1":
        El, F2, H = shape
        Fl = F2 // 2
        F, E, e0 = Fl * tp, El * info.ep_size, info.ep_rank * El
        if tp == 1:
            return [Chunk(key, (L, E, 2 * F, H), (layer, e0, 0, 0), (), 1)]
        return [Chunk(key, (L, E, 2 * F, H), (layer, e0, r * Fl, 0), ((1, 0, Fl),), 1),
                Chunk(key, (L, E, 2 * F, H), (layer, e0, F + r * Fl, 0), ((1, Fl, Fl),), 1)]
    if kind == "experts.w2":
        El, H, Fl = shape
        E, e0 = El * info.ep_size, info.ep_rank * El
        return [Chunk(key, (L, E, H, Fl * tp), (layer, e0, 0, r * Fl), (), 1)]
    # replicated per-layer tensors (norms, router)
    return [Chunk(key, (L, *shape), (layer,) + (0,) * len(shape), (), 1)]


def model_space_items(tensors: Dict[str, torch.Tensor], cfg: Qwen3Config, info: ShardInfo,
                      prefix: str = "") -> Dict[str, List[Tuple[Chunk, torch.Tensor]]]:
    """key -> [(chunk, chunk view)] for local tensors shaped like the engine's
    parameters (``prefix`` is prepended to every key)."""
    out: Dict[str, List[Tuple[Chunk, torch.Tensor]]] = {}
    for name, t in tensors.items():
        for c in param_chunks(name, t.shape, cfg, info):
            c = dataclasses.replace(c, key=prefix + c.key)
            out.setdefault(c.key, []).append((c, c.view(t)))
    return out


def _write_item(c: Chunk, t: torch.Tensor) -> WriteItem:
    return WriteItem(index=MetadataIndex(c.key, torch.Size(c.offsets)), type=WriteItemType.SHARD,
                     tensor_data=TensorWriteData(chunk=ChunkStorageMetadata(offsets=torch.Size(c.offsets),
                                                                            sizes=t.shape),
                                                 properties=TensorProperties.create_from_tensor(t),
                                                 size=torch.Size(c.gshape)))


class ChunkSavePlanner(DefaultSavePlanner):
    """Saves the plain state dict as usual plus the given chunked tensors (DCP
    keeps one copy of a chunk that several ranks write at the same offset)."""

    def __init__(self, chunks: Dict[str, List[Tuple[Chunk, torch.Tensor]]]):
        super().__init__()
        self._chunks = {(c.key, tuple(c.offsets)): t for items in chunks.values() for c, t in items}
        self._items = [_write_item(c, t) for items in chunks.values() for c, t in items]

    def create_local_plan(self):
        plan = super().create_local_plan()
        self.plan = dataclasses.replace(plan, items=list(plan.items) + self._items)
        return self.plan

    def lookup_object(self, index: MetadataIndex):
        t = self._chunks.get((index.fqn, tuple(index.offset or ())))
        if t is not None:
            return t.detach().contiguous()
        return super().lookup_object(index)


class ChunkLoadPlanner(DefaultLoadPlanner):
    """Loads the plain state dict as usual and fills the given chunk views
    (any saved chunking is read back: DCP reshards by overlap)."""

    def __init__(self, chunks: Dict[str, List[Tuple[Chunk, torch.Tensor]]]):
        super().__init__()
        self._chunks = chunks
        self._views = {(c.key, tuple(c.offsets)): t for items in chunks.values() for c, t in items}

    def create_local_plan(self):
        plan = super().create_local_plan()
        items = list(plan.items)
        for key, pairs in self._chunks.items():
            md = self.metadata.state_dict_metadata.get(key)
            if md is None:
                raise RuntimeError(f"Missing key in checkpoint: {key}")
            if tuple(md.size) != tuple(pairs[0][0].gshape):
                raise ValueError(f"{key}: saved shape {tuple(md.size)} but this model needs {pairs[0][0].gshape}")
            local = [ChunkStorageMetadata(offsets=torch.Size(c.offsets), sizes=t.shape) for c, t in pairs]
            items += create_read_items_for_chunk_list(key, md, local)
        self.plan = dataclasses.replace(plan, items=items)
        return self.plan

    def lookup_tensor(self, index: MetadataIndex) -> torch.Tensor:
        t = self._views.get((index.fqn, tuple(index.offset or ())))
        if t is not None:
            return t
        return super().lookup_tensor(index)
