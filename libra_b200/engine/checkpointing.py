"""Versioned checkpoints: Megatron-Core ``torch_dist`` layout + HF export.

Directory layout per version (reference ``engine/megatron_core_checkpointing.py``
and ``docs/megatron_core_backend.md:30-39``)::

    <sync_path>/v<N>/megatron_dist/         torch.distributed.checkpoint shards + .metadata
    <sync_path>/v<N>/model.safetensors      HF-format weights for rollout reload
    <sync_path>/v<N>/config.json            HF Qwen3 config of the model
    <sync_path>/v<N>/megatron_checkpoint_manifest.json
    <sync_path>/v<N>/sync_progress/rank_<R>.json

``megatron_dist`` holds Megatron-Core's model-space layout (``mcore_layout``):
one DCP tensor per parameter kind in its global shape, layers stacked on a
leading axis (``decoder.layers.self_attention.linear_qkv.weight`` is
``[layers, (q + 2 kv) * head_dim, hidden]`` with the rows per query group),
tensor-parallel and expert-parallel ranks writing their chunks at global
offsets, and the distributed optimizer's fp32 master weights and Adam moments
under ``optimizer.state.{fp32_param,exp_avg,exp_avg_sq}.<key>`` in the same
shapes.  A checkpoint written at one TP/PP/EP/DP layout loads at another: each
rank reads the chunks it needs.  Non-tensor state (iteration, optimizer step
and hyper-parameters) is in ``common.pt``; ``metadata.json`` names the
backends, as Megatron-Core's loader expects.

``to_mcore`` / ``from_mcore`` are the per-layer state-dict names of the same
tensors for one unsharded model (QKV in per-group order, fc1 ``[gate; up]``,
GroupedMLP expert-major ``weight1`` / ``weight2``).
"""

from __future__ import annotations

import json
import os
import time
from dataclasses import asdict, dataclass
from pathlib import Path
from typing import Any, Dict, Optional

import torch
import torch.distributed as dist

from libra_b200.engine.mcore_layout import (OPTIM_KINDS, ChunkLoadPlanner, ChunkSavePlanner, ShardInfo,
                                            model_space_items)
from libra_b200.models.qwen3 import Qwen3Config


@dataclass(frozen=True)
class MegatronCheckpointManifest:
    version: int
    checkpoint_format: str
    distributed_checkpoint: str
    rollout_export: str
    world_size: int
    tensor_parallel_size: int
    pipeline_parallel_size: int
    context_parallel_size: int
    expert_parallel_size: int
    data_parallel_size: int
    includes_optimizer: bool
    completed_at: float


# ----------------------------------------------------------------------------- key maps
def mcore_qkv_rows(cfg: Qwen3Config, nq: Optional[int] = None, nkv: Optional[int] = None) -> torch.Tensor:
    """Row index list taking [q | k | v] to Megatron's per-group [q.., k, v] order."""
    D = cfg.head_dim
    nq = nq or cfg.num_attention_heads
    nkv = nkv or cfg.num_key_value_heads
    per = nq // nkv
    rows = []
    for g in range(nkv):
        for j in range(per):
            rows.extend(range((g * per + j) * D, (g * per + j + 1) * D))
        rows.extend(range(nq * D + g * D, nq * D + (g + 1) * D))
        rows.extend(range((nq + nkv) * D + g * D, (nq + nkv) * D + (g + 1) * D))
    return torch.tensor(rows, dtype=torch.long)


MCORE_METADATA = {"sharded_backend": "torch_dist", "sharded_backend_version": 1,
                  "common_backend": "torch", "common_backend_version": 1}


def _shard_info(engine) -> ShardInfo:
    return ShardInfo(tp_size=int(getattr(engine, "tp_size", 1)), tp_rank=int(getattr(engine, "tp_rank", 0)),
                     ep_size=int(getattr(engine, "ep_size", 1)), ep_rank=int(getattr(engine, "ep_rank", 0)))


def _param_group(engine) -> Dict[str, Any]:
    o = engine.optim
    return {"step": int(engine.step_count), "lr": float(o.lr), "betas": tuple(o.betas), "eps": float(o.eps),
            "weight_decay": float(o.weight_decay), "max_grad_norm": float(o.max_grad_norm)}


_STATE_NAMES = {"fp32_param": "master", "exp_avg": "exp_avg", "exp_avg_sq": "exp_avg_sq"}
_EXPERT_NAMES = {"fp32_param": "x_master", "exp_avg": "x_m", "exp_avg_sq": "x_v"}


def _dense_params(engine):
    """(name, shape, start, end) in the flat buffer of the parameters that the
    distributed optimizer shards over the data-parallel group, by offset."""
    out = []
    for name, p in engine.params.items():
        a = engine.layout.offsets[name]
        if a < engine.dense_numel:
            out.append((name, tuple(p.shape), a, a + p.numel()))
    return sorted(out, key=lambda x: x[2])


def _expert_state(engine) -> Dict[str, Dict[str, torch.Tensor]]:
    """This rank's expert parameters' optimizer state (held whole by every rank
    with those experts), as parameter-shaped views."""
    out = {k: {} for k in OPTIM_KINDS}
    if getattr(engine, "x_master", None) is None:
        return out
    for name, p in engine.params.items():
        a = engine.layout.offsets[name]
        if a >= engine.dense_numel:
            for kind, attr in _EXPERT_NAMES.items():
                out[kind][name] = getattr(engine, attr)[a - engine.dense_numel:a - engine.dense_numel + p.numel()] \
                    .view(p.shape)
    return out


def _optimizer_state_for_save(engine) -> Dict[str, Dict[str, torch.Tensor]]:
    """kind -> {parameter name -> full local (TP/EP-shard) state tensor} for the
    parameters this rank writes.  A parameter inside one data-parallel shard is
    written by that shard's rank; one that straddles shards is assembled on the
    rank holding its first element from the pieces of the others (point-to-point
    over the data-parallel group; every rank walks the same list in order)."""
    state = engine.optimizer_state_tensors()
    out = _expert_state(engine)
    S, s0 = engine.shard_numel, engine.shard_start
    me = engine.get_data_parallel_rank()
    if not engine.sharded:
        if me == 0:
            for name, shape, a, b in _dense_params(engine):
                for kind, attr in _STATE_NAMES.items():
                    out[kind][name] = state[attr][a:b].view(shape)
        return out
    group = engine.dp_group
    xdev = engine.device if dist.get_backend(group) == "nccl" else torch.device("cpu")
    for name, shape, a, b in _dense_params(engine):
        r0, r1 = a // S, (b - 1) // S
        if r0 == r1:
            if me == r0:
                for kind, attr in _STATE_NAMES.items():
                    out[kind][name] = state[attr][a - s0:b - s0].view(shape)
            continue
        if me == r0:
            buf = torch.empty(3, b - a, dtype=torch.float32, device=xdev)
            for j, attr in enumerate(_STATE_NAMES.values()):
                buf[j, :(r0 + 1) * S - a].copy_(state[attr][a - s0:])
        for r in range(r0 + 1, r1 + 1):
            lo, hi = max(a, r * S), min(b, (r + 1) * S)
            if me == r:
                piece = torch.stack([state[attr][lo - s0:hi - s0].float().to(xdev) for attr in _STATE_NAMES.values()])
                dist.send(piece, group=group, group_dst=r0)
            elif me == r0:
                piece = torch.empty(3, hi - lo, dtype=torch.float32, device=xdev)
                dist.recv(piece, group=group, group_src=r)
                buf[:, lo - a:hi - a].copy_(piece)
        if me == r0:
            for j, (kind, attr) in enumerate(_STATE_NAMES.items()):
                out[kind][name] = buf[j].to(state[attr].dtype).view(shape)
    return out


class _OptimizerLoad:
    """Load targets for the optimizer state: parameter-shaped views into this
    rank's shard for parameters inside it, temporaries for parameters that
    straddle its edges (their overlap is copied in by ``finish``)."""

    def __init__(self, engine):
        self.engine = engine
        self.state = engine.optimizer_state_tensors()
        self.targets = _expert_state(engine)
        self.partial = []
        S, s0 = engine.shard_numel, engine.shard_start
        for name, shape, a, b in _dense_params(engine):
            lo, hi = max(a, s0), min(b, s0 + S)
            if lo >= hi:
                continue
            for kind, attr in _STATE_NAMES.items():
                src = self.state[attr]
                if lo == a and hi == b:
                    self.targets[kind][name] = src[a - s0:b - s0].view(shape)
                else:
                    t = torch.zeros(shape, dtype=src.dtype, device=src.device)
                    self.targets[kind][name] = t
                    self.partial.append((attr, t, lo - a, hi - a, lo - s0))

    def finish(self) -> None:
        for attr, t, x0, x1, d0 in self.partial:
            self.state[attr][d0:d0 + x1 - x0].copy_(t.reshape(-1)[x0:x1])
        if getattr(self.engine, "_offload_k", 0):
            self.engine.load_optimizer_state_tensors(self.state)


def to_mcore(params: Dict[str, torch.Tensor], cfg: Qwen3Config) -> Dict[str, torch.Tensor]:
    """MCore names for the parameters present (a pipeline stage holds a subset: its
    layers keep their global indices, as in MCore's pipeline-parallel checkpoints)."""
    perm = mcore_qkv_rows(cfg)
    out: Dict[str, torch.Tensor] = {}
    if "embed_tokens" in params:
        out["embedding.word_embeddings.weight"] = params["embed_tokens"]
    for i in range(cfg.num_hidden_layers):
        p, m = f"layers.{i}.", f"decoder.layers.{i}."
        if p + "input_layernorm" not in params:
            continue
        out[m + "input_layernorm.weight"] = params[p + "input_layernorm"]
        out[m + "self_attention.linear_qkv.weight"] = params[p + "qkv_proj"].index_select(0, perm.to(params[p + "qkv_proj"].device))
        out[m + "self_attention.q_layernorm.weight"] = params[p + "q_norm"]
        out[m + "self_attention.k_layernorm.weight"] = params[p + "k_norm"]
        out[m + "self_attention.linear_proj.weight"] = params[p + "o_proj"]
        out[m + "pre_mlp_layernorm.weight"] = params[p + "post_attention_layernorm"]
        if cfg.is_moe:
            E, H = cfg.num_experts, cfg.hidden_size
            out[m + "mlp.router.weight"] = params[p + "router"]
            # GroupedMLP: weight1 [H, E*2F] (expert-major), weight2 [E*F, H]
            out[m + "mlp.experts.weight1"] = params[p + "experts.w1"].permute(2, 0, 1).reshape(H, -1)
            out[m + "mlp.experts.weight2"] = params[p + "experts.w2"].permute(0, 2, 1).reshape(-1, H)
        else:
            out[m + "mlp.linear_fc1.weight"] = params[p + "gate_up_proj"]
            out[m + "mlp.linear_fc2.weight"] = params[p + "down_proj"]
    if "norm" in params:
        out["decoder.final_layernorm.weight"] = params["norm"]
    if not cfg.tie_word_embeddings and "lm_head" in params:
        out["output_layer.weight"] = params["lm_head"]
    return out


def from_mcore(sd: Dict[str, torch.Tensor], params: Dict[str, torch.Tensor], cfg: Qwen3Config) -> None:
    inv = torch.argsort(mcore_qkv_rows(cfg))
    with torch.no_grad():
        if "embed_tokens" in params:
            params["embed_tokens"].copy_(sd["embedding.word_embeddings.weight"])
        for i in range(cfg.num_hidden_layers):
            p, m = f"layers.{i}.", f"decoder.layers.{i}."
            if p + "input_layernorm" not in params:
                continue
            params[p + "input_layernorm"].copy_(sd[m + "input_layernorm.weight"])
            qkv = sd[m + "self_attention.linear_qkv.weight"]
            params[p + "qkv_proj"].copy_(qkv.index_select(0, inv.to(qkv.device)))
            params[p + "q_norm"].copy_(sd[m + "self_attention.q_layernorm.weight"])
            params[p + "k_norm"].copy_(sd[m + "self_attention.k_layernorm.weight"])
            params[p + "o_proj"].copy_(sd[m + "self_attention.linear_proj.weight"])
            params[p + "post_attention_layernorm"].copy_(sd[m + "pre_mlp_layernorm.weight"])
            if cfg.is_moe:
                E, H = cfg.num_experts, cfg.hidden_size
                params[p + "router"].copy_(sd[m + "mlp.router.weight"])
                params[p + "experts.w1"].copy_(sd[m + "mlp.experts.weight1"].reshape(H, E, -1).permute(1, 2, 0))
                params[p + "experts.w2"].copy_(sd[m + "mlp.experts.weight2"].reshape(E, -1, H).permute(0, 2, 1))
            else:
                params[p + "gate_up_proj"].copy_(sd[m + "mlp.linear_fc1.weight"])
                params[p + "down_proj"].copy_(sd[m + "mlp.linear_fc2.weight"])
        if "norm" in params:
            params["norm"].copy_(sd["decoder.final_layernorm.weight"])
        if not cfg.tie_word_embeddings and "lm_head" in params:
            params["lm_head"].copy_(sd["output_layer.weight"])


def to_hf(params: Dict[str, torch.Tensor], cfg: Qwen3Config) -> Dict[str, torch.Tensor]:
    """HF Qwen3 / Qwen3-MoE parameter names (split QKV and gate/up)."""
    D, nq, nkv = cfg.head_dim, cfg.num_attention_heads, cfg.num_key_value_heads
    out = {"model.embed_tokens.weight": params["embed_tokens"], "model.norm.weight": params["norm"]}
    for i in range(cfg.num_hidden_layers):
        p, h = f"layers.{i}.", f"model.layers.{i}."
        qkv = params[p + "qkv_proj"]
        out[h + "self_attn.q_proj.weight"] = qkv[: nq * D]
        out[h + "self_attn.k_proj.weight"] = qkv[nq * D:(nq + nkv) * D]
        out[h + "self_attn.v_proj.weight"] = qkv[(nq + nkv) * D:]
        out[h + "self_attn.q_norm.weight"] = params[p + "q_norm"]
        out[h + "self_attn.k_norm.weight"] = params[p + "k_norm"]
        out[h + "self_attn.o_proj.weight"] = params[p + "o_proj"]
        out[h + "input_layernorm.weight"] = params[p + "input_layernorm"]
        out[h + "post_attention_layernorm.weight"] = params[p + "post_attention_layernorm"]
        if cfg.is_moe:
            out[h + "mlp.gate.weight"] = params[p + "router"]
            Fe = cfg.moe_intermediate_size
            for e in range(cfg.num_experts):
                w1 = params[p + "experts.w1"][e]
                out[h + f"mlp.experts.{e}.gate_proj.weight"] = w1[:Fe]
                out[h + f"mlp.experts.{e}.up_proj.weight"] = w1[Fe:]
                out[h + f"mlp.experts.{e}.down_proj.weight"] = params[p + "experts.w2"][e]
        else:
            gu = params[p + "gate_up_proj"]
            F = gu.shape[0] // 2
            out[h + "mlp.gate_proj.weight"] = gu[:F]
            out[h + "mlp.up_proj.weight"] = gu[F:]
            out[h + "mlp.down_proj.weight"] = params[p + "down_proj"]
    if not cfg.tie_word_embeddings:
        out["lm_head.weight"] = params["lm_head"]
    return out


def from_hf(sd: Dict[str, torch.Tensor], params: Dict[str, torch.Tensor], cfg: Qwen3Config) -> None:
    with torch.no_grad():
        params["embed_tokens"].copy_(sd["model.embed_tokens.weight"])
        params["norm"].copy_(sd["model.norm.weight"])
        for i in range(cfg.num_hidden_layers):
            p, h = f"layers.{i}.", f"model.layers.{i}."
            params[p + "qkv_proj"].copy_(torch.cat([sd[h + "self_attn.q_proj.weight"], sd[h + "self_attn.k_proj.weight"],
                                                    sd[h + "self_attn.v_proj.weight"]]))
            params[p + "q_norm"].copy_(sd[h + "self_attn.q_norm.weight"])
            params[p + "k_norm"].copy_(sd[h + "self_attn.k_norm.weight"])
            params[p + "o_proj"].copy_(sd[h + "self_attn.o_proj.weight"])
            params[p + "input_layernorm"].copy_(sd[h + "input_layernorm.weight"])
            params[p + "post_attention_layernorm"].copy_(sd[h + "post_attention_layernorm.weight"])
            if cfg.is_moe:
                params[p + "router"].copy_(sd[h + "mlp.gate.weight"])
                for e in range(cfg.num_experts):
                    params[p + "experts.w1"][e].copy_(torch.cat([sd[h + f"mlp.experts.{e}.gate_proj.weight"],
                                                                 sd[h + f"mlp.experts.{e}.up_proj.weight"]]))
                    params[p + "experts.w2"][e].copy_(sd[h + f"mlp.experts.{e}.down_proj.weight"])
            else:
                params[p + "gate_up_proj"].copy_(torch.cat([sd[h + "mlp.gate_proj.weight"], sd[h + "mlp.up_proj.weight"]]))
                params[p + "down_proj"].copy_(sd[h + "mlp.down_proj.weight"])
        if not cfg.tie_word_embeddings:
            params["lm_head"].copy_(sd["lm_head.weight"])


def hf_config_dict(cfg: Qwen3Config) -> Dict[str, Any]:
    d = {"architectures": ["Qwen3MoeForCausalLM" if cfg.is_moe else "Qwen3ForCausalLM"],
         "model_type": "qwen3_moe" if cfg.is_moe else "qwen3", "vocab_size": cfg.vocab_size,
         "hidden_size": cfg.hidden_size, "intermediate_size": cfg.intermediate_size,
         "num_hidden_layers": cfg.num_hidden_layers, "num_attention_heads": cfg.num_attention_heads,
         "num_key_value_heads": cfg.num_key_value_heads, "head_dim": cfg.head_dim, "rope_theta": cfg.rope_theta,
         "rms_norm_eps": cfg.rms_norm_eps, "tie_word_embeddings": cfg.tie_word_embeddings,
         "max_position_embeddings": cfg.max_position_embeddings, "torch_dtype": "bfloat16", "hidden_act": "silu"}
    if cfg.is_moe:
        d.update({"num_experts": cfg.num_experts, "num_experts_per_tok": cfg.num_experts_per_tok,
                  "moe_intermediate_size": cfg.moe_intermediate_size, "norm_topk_prob": cfg.norm_topk_prob})
    return d


# ----------------------------------------------------------------------------- manager
def _rank() -> int:
    return dist.get_rank() if dist.is_available() and dist.is_initialized() else 0


def _world() -> int:
    return dist.get_world_size() if dist.is_available() and dist.is_initialized() else 1


def _barrier() -> None:
    if _world() > 1:
        dist.barrier()


def _write_json(path: Path, obj: Any) -> None:
    path.parent.mkdir(parents=True, exist_ok=True)
    tmp = path.with_name(f".{path.name}.{os.getpid()}.tmp")
    tmp.write_text(json.dumps(obj, indent=2, default=str), encoding="utf-8")
    os.replace(tmp, path)


class DistributedCheckpointManager:
    def __init__(self, sync_path: str, checkpoint_format: str = "torch_dist", fully_parallel_save: bool = True,
                 async_save: bool = False):
        if checkpoint_format != "torch_dist":
            raise ValueError("Only torch_dist checkpoints are supported")
        self.sync_path = Path(sync_path)
        self.checkpoint_format = checkpoint_format
        self.fully_parallel_save = fully_parallel_save
        self.async_save = async_save

    def _progress(self, vdir: Path, version: int, phase: str) -> None:
        _write_json(vdir / "sync_progress" / f"rank_{_rank()}.json",
                    {"rank": _rank(), "version": version, "phase": phase, "timestamp": time.time()})

    def save(self, engine, version: int, export_for_rollout: bool = True, include_optimizer: bool = True,
             export_only: Optional[bool] = None) -> Path:
        import torch.distributed.checkpoint as dcp

        if export_only is None:
            export_only = os.environ.get("MEGATRON_ROLLOUT_EXPORT_ONLY", "0") == "1"
        vdir = self.sync_path / f"v{version}"
        ddir = vdir / "megatron_dist"
        if _rank() == 0:
            (ddir if not export_only else vdir).mkdir(parents=True, exist_ok=True)
        _barrier()
        cfg = engine.cfg
        params = {k: v.detach() for k, v in engine.params.items()}
        if export_only:
            self._progress(vdir, version, "dist_checkpoint_skipped")
        else:
            self._progress(vdir, version, "before_sharded_state_dict")
            info = _shard_info(engine)
            chunks = model_space_items(params, cfg, info)
            with_optim = include_optimizer and getattr(engine, "master", None) is not None
            if with_optim:
                for kind, tensors in _optimizer_state_for_save(engine).items():
                    chunks.update(model_space_items(tensors, cfg, info, prefix=f"optimizer.state.{kind}."))
            self._progress(vdir, version, "before_dist_checkpoint_save")
            dcp.save({}, checkpoint_id=str(ddir), planner=ChunkSavePlanner(chunks))
            if _rank() == 0:
                common = {"checkpoint_version": 3.0, "iteration": int(version)}
                if with_optim:
                    common["optimizer"] = {"param_groups": [_param_group(engine)]}
                torch.save(common, ddir / "common.pt")
                _write_json(ddir / "metadata.json", MCORE_METADATA)
            _barrier()
            self._progress(vdir, version, "after_dist_checkpoint_save")
        if export_for_rollout and hasattr(engine, "export_params"):
            params = engine.export_params()  # pipeline stages: the full set on rank 0 (collective)
        if export_for_rollout and _rank() == 0:
            from safetensors.torch import save_file

            self._progress(vdir, version, "before_streaming_hf_export")
            hf = {k: v.contiguous().cpu() for k, v in to_hf(params, cfg).items()}
            save_file(hf, str(vdir / "model.safetensors"), metadata={"format": "pt", "version": str(version)})
            _write_json(vdir / "config.json", hf_config_dict(cfg))
            self._progress(vdir, version, "after_streaming_hf_export")
        _barrier()
        if _rank() == 0:
            man = MegatronCheckpointManifest(
                version=int(version), checkpoint_format=self.checkpoint_format,
                distributed_checkpoint="" if export_only else str(ddir),
                rollout_export=str(vdir) if export_for_rollout else "", world_size=_world(),
                tensor_parallel_size=int(getattr(engine, "tp_size", 1)),
                pipeline_parallel_size=int(getattr(engine, "pp_size", 1)),
                context_parallel_size=1, expert_parallel_size=int(getattr(engine, "ep_size", 1)),
                data_parallel_size=int(engine.get_data_parallel_world_size()),
                includes_optimizer=bool(include_optimizer and not export_only), completed_at=time.time())
            _write_json(vdir / "megatron_checkpoint_manifest.json", asdict(man))
        _barrier()
        self._progress(vdir, version, "complete")
        return vdir

    def load(self, engine, version: Optional[int] = None, load_optimizer: bool = True) -> int:
        import torch.distributed.checkpoint as dcp

        if version is None:
            version = latest_version(self.sync_path)
            if version is None:
                raise FileNotFoundError(f"no checkpoint under {self.sync_path}")
        vdir = self.sync_path / f"v{version}"
        if not (vdir / "megatron_checkpoint_manifest.json").exists():
            raise FileNotFoundError(f"Incomplete checkpoint: {vdir / 'megatron_checkpoint_manifest.json'} does not exist")
        cfg = engine.cfg
        ddir = vdir / "megatron_dist"
        info = _shard_info(engine)
        params = {k: v.detach() for k, v in engine.params.items()}
        chunks = model_space_items(params, cfg, info)
        common = torch.load(ddir / "common.pt", weights_only=True) if (ddir / "common.pt").exists() else {}
        optim = None
        if load_optimizer and getattr(engine, "master", None) is not None and "optimizer" in common:
            optim = _OptimizerLoad(engine)
            for kind, tensors in optim.targets.items():
                chunks.update(model_space_items(tensors, cfg, info, prefix=f"optimizer.state.{kind}."))
        with torch.no_grad():
            dcp.load({}, checkpoint_id=str(ddir), planner=ChunkLoadPlanner(chunks))
            if optim is not None:
                optim.finish()
                engine.step_count = int(common["optimizer"]["param_groups"][0]["step"])
        engine.set_version(int(version))
        _barrier()
        return int(version)

    def prune(self, keep_latest: int, protect: Optional[int] = None) -> None:
        """Delete all but the newest ``keep_latest`` versions (never ``protect``)."""
        import shutil

        if _rank() != 0 or keep_latest <= 0:
            return
        versions = sorted(all_versions(self.sync_path))
        for v in versions[:-keep_latest]:
            if v != protect:
                shutil.rmtree(self.sync_path / f"v{v}", ignore_errors=True)


def all_versions(root) -> list:
    root = Path(root)
    if not root.exists():
        return []
    out = []
    for p in root.iterdir():
        if p.is_dir() and p.name.startswith("v") and p.name[1:].isdigit() and (p / "megatron_checkpoint_manifest.json").exists():
            out.append(int(p.name[1:]))
    return out


def latest_version(root) -> Optional[int]:
    vs = all_versions(root)
    return max(vs) if vs else None


def load_params_into(params: Dict[str, torch.Tensor], path: str, cfg: Optional[Qwen3Config] = None) -> None:
    """Load HF safetensors (a version dir or file) into parameter views."""
    from safetensors.torch import load_file

    p = Path(path)
    f = p / "model.safetensors" if p.is_dir() else p
    sd = load_file(str(f), device=str(next(iter(params.values())).device))
    if cfg is None:
        cfg_path = f.parent / "config.json"
        d = json.loads(cfg_path.read_text())
        cfg = Qwen3Config(vocab_size=d["vocab_size"], hidden_size=d["hidden_size"],
                          intermediate_size=d["intermediate_size"], num_hidden_layers=d["num_hidden_layers"],
                          num_attention_heads=d["num_attention_heads"], num_key_value_heads=d["num_key_value_heads"],
                          head_dim=d.get("head_dim", d["hidden_size"] // d["num_attention_heads"]),
                          tie_word_embeddings=d.get("tie_word_embeddings", False),
                          num_experts=d.get("num_experts", 0) if "moe" in d.get("model_type", "") else 0,
                          num_experts_per_tok=d.get("num_experts_per_tok", 8),
                          moe_intermediate_size=d.get("moe_intermediate_size", 768))
    from_hf(sd, params, cfg)
