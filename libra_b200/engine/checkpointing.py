"""Versioned checkpoints: Megatron-Core ``torch_dist`` layout + HF export.

Directory layout per version (reference ``engine/megatron_core_checkpointing.py``
and ``docs/megatron_core_backend.md:30-39``)::

    <sync_path>/v<N>/megatron_dist/         torch.distributed.checkpoint shards + .metadata
    <sync_path>/v<N>/model.safetensors      HF-format weights for rollout reload
    <sync_path>/v<N>/config.json            HF Qwen3 config of the model
    <sync_path>/v<N>/megatron_checkpoint_manifest.json
    <sync_path>/v<N>/sync_progress/rank_<R>.json

The sharded state dict uses Megatron-Core GPT key names
(``decoder.layers.{i}.self_attention.linear_qkv.weight`` ...), with the QKV
rows in Megatron's per-query-group order ``[group][q heads of group, k, v]``
(this engine keeps them as ``[all q | all k | all v]``; ``mcore_qkv_rows``
is the row permutation).  fc1 is ``[gate; up]`` in both.  Optimizer state is
the distributed-optimizer layout: every DP rank saves its flat fp32 shard of
master weights and Adam moments (``optimizer.shard_<r>.*``) plus the step.
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


def _optim_prefix(engine, dp_rank: int) -> str:
    """Key prefix of one data-parallel shard of the optimizer state; tensor-
    parallel ranks and pipeline stages hold different parameters, so each has
    its own shards."""
    pre = "optimizer."
    if int(getattr(engine, "tp_size", 1)) > 1:
        pre += f"tp{int(engine.tp_rank)}."
    if int(getattr(engine, "pp_size", 1)) > 1:
        pre += f"pp{int(engine.pp_rank)}."
    return f"{pre}shard_{dp_rank}"


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
            sd: Dict[str, Any] = {"checkpoint_version": 3.0, "iteration": int(version)}
            sd.update({f"model.{k}": v for k, v in to_mcore(params, cfg).items()})
            if include_optimizer and getattr(engine, "master", None) is not None:
                r = engine.get_data_parallel_rank() if engine.sharded else 0
                if engine.sharded or engine.get_data_parallel_rank() == 0:
                    state = engine.optimizer_state_tensors() if hasattr(engine, "optimizer_state_tensors") else \
                        {"master": engine.master, "exp_avg": engine.exp_avg, "exp_avg_sq": engine.exp_avg_sq}
                    for n, t in state.items():
                        sd[f"{_optim_prefix(engine, r)}.{n}"] = t
                sd["optimizer.step"] = torch.tensor(engine.step_count)
            self._progress(vdir, version, "before_dist_checkpoint_save")
            dcp.save(sd, checkpoint_id=str(ddir))
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
                tensor_parallel_size=int(getattr(engine, "tp_size", 1)), pipeline_parallel_size=1,
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
        params = {k: v.detach() for k, v in engine.params.items()}
        tmpl: Dict[str, Any] = {f"model.{k}": v.clone() for k, v in to_mcore(params, cfg).items()}
        if load_optimizer and getattr(engine, "master", None) is not None:
            r = engine.get_data_parallel_rank() if engine.sharded else 0
            split = bool(getattr(engine, "_offload_k", 0))
            state = engine.optimizer_state_tensors() if split else \
                {"master": engine.master, "exp_avg": engine.exp_avg, "exp_avg_sq": engine.exp_avg_sq}
            for n, t in state.items():
                tmpl[f"{_optim_prefix(engine, r)}.{n}"] = t
            tmpl["optimizer.step"] = torch.tensor(0)
        dcp.load(tmpl, checkpoint_id=str(vdir / "megatron_dist"))
        if load_optimizer and getattr(engine, "_offload_k", 0):
            r = engine.get_data_parallel_rank() if engine.sharded else 0
            engine.load_optimizer_state_tensors({n: tmpl[f"{_optim_prefix(engine, r)}.{n}"]
                                                 for n in ("master", "exp_avg", "exp_avg_sq")})
        from_mcore({k[len("model."):]: v for k, v in tmpl.items() if k.startswith("model.")}, params, cfg)
        if "optimizer.step" in tmpl:
            engine.step_count = int(tmpl["optimizer.step"])
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
