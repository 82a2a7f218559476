"""Training engine protocol and the native B200 training engine.

``TrainEngine`` is the protocol the trainer talks to (reference
``engine/train_engine.py:90-171``).  ``B200TrainEngine`` replaces the
reference's three backends (FSDP, Megatron3D, Megatron-Core) with one engine:

* parameters: one flat bf16 buffer; ``nn.Parameter`` objects alias slices of it.
* gradients: one flat fp32 buffer, filled by the GEMM epilogues through the
  ``main_grad`` views (Megatron-Core's gradient-accumulation fusion).
* optimizer: AdamW (betas 0.9/0.95, eps 1e-8, wd 0.01, clip 1.0 — reference
  ``engine/megatron_core_train_engine.py:228-261``) over a flat fp32 master copy.
  With ``use_distributed_optimizer`` and DP > 1 each rank owns a 1/DP shard of
  master/Adam state; gradients are reduce-scattered and the updated bf16 shard
  is all-gathered (distributed optimizer of Megatron-Core).
* GRPO loss: PPO-clip with the log-ratio clamped to [-20, 20] and the k3 KL
  ``(r - 1) - log r`` (reference ``engine/megatron_core_train_engine.py:950-986``),
  aggregated exactly as the reference does: masked token mean inside each
  group of ``micro_batch_size`` consecutive trajectories, averaged over the
  groups.  That aggregation is expressed as one weight per action token, so it
  does not depend on how the work is chunked for execution.
* execution chunks: consecutive trajectories packed into one token stream (no
  padding) up to ``max_tokens_per_micro_batch`` tokens, which bounds activation
  memory independently of the trajectory lengths.
"""

from __future__ import annotations

import math
import os
import time
from dataclasses import dataclass
from typing import Any, Dict, Iterable, List, Optional, Protocol

import torch
import torch.distributed as dist

from libra_b200 import ops
from libra_b200.models.qwen3 import (PackedBatch, ParamLayout, Qwen3Config, Qwen3Model, get_config, init_params,
                                     is_expert_param, pack_sequences, param_shapes)
from libra_b200.utils import nvtx


class TrainEngine(Protocol):
    """What the async trainer needs from a training backend."""

    def initialize(self, max_seq_length: int = 2048) -> None: ...
    def get_version(self) -> int: ...
    def set_version(self, version: int) -> None: ...
    def grpo_update(self, trajectories: List[Dict[str, Any]], ppo_epochs: int = 1) -> Dict[str, float]: ...
    def recompute_logprobs(self, trajectories: List[Dict[str, Any]]) -> None: ...
    def save_weights(self, path: str, version: int) -> None: ...
    def get_data_parallel_rank(self) -> int: ...
    def get_data_parallel_world_size(self) -> int: ...
    def is_batch_source(self) -> bool: ...
    def get_local_batch_size(self, global_batch_size: int) -> int: ...
    def distribute_trajectories(self, trajectories): ...
    def align_distributed_trajectories(self, trajectories): ...


@dataclass
class OptimConfig:
    lr: float = 1e-6
    betas: tuple = (0.9, 0.95)
    eps: float = 1e-8
    weight_decay: float = 0.01
    max_grad_norm: float = 1.0


class B200TrainEngine:
    """Native GRPO training engine (single process per GPU)."""

    train_backend = "b200"
    _peer_grad = None      # PeerGradReduce when the DP exchange runs over peer memory
    _offload_k = 0         # elements of the dense optimizer shard stepped on the host
    _sq_ready = False      # the reduce left the global squared gradient norm in sq_norm

    def __init__(self, model: Any = "qwen3-4b", learning_rate: float = 1e-6, kl_coef: float = 0.001,
                 clip_epsilon: float = 0.2, micro_batch_size: int = 4, recompute_micro_batch_size: int = 0,
                 device: Optional[torch.device] = None, seed: int = 0, recompute_activations: bool = False,
                 use_distributed_optimizer: bool = True, dp_group=None, temperature: float = 1.0,
                 max_grad_norm: float = 1.0, tp_size: int = 1, model_path: str = "",
                 max_tokens_per_micro_batch: int = 16384, max_tokens_per_recompute_batch: int = 65536,
                 ep_size: int = 1, sequence_parallel: bool = False, precision_aware_optimizer: bool = False,
                 optimizer_cpu_offload: bool = False, optimizer_offload_fraction: float = 0.0, pp_size: int = 1):
        self.cfg: Qwen3Config = get_config(model)
        self.model_path = model_path
        self.optim = OptimConfig(lr=learning_rate, max_grad_norm=max_grad_norm)
        self.kl_coef = kl_coef
        self.clip_epsilon = clip_epsilon
        self.micro_batch_size = max(1, int(micro_batch_size))
        self.recompute_micro_batch_size = int(recompute_micro_batch_size) or self.micro_batch_size
        self.max_tokens_per_micro_batch = int(max_tokens_per_micro_batch)
        self.max_tokens_per_recompute_batch = int(max_tokens_per_recompute_batch)
        self.seed = seed
        self.recompute_activations = recompute_activations
        self.use_distributed_optimizer = use_distributed_optimizer
        self.temperature = temperature
        self.tp_size = tp_size
        # pipeline parallelism: this rank holds a contiguous range of layers (1F1B over NCCL p2p)
        self.pp_size = max(1, int(pp_size))
        self.sequence_parallel = bool(sequence_parallel) and tp_size > 1
        # precision-aware optimizer (MCore use_precision_aware_optimizer): Adam moments stored in bf16
        # (updated in fp32 inside the kernel), fp32 master weights; 8 instead of 12 bytes per parameter
        self.precision_aware_optimizer = bool(precision_aware_optimizer)
        # optimizer CPU offload: this fraction of the dense optimizer shard keeps its master weights and
        # moments in host memory (pinned on GPU engines) and is stepped on the CPU
        frac = float(optimizer_offload_fraction) if optimizer_cpu_offload else 0.0
        if not 0.0 <= frac <= 1.0:
            raise ValueError("optimizer_offload_fraction must lie in [0, 1]")
        self.optimizer_offload_fraction = frac
        self.ep_size = max(1, int(ep_size))
        if self.ep_size > 1 and not self.cfg.is_moe:
            raise ValueError(f"ep_size={self.ep_size} needs a mixture-of-experts model")
        self.current_version = 0
        self.step_count = 0
        self.dp_group = dp_group
        self.rank = int(os.environ.get("RANK", "0"))
        self.world_size = int(os.environ.get("WORLD_SIZE", "1"))
        if device is None:
            if torch.cuda.is_available():
                device = torch.device("cuda", int(os.environ.get("LOCAL_RANK", "0")))
            else:
                device = torch.device("cpu")
        self.device = torch.device(device)
        if self.device.type == "cuda" and self.device.index is None:
            self.device = torch.device("cuda", torch.cuda.current_device())
        self.model: Optional[Qwen3Model] = None
        self.last_timing: Dict[str, float] = {}
        self.io_bytes = {"h2d": 0, "d2h": 0}  # host<->device traffic of the public API calls
        self.elastic_gradient_domain = None
        self._pending_hybrid_gradients: List[Any] = []
        self.elastic_update_publisher = None  # callable(reduced flat grad, step, version) for lockstep hybrids
        self.elastic_payload_wait_s = 0.0  # >0: wait this long for every active hybrid replica's payload
        # True when the hybrid replicas trained their own shares of this replica's batch: the merged
        # gradient is then the mean over the core and the hybrids (each already a mean over its share)
        self.elastic_average_merged = False

    # ------------------------------------------------------------------ setup
    def initialize(self, max_seq_length: int = 2048) -> None:
        if self.device.type == "cuda":
            torch.cuda.set_device(self.device)
            ops.ext()  # fail loudly when the kernels are not built
        self.max_seq_length = max_seq_length
        self.tp_group, self.tp_rank, self.mesh = None, 0, None
        self._init_pipeline()
        if self.tp_size > 1:
            # TP groups are consecutive ranks (inside the box); DP runs across them
            from libra_b200.parallel.mesh import ParallelMesh

            if not dist.is_initialized():
                raise RuntimeError("tensor parallelism needs an initialized process group")
            self.mesh = ParallelMesh(dist.get_world_size(), tp=self.tp_size)
            rank = dist.get_rank()
            self.tp_group = self.mesh.group("tp", rank)
            self.tp_rank = self.mesh.coords(rank).tp
            if self.dp_group is None:
                self.dp_group = self.mesh.group("dp", rank)
        self.dp_size = dist.get_world_size(self.dp_group) if dist.is_initialized() else 1
        self.dp_rank = dist.get_rank(self.dp_group) if dist.is_initialized() else 0
        self._init_expert_parallel()
        shapes = param_shapes(self.cfg, self.tp_size, self.tp_rank, self.ep_size)
        if self.pp_size > 1:
            shapes = [(n, sh) for n, sh in shapes if self._stage_owns(n)]
        unit = ParamLayout.ALIGN * self.dp_size
        if self.ep_size > 1:
            # dense parameters first (sharded over the data-parallel group by the distributed optimizer),
            # then this rank's experts (owned whole, reduced over the ranks that hold the same experts)
            dense = [(n, sh) for n, sh in shapes if not is_expert_param(n)]
            experts = [(n, sh) for n, sh in shapes if is_expert_param(n)]
            self.layout = ParamLayout(dense + experts)
            d_end = self.layout.offsets[experts[0][0]]
            self.dense_numel = (d_end + unit - 1) // unit * unit
            self.layout.shift([n for n, _ in experts], self.dense_numel - d_end)
            self.padded_numel = self.layout.numel
        else:
            self.layout = ParamLayout(shapes)
            # pad so the flat buffer splits evenly into DP shards of 128-element multiples
            self.padded_numel = (self.layout.numel + unit - 1) // unit * unit
            self.dense_numel = self.padded_numel
        dev = self.device
        self.flat_param = torch.zeros(self.padded_numel, dtype=torch.bfloat16, device=dev)
        self.flat_grad = torch.zeros(self.padded_numel, dtype=torch.float32, device=dev)
        views = self.layout.views(self.flat_param)
        E_l = self.cfg.num_experts // self.ep_size if self.cfg.is_moe else 0
        if self.pp_size > 1:
            # every stage takes its slice of the full model's initialisation (identical to one rank's)
            full_layout = ParamLayout(param_shapes(self.cfg))
            full = full_layout.views(torch.empty(full_layout.numel, dtype=torch.bfloat16, device=dev))
            init_params(self.cfg, full, seed=self.seed)
            with torch.no_grad():
                for name, v in views.items():
                    v.copy_(full[name])
            del full
        else:
            init_params(self.cfg, views, seed=self.seed + 7919 * self.tp_rank, expert_offset=self.ep_rank * E_l)
        grad_views = self.layout.views(self.flat_grad)
        self.params: Dict[str, torch.nn.Parameter] = {}
        for name, v in views.items():
            p = torch.nn.Parameter(v, requires_grad=True)
            p.main_grad = grad_views[name]
            # Ops without a fused main_grad path (the CPU reference ops) leave an
            # ordinary .grad; fold it into the flat fp32 buffer as it arrives.
            p.register_post_accumulate_grad_hook(_fold_grad_into_main)
            self.params[name] = p
        self.sharded = self.use_distributed_optimizer and self.dp_size > 1
        shard = self.dense_numel // self.dp_size if self.sharded else self.dense_numel
        self.shard_numel = shard
        self.shard_start = self.dp_rank * shard if self.sharded else 0
        mdt = torch.bfloat16 if self.precision_aware_optimizer else torch.float32
        # offloaded prefix [0, k) of the shard lives on the host; the device keeps [k, shard)
        k = int(shard * self.optimizer_offload_fraction) // 4 * 4
        self._offload_k = k
        src = self.flat_param[self.shard_start:self.shard_start + shard]
        self.master = src[k:].float().clone()
        self.exp_avg = torch.zeros(self.master.shape, dtype=mdt, device=dev)
        self.exp_avg_sq = torch.zeros(self.master.shape, dtype=mdt, device=dev)
        self._host_opt = None
        if k:
            pin = dict(pin_memory=dev.type == "cuda")
            host_master = src[:k].float().cpu()
            self._host_opt = {"master": host_master.pin_memory() if dev.type == "cuda" else host_master.clone(),
                              "exp_avg": torch.zeros(k, dtype=mdt, **pin), "exp_avg_sq": torch.zeros(k, dtype=mdt, **pin),
                              "grad": torch.zeros(k, dtype=torch.float32, **pin),
                              "param": torch.zeros(k, dtype=torch.bfloat16, **pin)}
        self.grad_shard = (torch.zeros(shard, dtype=torch.float32, device=dev) if self.sharded
                           else self.flat_grad[:self.dense_numel])
        self.sq_norm = torch.zeros(1, dtype=torch.float32, device=dev)
        # expert segment: fp32 master and Adam moments of this rank's experts (not sharded further)
        self.x_master = self.x_m = self.x_v = None
        if self.padded_numel > self.dense_numel:
            self.x_master = self.flat_param[self.dense_numel:].float().clone()
            self.x_m = torch.zeros_like(self.x_master)
            self.x_v = torch.zeros_like(self.x_master)
        self.ep_exchange = None
        if self.ep_size > 1 and dev.type == "cuda" and not self._gloo():
            from libra_b200.parallel.expert_parallel import PeerExpertExchange

            tokens = max(self.max_tokens_per_micro_batch, self.max_tokens_per_recompute_batch)
            k = self.cfg.num_experts_per_tok
            # receive capacity: twice a balanced share of the tokens' assignments plus the group padding;
            # a layer that would receive more rows is refused by the dispatch kernel (error word)
            rows = 2 * tokens * k + 128 * (self.cfg.num_experts // self.ep_size + 1)
            self.ep_exchange = PeerExpertExchange(self.ep_group, rows, self.cfg.hidden_size, dev)
        self.model = Qwen3Model(self.cfg, self.params, recompute=self.recompute_activations, tp_group=self.tp_group,
                                tp_size=self.tp_size, tp_rank=self.tp_rank, ep_group=self.ep_group,
                                ep_size=self.ep_size, ep_exchange=self.ep_exchange,
                                sequence_parallel=self.sequence_parallel)
        self.sequence_parallel = self.model.sp  # off for mixture-of-experts layers
        if self.pp_size > 1:
            from libra_b200.parallel.pipeline import P2P

            self._p2p = P2P(None, self.pp_prev, self.pp_next, dtype=torch.bfloat16, device=dev)
            # the last stage counts the tied embedding once in the global gradient norm
            self._pp_dup = []
            if self.pp_rank == self.pp_size - 1 and self.cfg.tie_word_embeddings and "embed_tokens" in self.params:
                a, b = self.layout.segment("embed_tokens")
                lo, hi = self.shard_start, self.shard_start + self.shard_numel
                if max(a, lo) < min(b, hi):
                    self._pp_dup.append((max(a, lo) - lo, min(b, hi) - lo))
        if (self.sequence_parallel and dev.type == "cuda" and dist.get_backend(self.tp_group) == "nccl"
                and os.environ.get("LIBRA_SP_FUSED", "1") != "0"):
            # row-parallel linears (o_proj, down_proj: output width H) reduce-scatter inside the GEMM
            # kernel over NVLink peer memory, for chunks up to the larger token budget
            from libra_b200.parallel.sequence_parallel import enable_fused_sequence_parallel, sp_multiple

            m = sp_multiple(self.tp_size, dev)
            rows = max(self.max_tokens_per_micro_batch, self.max_tokens_per_recompute_batch)
            enable_fused_sequence_parallel(self.tp_group, (rows + m - 1) // m * m, [self.cfg.hidden_size], [], dev)
        from libra_b200.parallel.tensor_parallel import tp_partial_grad_params

        if (self.tp_size > 1 and dev.type == "cuda" and dist.get_backend(self.tp_group) == "nccl"
                and os.environ.get("LIBRA_TP_PEER_LOGPROB", "1") != "0"):
            # the LM head's per-row shard statistics are exchanged over peer memory (one kernel, no NCCL)
            from libra_b200.parallel.tensor_parallel import enable_peer_logprob_exchange

            enable_peer_logprob_exchange(self.tp_group, max(self.max_tokens_per_micro_batch,
                                                            self.max_tokens_per_recompute_batch), dev)
        self._tp_partial = [self.params[n].main_grad for n in tp_partial_grad_params(
            list(self.params), self.sequence_parallel)] if self.tp_size > 1 else []
        # replicated (1-D) parameters inside this rank's optimizer shard: the
        # global grad norm counts them once, not once per TP rank
        self._tp_replicated = []
        if self.tp_size > 1:
            lo, hi = self.shard_start, self.shard_start + self.shard_numel
            for n, p in self.params.items():
                if p.dim() == 1:
                    a, b = self.layout.segment(n)
                    a, b = max(a, lo), min(b, hi)
                    if a < b:
                        self._tp_replicated.append((a - lo, b - lo))
        self._peer_grad = None
        self._sq_ready = False
        if self._peer_dp_applies():
            self.enable_peer_data_parallel()

    def _init_pipeline(self) -> None:
        """Pipeline stages over the mesh (TP, DP, PP fastest first): this rank's
        layer range, its neighbours in the pipeline, and the group that sums the
        tied word embedding's gradient between the first and the last stage."""
        self.pp_rank, self.pp_group, self.pp_prev, self.pp_next, self.pp_embed_group = 0, None, None, None, None
        self.stage_layers = range(self.cfg.num_hidden_layers)
        if self.pp_size <= 1:
            return
        if self.tp_size != 1 or self.ep_size != 1:
            raise ValueError("pipeline parallelism runs with tp_size=1 and ep_size=1")
        if not dist.is_initialized():
            raise RuntimeError("pipeline parallelism needs an initialized process group")
        from libra_b200.parallel.mesh import ParallelMesh
        from libra_b200.parallel.pipeline import PipelineStage

        rank = dist.get_rank()
        self.mesh = ParallelMesh(dist.get_world_size(), pp=self.pp_size)
        c = self.mesh.coords(rank)
        self.pp_rank = c.pp
        self.pp_group = self.mesh.group("pp", rank)
        if self.dp_group is None:
            self.dp_group = self.mesh.group("dp", rank)
        members = self.mesh.members("pp", rank)
        self.pp_prev = members[self.pp_rank - 1] if self.pp_rank > 0 else None
        self.pp_next = members[self.pp_rank + 1] if self.pp_rank + 1 < self.pp_size else None
        self.pp_first, self.pp_last = members[0], members[-1]
        self.stage_layers = PipelineStage.split_layers(self.cfg.num_hidden_layers, self.pp_size)[self.pp_rank]
        if self.cfg.tie_word_embeddings:
            for d in range(self.mesh.dp):  # every rank creates every group, in the same order
                ranks = [self.mesh.rank_of(dp=d, pp=0), self.mesh.rank_of(dp=d, pp=self.pp_size - 1)]
                grp = dist.new_group(ranks)
                if rank in ranks:
                    self.pp_embed_group = grp

    def _stage_owns(self, name: str) -> bool:
        first, last = self.pp_rank == 0, self.pp_rank == self.pp_size - 1
        if name.startswith("layers."):
            return int(name.split(".")[1]) in self.stage_layers
        if name == "embed_tokens":
            return first or (last and self.cfg.tie_word_embeddings)
        return last  # final norm, untied LM head

    # ------------------------------------------------------------------ pipeline stages
    def _pp_stage(self, mb: Dict[str, Any], x: Optional[torch.Tensor]) -> torch.Tensor:
        """This stage's layers; the last stage returns the action tokens' logprobs."""
        m, batch = self.model, mb["batch"]
        if self.pp_rank == 0:
            x = m.embed(batch.tokens)
        for i in self.stage_layers:
            if self.recompute_activations and torch.is_grad_enabled():
                x = torch.utils.checkpoint.checkpoint(m._layer, i, x, batch.positions, batch.cu_seqlens,
                                                      batch.max_seqlen, batch.tiles, use_reentrant=False)
            else:
                x = m._layer(i, x, batch.positions, batch.cu_seqlens, batch.max_seqlen, batch.tiles)
        if self.pp_rank < self.pp_size - 1:
            return x
        h = ops.rmsnorm(x, m.p["norm"], self.cfg.rms_norm_eps)
        rows = h.index_select(0, batch.action_rows)
        return ops.lm_head_logprob(rows, m.lm_head_weight, batch.action_targets, self.temperature)

    @torch.no_grad()
    def _pp_logprobs(self, device_batches: List[Dict[str, Any]]) -> List[torch.Tensor]:
        """Forward-only pipeline over the chunks (each stage receives, runs its
        layers, sends on; the sends are asynchronous, so consecutive chunks
        overlap across stages); the last stage's logprobs are broadcast to every
        stage of the pipeline."""
        out = []
        last = self.pp_rank == self.pp_size - 1
        for mb in device_batches:
            y = self._pp_stage(mb, self._p2p.recv_forward())
            if last:
                out.append(y.float().contiguous())
            else:
                self._p2p.send_forward(y)
                out.append(torch.empty(int(mb["batch"].action_rows.numel()), dtype=torch.float32,
                                       device=self.device))
        self._p2p.wait_sends()
        for t in out:
            dist.broadcast(t, src=self.pp_last, group=self.pp_group)
        return out

    def _pp_forward_backward(self, device_micro_batches: List[Dict[str, Any]], acc: torch.Tensor) -> None:
        """1F1B over the chunks (parallel/pipeline.py): the last stage turns
        logprobs into the GRPO loss; afterwards the first and last stages sum
        the tied embedding's gradient and the loss statistics reach every stage."""
        from libra_b200.parallel.pipeline import allreduce_tied_embedding_grad, one_f_one_b

        last = self.pp_rank == self.pp_size - 1

        def stage(mb, x):
            y = self._pp_stage(mb, x)
            if not last:
                return y
            loss, pg, kl = self.loss(y, mb["old_logp"], mb["adv"], mb.get("w"))
            acc.add_(torch.stack([loss.detach(), pg.detach(), kl.detach()]))
            return loss

        with nvtx.nvtx_range("forward_backward"):
            one_f_one_b(stage, device_micro_batches, self._p2p, self.pp_size, self.pp_rank)
        if self.pp_embed_group is not None:
            allreduce_tied_embedding_grad(self.params["embed_tokens"], self.pp_embed_group)
        dist.broadcast(acc, src=self.pp_last, group=self.pp_group)

    def export_params(self) -> Dict[str, torch.Tensor]:
        """Every parameter of the full (unsharded) model for an export (HF weights
        for rollout, an in-process rollout engine): tensor-parallel shards are
        gathered to the replica's first TP rank and merged; pipeline stages send
        theirs to the first stage.  Collective over the first data-parallel
        replica's TP or pipeline group; other ranks return their own tensors."""
        local = {k: v.detach() for k, v in self.params.items()}
        if self.ep_size > 1:
            # experts are split over the first EP group: gather them in EP-rank order (the dense part is
            # the same on every rank)
            if self.dp_rank >= self.ep_size:
                return local
            mine = {k: v.cpu() for k, v in local.items() if is_expert_param(k)}
            parts = [None] * self.ep_size
            dist.all_gather_object(parts, mine, group=self.ep_group)
            out = dict(local)
            for k in mine:
                out[k] = torch.cat([p[k] for p in parts]).to(local[k].device)
            return out
        if self.tp_size > 1:
            if self.mesh.coords(dist.get_rank()).dp != 0:
                return local
            first = dist.get_global_rank(self.tp_group, 0)
            parts = [None] * self.tp_size if self.tp_rank == 0 else None
            dist.gather_object({k: v.cpu() for k, v in local.items()}, parts, dst=first, group=self.tp_group)
            if self.tp_rank != 0:
                return local
            from libra_b200.parallel.tensor_parallel import merge_tp_shards

            return merge_tp_shards(parts, self.cfg, self.tp_size)
        if self.pp_size <= 1 or self.mesh.coords(dist.get_rank()).dp != 0:
            return local
        parts = [None] * self.pp_size if self.pp_rank == 0 else None
        dist.gather_object({k: v.cpu() for k, v in local.items()}, parts, dst=self.pp_first, group=self.pp_group)
        if self.pp_rank != 0:
            return local
        full: Dict[str, torch.Tensor] = {}
        for part in parts:
            full.update(part)
        return full

    def _init_expert_parallel(self) -> None:
        """Expert-parallel groups inside the data-parallel group: ``ep_group`` =
        ``ep_size`` consecutive DP ranks that split the experts between them;
        ``edp_group`` = the DP ranks holding the same experts (their expert
        gradients are summed)."""
        self.ep_group = self.edp_group = None
        self.ep_rank = 0
        if self.ep_size <= 1:
            return
        if self.tp_size > 1:
            raise ValueError("expert parallelism runs with tp_size=1 (attention and dense layers data-parallel)")
        if not dist.is_initialized():
            raise RuntimeError("expert parallelism needs an initialized process group")
        ep = self.ep_size
        if self.dp_size % ep:
            raise ValueError(f"ep_size={ep} must divide the data-parallel size {self.dp_size}")
        ranks = dist.get_process_group_ranks(self.dp_group) if self.dp_group is not None else \
            list(range(dist.get_world_size()))
        for g0 in range(0, len(ranks), ep):  # every rank creates every group, in the same order
            grp = dist.new_group(ranks[g0:g0 + ep])
            if g0 <= self.dp_rank < g0 + ep:
                self.ep_group = grp
        for i in range(ep):
            grp = dist.new_group(ranks[i::ep])
            if self.dp_rank % ep == i:
                self.edp_group = grp
        self.ep_rank = self.dp_rank % ep

    def _align_chunks(self, chunks: List[List[int]]) -> List[List[int]]:
        """Expert parallelism exchanges tokens in every MoE layer of every
        forward/backward, so all ranks of an EP group must run the same number
        of chunks: split the largest chunks until every rank has the group's
        maximum."""
        if self.ep_size <= 1:
            return chunks
        dev = self.device if not self._gloo() else torch.device("cpu")
        n = torch.tensor([len(chunks)], dtype=torch.int64, device=dev)
        dist.all_reduce(n, op=dist.ReduceOp.MAX, group=self.ep_group)
        target = int(n.item())
        chunks = [list(c) for c in chunks]
        while len(chunks) < target:
            i = max(range(len(chunks)), key=lambda j: len(chunks[j]))
            if len(chunks[i]) < 2:
                raise RuntimeError(f"expert-parallel ranks need {target} chunks but this rank has only "
                                   f"{sum(len(c) for c in chunks)} trajectories")
            c = chunks[i]
            chunks[i:i + 1] = [c[:len(c) // 2], c[len(c) // 2:]]
        return chunks

    # ------------------------------------------------------------------ protocol helpers
    def get_version(self) -> int:
        return self.current_version

    def set_version(self, version: int) -> None:
        self.current_version = int(version)

    def get_data_parallel_rank(self) -> int:
        return getattr(self, "dp_rank", 0)

    def get_data_parallel_world_size(self) -> int:
        return getattr(self, "dp_size", 1)

    def is_batch_source(self) -> bool:
        # every DP replica owns its batch; with pipeline stages its first stage collects it
        return getattr(self, "pp_rank", 0) == 0

    def get_local_batch_size(self, global_batch_size: int) -> int:
        return int(global_batch_size) // max(1, self.get_data_parallel_world_size())

    def distribute_trajectories(self, trajectories):
        if self.pp_size > 1 and getattr(self, "pp_group", None) is not None:
            box = [trajectories or []]  # the replica's first stage hands its batch to the other stages
            dist.broadcast_object_list(box, src=self.pp_first, group=self.pp_group)
            return box[0]
        return trajectories or []

    def align_distributed_trajectories(self, trajectories):
        return trajectories  # packed sequences need no cross-rank padding

    def num_parameters(self) -> int:
        return self.layout.numel

    # ------------------------------------------------------------------ batching
    @staticmethod
    def _traj_tensors(traj: Dict[str, Any]):
        ids = traj["input_ids"].reshape(-1)
        mask = traj.get("loss_mask")
        mask = torch.ones_like(ids) if mask is None else mask.reshape(-1)
        return ids, mask

    def pack(self, trajectories: List[Dict[str, Any]], with_old_logprobs: bool = True,
             traj_weights: Optional[List[float]] = None) -> Dict[str, Any]:
        """Pack trajectories (host tensors) into one host micro-batch.

        ``traj_weights[i]`` is the loss weight of every action token of
        trajectory i (see ``loss_weights``)."""
        ids, masks = zip(*(self._traj_tensors(t) for t in trajectories))
        pad = 1
        if self.sequence_parallel:
            from libra_b200.parallel.sequence_parallel import sp_multiple

            pad = sp_multiple(self.tp_size, self.device)
        batch = pack_sequences(list(ids), list(masks), pad_multiple=pad)
        extra: Dict[str, torch.Tensor] = {}
        if with_old_logprobs:
            old = torch.cat([t["logprobs"].reshape(-1).float() for t in trajectories])
            # old logprob of the action token at packed row r+1
            extra["old_logp"] = old.index_select(0, batch.action_rows + 1)
            adv = torch.tensor([float(t.get("advantages", t["rewards"]).reshape(-1)[0]) for t in trajectories])
            sidx = batch.seq_index.long()
            extra["adv"] = adv.index_select(0, sidx)
            w = torch.tensor(traj_weights if traj_weights is not None else [1.0] * len(trajectories),
                             dtype=torch.float32)
            extra["w"] = w.index_select(0, sidx)
            extra["rewards"] = torch.tensor([float(t["rewards"].reshape(-1)[0]) for t in trajectories])
        return {"batch": batch, **extra}

    def loss_weights(self, trajectories: List[Dict[str, Any]]) -> List[float]:
        """Per-trajectory token weight reproducing the reference loss aggregation:
        mean over groups of ``micro_batch_size`` trajectories of the group's
        masked token mean  =>  w = 1 / (actions in the group * number of groups)."""
        n = len(trajectories)
        groups = [list(range(s, min(n, s + self.micro_batch_size))) for s in range(0, n, self.micro_batch_size)]
        w = [0.0] * n
        for g in groups:
            count = sum(int(self._traj_tensors(trajectories[i])[1].reshape(-1)[1:].sum()) for i in g)
            for i in g:
                w[i] = 1.0 / (max(count, 1) * len(groups))
        return w

    def to_device(self, packed: Dict[str, Any]) -> Dict[str, Any]:
        dev = self.device
        if dev.type == "cuda":
            b = _pin_batch(packed["batch"])
            self.io_bytes["h2d"] += sum(t.numel() * t.element_size() for t in
                                        (b.tokens, b.positions, b.cu_seqlens, b.action_rows, b.action_targets,
                                         b.seq_index, b.attn_tiles, b.attn_kv_tiles) if t is not None)
            out = {"batch": b.to(dev, non_blocking=True)}
            for k, v in packed.items():
                if k != "batch":
                    out[k] = (v if v.is_pinned() else v.pin_memory()).to(dev, non_blocking=True)
                    self.io_bytes["h2d"] += v.numel() * v.element_size()
            return out
        return {"batch": packed["batch"], **{k: v for k, v in packed.items() if k != "batch"}}

    @staticmethod
    def chunk_by_tokens(trajectories: List[Dict[str, Any]], max_tokens: int) -> List[List[int]]:
        """Consecutive trajectory index chunks of at most ``max_tokens`` tokens (>= 1 trajectory each)."""
        chunks, cur, cur_tokens = [], [], 0
        for i, t in enumerate(trajectories):
            n = int(t["input_ids"].numel())
            if cur and cur_tokens + n > max_tokens:
                chunks.append(cur)
                cur, cur_tokens = [], 0
            cur.append(i)
            cur_tokens += n
        if cur:
            chunks.append(cur)
        return chunks

    def micro_batches(self, trajectories: List[Dict[str, Any]], size: int) -> Iterable[List[Dict[str, Any]]]:
        for s in range(0, len(trajectories), size):
            yield trajectories[s:s + size]

    def prepare_update(self, trajectories: List[Dict[str, Any]]) -> List[Dict[str, Any]]:
        """Host-side packed execution chunks (with loss weights) for one update."""
        w = self.loss_weights(trajectories)
        return [self.pack([trajectories[i] for i in idx], True, [w[i] for i in idx])
                for idx in self._align_chunks(self.chunk_by_tokens(trajectories, self.max_tokens_per_micro_batch))]

    def prepare_recompute(self, trajectories: List[Dict[str, Any]]):
        """(trajectory chunk, packed host batch) pairs for logprob recompute."""
        out = []
        limit = self.max_tokens_per_recompute_batch if self.ep_size <= 1 else self.max_tokens_per_micro_batch
        for idx in self._align_chunks(self.chunk_by_tokens(trajectories, limit)):
            chunk = [trajectories[i] for i in idx]
            out.append((chunk, self.pack(chunk, with_old_logprobs=False)))
        return out

    # ------------------------------------------------------------------ math
    def loss(self, logp, old_logp, adv, weight=None):
        """Weighted PPO-clip + k3-KL.  Without ``weight`` every token gets 1/count
        (the masked token mean of one micro-batch)."""
        log_ratio = logp - old_logp
        ratio = torch.exp(log_ratio.clamp(-20.0, 20.0))
        clipped = ratio.clamp(1.0 - self.clip_epsilon, 1.0 + self.clip_epsilon)
        pg = torch.maximum(-adv * ratio, -adv * clipped)
        kl = (ratio - 1.0) - log_ratio
        if weight is None:
            weight = torch.full_like(logp, 1.0 / max(int(logp.numel()), 1))
        pg_loss = (pg * weight).sum()
        kl_loss = (kl * weight).sum()
        return pg_loss + self.kl_coef * kl_loss, pg_loss, kl_loss

    # ------------------------------------------------------------------ public API
    @torch.no_grad()
    def recompute_logprobs(self, trajectories: List[Dict[str, Any]]) -> None:
        """Refresh trajectory["logprobs"] with the current policy (host tensors in, host tensors out)."""
        results = []
        prepared = self.prepare_recompute(trajectories)
        pp_lps = self._pp_logprobs([self.to_device(h) for _, h in prepared]) if self.pp_size > 1 else None
        for j, (chunk, host) in enumerate(prepared):
            if pp_lps is not None:
                lp = pp_lps[j]
            else:
                dev_mb = self.to_device(host)
                with nvtx.nvtx_range("recompute_forward"):
                    lp = self.model.action_logprobs(dev_mb["batch"], self.temperature)
            results.append((chunk, host["batch"], lp.to("cpu", non_blocking=True)))
            self.io_bytes["d2h"] += lp.numel() * lp.element_size()
        if self.device.type == "cuda":
            torch.cuda.current_stream(self.device).synchronize()
        for chunk, batch, lp in results:
            cu = batch.cu_seqlens.tolist()
            rows = batch.action_rows + 1
            for i, traj in enumerate(chunk):
                L = cu[i + 1] - cu[i]
                sel = (rows >= cu[i]) & (rows < cu[i + 1])
                updated = torch.zeros(L, dtype=torch.float32)
                updated[rows[sel] - cu[i]] = lp[sel]
                traj["logprobs"] = updated.view(1, L)

    def grpo_update(self, trajectories: List[Dict[str, Any]], ppo_epochs: int = 1) -> Dict[str, float]:
        """One optimizer step per PPO epoch over the whole batch (host inputs)."""
        epoch_stats = []
        for _ in range(ppo_epochs):
            mbs = [self.to_device(h) for h in self.prepare_update(trajectories)]
            epoch_stats.append(self.update_packed(mbs))
        merged = _merge_stats(epoch_stats)
        merged["version"] = self.current_version
        return merged

    def update_packed(self, device_micro_batches: List[Dict[str, Any]], sync_stats: bool = True) -> Dict[str, Any]:
        """Forward/backward over device-resident weighted chunks + optimizer step."""
        self.flat_grad.zero_()
        acc = torch.zeros(3, dtype=torch.float32, device=self.device)
        if self.pp_size > 1:
            self._pp_forward_backward(device_micro_batches, acc)
        for mb in device_micro_batches if self.pp_size == 1 else []:
            with nvtx.nvtx_range("forward_backward"):
                logp = self.model.action_logprobs(mb["batch"], self.temperature)
                loss, pg, kl = self.loss(logp, mb["old_logp"], mb["adv"], mb.get("w"))
                loss.backward()
            acc += torch.stack([loss.detach(), pg.detach(), kl.detach()])
        with nvtx.nvtx_range("grad_reduce"):
            self._apply_elastic_inter_replica_gradients()
            for g in self._tp_partial:  # per-head norm weights see only this rank's heads
                dist.all_reduce(g, group=self.tp_group)
            self._reduce_gradients()
            self._publish_elastic_update()
        with nvtx.nvtx_range("optimizer_step"):
            self._optimizer_step()
        if not sync_stats:
            return {"loss_sum": acc}
        rewards = [mb["rewards"] for mb in device_micro_batches if "rewards" in mb]
        r = torch.cat(rewards) if rewards else torch.zeros(0, device=self.device)
        parts = [acc, r.sum().reshape(1).float(), self.sq_norm]
        if self.device.type == "cuda":
            # the error word rides along with the stats read: a bounded wait that gave up inside this step
            # (the fused parameter gather waits on its peers) surfaces here, before the next forward
            parts.append(ops.error_flag(self.device)[:1].float())
        vals = torch.cat(parts).tolist()
        self.io_bytes["d2h"] += 4 * len(vals)
        if self.device.type == "cuda" and vals[-1] != 0:
            ops.error_flag(self.device)[0].zero_()
            raise ops.KernelError(int(vals[-1]), f"{self.device} (GRPO update)")
        out = {"loss": vals[0], "pg_loss": vals[1], "kl": vals[2], "reward_sum": vals[3],
               "n_samples": float(r.numel()), "n_updates": 1.0, "reward_mean": vals[3] / max(r.numel(), 1),
               "grad_norm": math.sqrt(max(vals[4], 0.0))}
        return self._reduce_stats(out)

    # ------------------------------------------------------------------ gradients/optimizer
    def _gloo(self) -> bool:
        return dist.get_backend(self.dp_group) == "gloo"

    def _reduce_gradients(self) -> None:
        """DP gradient reduction: reduce-scatter (distributed optimizer) or all-reduce."""
        if self.dp_size <= 1 or not dist.is_initialized():
            return
        dense = self.flat_grad[:self.dense_numel]
        if self._peer_grad is not None:
            # one kernel: pull this rank's shard from every rank over NVLink, average, global sum of squares
            self._peer_grad.reduce(self.grad_shard, scale=1.0 / self.dp_size, sq_norm=self.sq_norm)
            self._sq_ready = True
        elif self.sharded:
            if self._gloo():  # gloo has no reduce_scatter_tensor
                dist.all_reduce(dense, op=dist.ReduceOp.SUM, group=self.dp_group)
                self.grad_shard.copy_(dense[self.shard_start:self.shard_start + self.shard_numel])
            else:
                dist.reduce_scatter_tensor(self.grad_shard, dense, op=dist.ReduceOp.SUM, group=self.dp_group)
            self.grad_shard.div_(self.dp_size)
        else:
            dist.all_reduce(dense, op=dist.ReduceOp.SUM, group=self.dp_group)
            dense.div_(self.dp_size)
        if self.padded_numel > self.dense_numel:
            # expert gradients already hold every EP rank's tokens (the exchange's backward brought them);
            # sum over the replicas of these experts, then average like the dense part
            xg = self.flat_grad[self.dense_numel:]
            if self.edp_group is not None and dist.get_world_size(self.edp_group) > 1:
                dist.all_reduce(xg, op=dist.ReduceOp.SUM, group=self.edp_group)
            xg.div_(self.dp_size)

    def _gather_params(self, shard_param: torch.Tensor) -> None:
        if self._gloo():
            parts = list(self.flat_param[:self.dense_numel].chunk(self.dp_size))
            dist.all_gather(parts, shard_param.clone(), group=self.dp_group)
            return
        dist.all_gather_into_tensor(self.flat_param[:self.dense_numel], shard_param.clone(), group=self.dp_group)

    def _optimizer_step(self) -> None:
        self.step_count += 1
        if self._sq_ready:  # the peer reduce-scatter left the global sum of squares of the dense gradient
            self._sq_ready = False
        else:
            self.sq_norm.zero_()
            ops.grad_sq_norm(self.grad_shard, self.sq_norm)
        if self.tp_size > 1:
            rep = torch.zeros(1, dtype=torch.float32, device=self.device)
            for a, b in self._tp_replicated:
                rep += self.grad_shard[a:b].float().pow(2).sum()
            both = torch.cat([self.sq_norm, rep])
            if self.sharded:
                dist.all_reduce(both, group=self.dp_group)
            total = both[:1].clone()
            dist.all_reduce(total, group=self.tp_group)
            self.sq_norm.copy_(total - (self.tp_size - 1) * both[1:])
        elif self.sharded and self._peer_grad is None:
            dist.all_reduce(self.sq_norm, op=dist.ReduceOp.SUM, group=self.dp_group)
        if self.pp_size > 1:
            # every stage holds its own layers: sum the stages, the tied embedding once (first stage's copy)
            dup = torch.zeros(1, dtype=torch.float32, device=self.device)
            if self.pp_rank == self.pp_size - 1 and self.cfg.tie_word_embeddings:
                for a, b in self._pp_dup:
                    dup += self.grad_shard[a:b].float().pow(2).sum()
                if self.sharded:
                    dist.all_reduce(dup, group=self.dp_group)
            total = self.sq_norm - dup
            dist.all_reduce(total, group=self.pp_group)
            self.sq_norm.copy_(total)
        o = self.optim
        if self.x_master is not None:
            # experts: the global norm adds every EP rank's experts once; the AdamW update of this rank's
            # experts writes their bf16 values in place (no gather: nobody else holds them)
            xg = self.flat_grad[self.dense_numel:]
            x_sq = torch.zeros(1, dtype=torch.float32, device=self.device)
            ops.grad_sq_norm(xg, x_sq)
            if self.ep_group is not None:
                dist.all_reduce(x_sq, op=dist.ReduceOp.SUM, group=self.ep_group)
            self.sq_norm.add_(x_sq)
            ops.adamw_step(self.x_master, xg, self.x_m, self.x_v, self.flat_param[self.dense_numel:], lr=o.lr,
                           beta1=o.betas[0], beta2=o.betas[1], eps=o.eps, weight_decay=o.weight_decay,
                           step=self.step_count, max_grad_norm=o.max_grad_norm, sq_norm=self.sq_norm)
        shard_param = self.flat_param[self.shard_start:self.shard_start + self.shard_numel]
        if self._offload_k:
            self._offloaded_step(shard_param)
            return
        peer = getattr(self, "_peer_param_gather", None)
        if peer is not None:  # AdamW stores the new bf16 shard straight into every rank's parameters
            peer.step(self.master, self.grad_shard, self.exp_avg, self.exp_avg_sq, lr=o.lr, beta1=o.betas[0],
                      beta2=o.betas[1], eps=o.eps, weight_decay=o.weight_decay, step=self.step_count,
                      max_grad_norm=o.max_grad_norm, sq_norm=self.sq_norm)
            return
        ops.adamw_step(self.master, self.grad_shard, self.exp_avg, self.exp_avg_sq, shard_param, lr=o.lr,
                       beta1=o.betas[0], beta2=o.betas[1], eps=o.eps, weight_decay=o.weight_decay,
                       step=self.step_count, max_grad_norm=o.max_grad_norm, sq_norm=self.sq_norm)
        if self.sharded:
            self._gather_params(shard_param)

    def _offloaded_step(self, shard_param: torch.Tensor) -> None:
        """AdamW with the optimizer state split between host and device: the
        device part runs as a kernel while the host steps its prefix (fp32
        math with torch's CPU kernels); the host result goes back with one
        pinned copy, then the data-parallel gather completes the parameters."""
        o, k, h = self.optim, self._offload_k, self._host_opt
        hp = dict(lr=o.lr, beta1=o.betas[0], beta2=o.betas[1], eps=o.eps, weight_decay=o.weight_decay,
                  step=self.step_count, max_grad_norm=o.max_grad_norm)
        cuda = self.device.type == "cuda"
        h["grad"].copy_(self.grad_shard[:k], non_blocking=cuda)
        sq_host = self.sq_norm.to("cpu", non_blocking=cuda)
        done = torch.cuda.Event() if cuda else None
        if cuda:
            done.record()
        if self.master.numel():
            ops.adamw_step(self.master, self.grad_shard[k:], self.exp_avg, self.exp_avg_sq, shard_param[k:],
                           sq_norm=self.sq_norm, **hp)
        if cuda:
            done.synchronize()
        ops.adamw_step(h["master"], h["grad"], h["exp_avg"], h["exp_avg_sq"], h["param"], sq_norm=sq_host, **hp)
        shard_param[:k].copy_(h["param"], non_blocking=cuda)
        self.io_bytes["d2h"] += 4 * k + 4
        self.io_bytes["h2d"] += 2 * k
        if self.sharded:
            self._gather_params(shard_param)

    def optimizer_state_tensors(self) -> Dict[str, torch.Tensor]:
        """Full-shard master weights and moments (host and device parts joined
        on the host when part of the state is offloaded)."""
        names = ("master", "exp_avg", "exp_avg_sq")
        if not self._offload_k:
            return {n: getattr(self, n) for n in names}
        return {n: torch.cat([self._host_opt[n], getattr(self, n).cpu()]) for n in names}

    def load_optimizer_state_tensors(self, state: Dict[str, torch.Tensor]) -> None:
        k = self._offload_k
        for n in ("master", "exp_avg", "exp_avg_sq"):
            t = state[n]
            if k:
                self._host_opt[n].copy_(t[:k])
            getattr(self, n).copy_(t[k:])

    def _peer_dp_applies(self) -> bool:
        """Whether the data-parallel gradient and parameter exchange runs over
        NVLink peer memory: a sharded distributed optimizer on NCCL ranks of one
        box (CUDA IPC), TP=1, at most 8 ranks; ``LIBRA_PEER_DP=0`` keeps NCCL.
        Every rank reaches the same answer (the host check is collective)."""
        if (self.device.type != "cuda" or not self.sharded or not dist.is_initialized() or self._gloo()
                or self.tp_size != 1 or self.dp_size > 8 or self.shard_numel % 4
                or os.environ.get("LIBRA_PEER_DP", "1") == "0"):
            return False
        hosts = [None] * self.dp_size
        dist.all_gather_object(hosts, os.uname().nodename, group=self.dp_group)
        return len(set(hosts)) == 1

    def enable_peer_data_parallel(self) -> None:
        """Collective over the DP group: gradient reduce-scatter (fused with the
        1/dp average and the global norm) and the parameter all-gather (fused
        into AdamW) over NVLink peer memory instead of NCCL."""
        from libra_b200.parallel.peer_grad_reduce import PeerGradReduce

        group = self.dp_group if self.dp_group is not None else dist.group.WORLD
        self._peer_grad = PeerGradReduce(group, self.flat_grad, self.shard_start, self.shard_numel)
        if not self._offload_k:  # with part of the state on the host the gather runs after both halves
            self.enable_fused_param_gather()

    def close_peer_data_parallel(self) -> None:
        for attr in ("_peer_grad", "_peer_param_gather"):
            obj = getattr(self, attr, None)
            if obj is not None:
                obj.close()
                setattr(self, attr, None)

    def enable_fused_param_gather(self) -> bool:
        """Collective over the DP group: fuse the distributed optimizer's parameter all-gather into the
        AdamW kernel (peer-memory stores over NVLink).  Returns False where it does not apply
        (no sharded optimizer, gloo ranks, or a shard that is not a multiple of 4 elements).
        Call it after ``initialize``."""
        if not hasattr(self, "sharded"):
            raise RuntimeError("enable_fused_param_gather() needs an initialized engine (call initialize() first)")
        if not self.sharded or self._gloo() or self.shard_numel % 4:
            return False
        from libra_b200.parallel.peer_param_gather import PeerParamGather

        group = self.dp_group if self.dp_group is not None else dist.group.WORLD
        self._peer_param_gather = PeerParamGather(group, self.flat_param, self.shard_start, self.shard_numel)
        return True

    def _reduce_stats(self, stats: Dict[str, float]) -> Dict[str, float]:
        if self.dp_size <= 1 or not dist.is_initialized():
            return stats
        vec = torch.tensor([stats["loss"], stats["pg_loss"], stats["kl"], stats["reward_sum"], stats["n_samples"],
                            stats["n_updates"], stats["grad_norm"]], dtype=torch.float32, device=self.device)
        dist.all_reduce(vec, group=self.dp_group)
        n = self.dp_size
        v = vec.tolist()
        return {"loss": v[0] / n, "pg_loss": v[1] / n, "kl": v[2] / n, "reward_sum": v[3], "n_samples": v[4],
                "n_updates": v[5], "reward_mean": v[3] / max(v[4], 1.0), "grad_norm": v[6] / n}

    def release_optimizer_state(self) -> None:
        """Drop master/Adam/gradient buffers (inference-only holders of the weights)."""
        self.close_peer_data_parallel()
        self.master = self.exp_avg = self.exp_avg_sq = None
        self._host_opt, self._offload_k = None, 0
        self.grad_shard = None
        self.flat_grad = torch.zeros(0, dtype=torch.float32, device=self.device)
        for p in self.params.values():
            p.main_grad = None
            p.requires_grad_(False)
        if self.device.type == "cuda":
            torch.cuda.empty_cache()


    # ------------------------------------------------------------------ elastic hybrid hooks
    # Reference contract: engine/train_engine.py:854-960 (core replica ids,
    # domain attach, payload queue, snapshot capture/load, merge before the
    # DP reduction).  Here the whole gradient is the flat fp32 buffer, so a
    # payload is one tensor and the merge is an in-place add into it.
    def get_elastic_core_replica_ids(self) -> List[str]:
        return [f"dp{i}" for i in range(max(1, getattr(self, "dp_size", self.world_size)))]

    def get_elastic_core_process_group(self):
        return self.dp_group if self.dp_group is not None else (dist.group.WORLD if dist.is_initialized() else None)

    def configure_elastic_training(self, core_replica_ids: Optional[List[str]] = None,
                                   decouple_communication_domains: bool = True):
        from libra_b200.infra.elastic.hybrid_pool import InterReplicaGradientDomain

        self.elastic_gradient_domain = InterReplicaGradientDomain(
            core_replica_ids=core_replica_ids or self.get_elastic_core_replica_ids(),
            process_group=None if decouple_communication_domains else self.get_elastic_core_process_group(),
            decouple_communication_domains=decouple_communication_domains)
        return self.elastic_gradient_domain

    def set_elastic_gradient_domain(self, domain) -> None:
        self.elastic_gradient_domain = domain
        if domain is not None and not domain.decoupled_communication_domains:
            domain.process_group = self.get_elastic_core_process_group()

    def enqueue_hybrid_gradient_payload(self, payload) -> None:
        self._pending_hybrid_gradients.append(payload)

    def _apply_elastic_inter_replica_gradients(self) -> int:
        """Add matching hybrid payloads into this core replica's gradient
        before the core DP reduction; returns how many were merged."""
        if self.elastic_gradient_domain is not None and self.elastic_payload_wait_s > 0:
            self._wait_for_hybrid_payloads(self.step_count + 1, self.elastic_payload_wait_s)
        pending, self._pending_hybrid_gradients = self._pending_hybrid_gradients, []
        if not pending or self.elastic_gradient_domain is None:
            return 0
        core_id = f"dp{getattr(self, 'dp_rank', 0)}"
        used = self.elastic_gradient_domain.usable_payloads(core_id, pending, step=self.step_count + 1,
                                                            state_version=-1)
        for p in used:
            (g,) = p.tensors
            if g.numel() != self.flat_grad.numel():
                raise ValueError(f"hybrid payload has {g.numel()} elements, expected {self.flat_grad.numel()}")
            self.flat_grad.add_(g.to(device=self.flat_grad.device, dtype=torch.float32).view(-1))
        if used and self.elastic_average_merged:
            self.flat_grad.div_(1 + len(used))
        return len(used)

    def _wait_for_hybrid_payloads(self, step: int, timeout_s: float) -> bool:
        """Bounded wait until every active hybrid replica targeting this core
        replica has queued its payload for ``step``; a late replica simply
        misses the step (its payload is dropped by the step check)."""
        domain = self.elastic_gradient_domain
        want = set(domain.active_hybrid_ids_for_core(f"dp{getattr(self, 'dp_rank', 0)}"))
        deadline = time.monotonic() + timeout_s
        while want:
            have = {p.replica_id for p in list(self._pending_hybrid_gradients) if p.step in (step, -1)}
            if want <= have:
                return True
            if time.monotonic() > deadline:
                return False
            time.sleep(0.002)
        return True

    def _publish_elastic_update(self) -> None:
        if self.elastic_update_publisher is None:
            return
        if self.sharded and dist.is_initialized():
            full = torch.empty_like(self.flat_grad)
            if self._gloo():
                parts = list(full.chunk(self.dp_size))
                dist.all_gather(parts, self.grad_shard.clone(), group=self.dp_group)
            else:
                dist.all_gather_into_tensor(full, self.grad_shard, group=self.dp_group)
        else:
            full = self.flat_grad
        self.elastic_update_publisher(full, self.step_count + 1, self.current_version)

    def get_elastic_state_snapshot_path(self, version: int) -> str:
        root = os.environ.get("ELASTIC_TRAINING_STATE_DIR", "./logs/elastic_training_state")
        return os.path.join(root, f"v{version}", f"rank_{self.rank}.pt")

    def capture_elastic_state_snapshot(self, worker_id: str = "", target_core_id: str = "") -> int:
        """Write weights + this rank's optimizer shard for a joining replica."""
        path = self.get_elastic_state_snapshot_path(self.current_version)
        os.makedirs(os.path.dirname(path), exist_ok=True)
        snap = {"flat_param": self.flat_param.cpu(), "version": self.current_version, "step": self.step_count,
                "dp_rank": getattr(self, "dp_rank", 0), "dp_size": getattr(self, "dp_size", 1),
                "hidden_size": self.cfg.hidden_size, "num_layers": self.cfg.num_hidden_layers,
                "optim": {"lr": self.optim.lr, "betas": list(self.optim.betas), "eps": self.optim.eps,
                          "weight_decay": self.optim.weight_decay, "max_grad_norm": self.optim.max_grad_norm},
                "loss": {"kl_coef": self.kl_coef, "clip_epsilon": self.clip_epsilon, "temperature": self.temperature}}
        if self.master is not None:
            snap.update(master=self.master.cpu(), exp_avg=self.exp_avg.cpu(), exp_avg_sq=self.exp_avg_sq.cpu(),
                        shard_start=self.shard_start)
        tmp = path + ".tmp"
        torch.save(snap, tmp)
        os.replace(tmp, path)
        return self.current_version

    def load_elastic_state_snapshot(self, snapshot_path: str) -> int:
        snap = torch.load(snapshot_path, map_location="cpu", weights_only=True)
        if snap["flat_param"].numel() != self.flat_param.numel():
            raise ValueError("elastic snapshot does not match this model's parameter layout")
        self.flat_param.copy_(snap["flat_param"])
        if self.master is not None and "master" in snap:
            if snap["master"].numel() == self.master.numel():
                self.master.copy_(snap["master"])
                self.exp_avg.copy_(snap["exp_avg"])
                self.exp_avg_sq.copy_(snap["exp_avg_sq"])
            else:  # different sharding: rebuild the fp32 master from the weights, restart moments
                self.master.copy_(self.flat_param[self.shard_start:self.shard_start + self.shard_numel].float())
                self.exp_avg.zero_()
                self.exp_avg_sq.zero_()
        self.current_version = int(snap["version"])
        self.step_count = int(snap["step"])
        if "optim" in snap:  # a joining replica must step exactly like its core replica
            o = snap["optim"]
            self.optim = OptimConfig(lr=float(o["lr"]), betas=tuple(o["betas"]), eps=float(o["eps"]),
                                     weight_decay=float(o["weight_decay"]), max_grad_norm=float(o["max_grad_norm"]))
            self.kl_coef = float(snap["loss"]["kl_coef"])
            self.clip_epsilon = float(snap["loss"]["clip_epsilon"])
            self.temperature = float(snap["loss"]["temperature"])
        return self.current_version

    def compute_gradient_payload(self, trajectories: List[Dict[str, Any]], *, replica_id: str, target_core_id: str,
                                 step: int, membership_epoch: int, replica_rank: int = 0,
                                 replica_world_size: int = 1, loss_scale: float = 1.0):
        """Hybrid-replica side: forward/backward into the flat gradient, no
        reduction and no optimizer step; the payload aliases ``flat_grad``."""
        from libra_b200.infra.elastic.hybrid_pool import GradientPayload

        self.flat_grad.zero_()
        for hb in self.prepare_update(trajectories):
            mb = self.to_device(hb)
            logp = self.model.action_logprobs(mb["batch"], self.temperature)
            loss, _, _ = self.loss(logp, mb["old_logp"], mb["adv"], mb.get("w"))
            (loss * loss_scale).backward()
        return GradientPayload(replica_id, target_core_id, (self.flat_grad,), False, replica_rank,
                               replica_world_size, step, self.current_version, membership_epoch)

    def apply_gradient_update(self, reduced_flat_grad: torch.Tensor) -> None:
        """Hybrid-replica side of lockstep: take the core's post-reduce
        gradient and run the same optimizer step, keeping weights identical."""
        self.flat_grad.copy_(reduced_flat_grad.to(self.flat_grad.device, torch.float32).view(-1))
        if self.sharded:
            self.grad_shard.copy_(self.flat_grad[self.shard_start:self.shard_start + self.shard_numel])
        self._optimizer_step()

    # ------------------------------------------------------------------ weights
    def state_dict(self) -> Dict[str, torch.Tensor]:
        return {k: v.detach() for k, v in self.params.items()}

    def save_weights(self, path: str, version: int) -> None:
        from libra_b200.engine.checkpointing import DistributedCheckpointManager

        DistributedCheckpointManager(path).save(self, version)

    def load_weights(self, path: str, version: Optional[int] = None) -> None:
        from libra_b200.engine.checkpointing import DistributedCheckpointManager

        DistributedCheckpointManager(path).load(self, version)


def _fold_grad_into_main(p: torch.nn.Parameter) -> None:
    if p.grad is not None:
        p.main_grad.add_(p.grad.float())
        p.grad = None


def _pin_batch(b: PackedBatch) -> PackedBatch:
    pin = lambda t: t if t is None or t.is_pinned() else t.pin_memory()  # noqa: E731
    return PackedBatch(pin(b.tokens), pin(b.positions), pin(b.cu_seqlens), b.max_seqlen, pin(b.action_rows),
                       pin(b.action_targets), pin(b.seq_index), pin(b.attn_tiles), pin(b.attn_kv_tiles))


def _merge_stats(stats: List[Dict[str, float]]) -> Dict[str, float]:
    if not stats:
        return {"loss": 0.0, "pg_loss": 0.0, "kl": 0.0, "reward_sum": 0.0, "reward_mean": 0.0, "n_samples": 0.0,
                "n_updates": 0.0}
    updates = sum(float(s.get("n_updates", 1.0)) for s in stats)
    samples = sum(float(s.get("n_samples", 0.0)) for s in stats)
    rsum = sum(float(s.get("reward_sum", 0.0)) for s in stats)
    wavg = lambda key: sum(float(s.get(key, 0.0)) * float(s.get("n_updates", 1.0)) for s in stats) / max(updates, 1.0)  # noqa: E731
    return {"loss": wavg("loss"), "pg_loss": wavg("pg_loss"), "kl": wavg("kl"), "reward_sum": rsum,
            "reward_mean": rsum / max(samples, 1.0), "n_samples": samples, "n_updates": updates,
            "grad_norm": wavg("grad_norm")}


def create_train_engine(config) -> B200TrainEngine:
    """Factory from an AsyncRLConfig (reference ``engine/train_factory.py:11-76``).

    Every ``train_backend`` value maps onto the native engine; the model preset
    is taken from ``model_path`` when it names a preset, else from model_arch.
    The parallel layout comes from the config: ``train_tp_size`` (tensor
    parallel groups of consecutive ranks), ``train_ep_size`` (experts spread
    over that many data-parallel ranks), ``train_pp_size`` (pipeline stages of
    contiguous layers, 1F1B) and ``sequence_parallel``.
    """
    name = os.path.basename(str(config.model_path)).lower()
    try:
        cfg = get_config(name)
    except KeyError:
        from libra_b200.models.qwen3 import config_from_arch

        cfg = config_from_arch(config.model_arch)
    return B200TrainEngine(model=cfg, learning_rate=config.learning_rate, kl_coef=config.kl_coef,
                           clip_epsilon=config.clip_epsilon, micro_batch_size=config.micro_batch_size,
                           recompute_micro_batch_size=config.recompute_micro_batch_size, seed=config.seed,
                           use_distributed_optimizer=config.use_distributed_optimizer,
                           temperature=config.temperature, model_path=config.model_path,
                           tp_size=int(getattr(config, "train_tp_size", 1) or 1),
                           ep_size=int(getattr(config, "train_ep_size", 1) or 1),
                           sequence_parallel=bool(getattr(config, "sequence_parallel", False)),
                           precision_aware_optimizer=bool(getattr(config, "megatron_use_precision_aware_optimizer",
                                                                  False)),
                           optimizer_cpu_offload=bool(getattr(config, "megatron_optimizer_cpu_offload", False)),
                           optimizer_offload_fraction=float(getattr(config, "megatron_optimizer_offload_fraction",
                                                                    0.0)),
                           pp_size=int(getattr(config, "train_pp_size", 1) or 1))
