"""Qwen3 decoder family (dense and MoE) on the libra_b200 fused operators.

Architecture as trained by the reference through Megatron-Core / HF
(``engine/megatron_core_train_engine.py:279-317``, model arch YAMLs
``configs/model_arch_config/qwen3-*.yaml``): pre-norm decoder blocks with GQA
attention, per-head q/k RMSNorm, rotary embedding (theta 1e6), SwiGLU MLP or a
top-k routed expert MLP, final RMSNorm and an LM head (tied to the embedding
for Qwen3-4B).

B200 design choices:

* Sequences are **packed** into one token stream with ``cu_seqlens`` instead of
  being padded to the batch maximum (the reference pads,
  ``engine/megatron_core_train_engine.py:400-488``), so no FLOPs are spent on
  padding.
* All parameters live in **one flat bf16 buffer** (``ParamLayout``); the
  optimizer, the gradient reduction and the rollout weight sync each operate
  on a single contiguous buffer.  Gradients accumulate into a parallel flat
  fp32 buffer through ``weight.main_grad`` views.
* QKV and gate/up projections are fused column blocks; the o-proj and down
  projections add the residual inside the GEMM epilogue.
* The LM head is evaluated only on rows whose next token is an action token and
  is fused with the log-softmax (no fp32 [tokens, vocab] tensor).
"""

from __future__ import annotations

import math
from dataclasses import dataclass, field, asdict
from typing import Dict, List, Optional, Tuple

import torch
import torch.nn as nn

from libra_b200 import ops


@dataclass
class Qwen3Config:
    vocab_size: int = 151936
    hidden_size: int = 2560
    intermediate_size: int = 9728
    num_hidden_layers: int = 36
    num_attention_heads: int = 32
    num_key_value_heads: int = 8
    head_dim: int = 128
    rope_theta: float = 1_000_000.0
    rms_norm_eps: float = 1e-6
    tie_word_embeddings: bool = True
    max_position_embeddings: int = 40960
    initializer_range: float = 0.02
    # MoE (num_experts == 0 -> dense)
    num_experts: int = 0
    num_experts_per_tok: int = 8
    moe_intermediate_size: int = 768
    norm_topk_prob: bool = True
    router_init_std: float = 1.0

    @property
    def is_moe(self) -> bool:
        return self.num_experts > 0

    @property
    def q_width(self) -> int:
        return self.num_attention_heads * self.head_dim

    @property
    def kv_width(self) -> int:
        return self.num_key_value_heads * self.head_dim

    def num_params(self) -> int:
        return sum(math.prod(shape) for _, shape in param_shapes(self))

    def active_params(self) -> int:
        if not self.is_moe:
            return self.num_params()
        total = 0
        for name, shape in param_shapes(self):
            n = math.prod(shape)
            if ".experts." in name:
                n = n * self.num_experts_per_tok // self.num_experts
            total += n
        return total

    def to_dict(self) -> dict:
        return asdict(self)


PRESETS: Dict[str, Qwen3Config] = {
    "qwen3-4b": Qwen3Config(),
    "qwen3-14b": Qwen3Config(hidden_size=5120, intermediate_size=17408, num_hidden_layers=40,
                             num_attention_heads=40, num_key_value_heads=8, tie_word_embeddings=False),
    "qwen3-30b-a3b": Qwen3Config(hidden_size=2048, intermediate_size=6144, num_hidden_layers=48,
                                 num_attention_heads=32, num_key_value_heads=4, tie_word_embeddings=False,
                                 num_experts=128, num_experts_per_tok=8, moe_intermediate_size=768),
    # CPU plumbing model (2 layers, hidden 256, 4/2 heads of 64, FFN 704, vocab 1024)
    "tiny": Qwen3Config(vocab_size=1024, hidden_size=256, intermediate_size=704, num_hidden_layers=2,
                        num_attention_heads=4, num_key_value_heads=2, head_dim=64, tie_word_embeddings=True,
                        max_position_embeddings=4096),
    # smallest GPU-kernel-compatible model (head_dim 128) for tests and smoke runs
    "tiny-gpu": Qwen3Config(vocab_size=2048, hidden_size=512, intermediate_size=1024, num_hidden_layers=2,
                            num_attention_heads=4, num_key_value_heads=2, head_dim=128, tie_word_embeddings=True,
                            max_position_embeddings=8192),
    "tiny-moe": Qwen3Config(vocab_size=2048, hidden_size=512, intermediate_size=1024, num_hidden_layers=2,
                            num_attention_heads=4, num_key_value_heads=2, head_dim=128, tie_word_embeddings=False,
                            num_experts=8, num_experts_per_tok=2, moe_intermediate_size=256,
                            max_position_embeddings=8192),
}


def get_config(name_or_cfg) -> Qwen3Config:
    if isinstance(name_or_cfg, Qwen3Config):
        return name_or_cfg
    key = str(name_or_cfg).lower()
    if key not in PRESETS:
        raise KeyError(f"unknown model preset {name_or_cfg!r}; known: {sorted(PRESETS)}")
    return PRESETS[key]


# ---------------------------------------------------------------------------
# parameter layout
# ---------------------------------------------------------------------------

def is_expert_param(name: str) -> bool:
    return name.endswith("experts.w1") or name.endswith("experts.w2")


def param_shapes(cfg: Qwen3Config, tp_size: int = 1, tp_rank: int = 0,
                 ep_size: int = 1) -> List[Tuple[str, Tuple[int, ...]]]:
    """Canonical (name, local shape) list for one tensor-parallel rank.

    Column-parallel blocks (QKV, gate/up, expert w1) are split along their
    output rows, row-parallel blocks (o-proj, down, expert w2) along their input
    columns, and the embedding / LM head along the vocabulary.
    """
    H, D = cfg.hidden_size, cfg.head_dim
    nq, nkv = cfg.num_attention_heads, cfg.num_key_value_heads
    if nq % tp_size or cfg.intermediate_size % tp_size or cfg.vocab_size % tp_size:
        raise ValueError(f"tp_size={tp_size} does not divide the model dimensions")
    kv_local = max(1, nkv // tp_size)  # replicate KV heads when tp > nkv
    nq_l = nq // tp_size
    V_l = cfg.vocab_size // tp_size
    shapes: List[Tuple[str, Tuple[int, ...]]] = [("embed_tokens", (V_l, H))]
    for i in range(cfg.num_hidden_layers):
        p = f"layers.{i}."
        shapes += [
            (p + "input_layernorm", (H,)),
            (p + "qkv_proj", ((nq_l + 2 * kv_local) * D, H)),
            (p + "q_norm", (D,)),
            (p + "k_norm", (D,)),
            (p + "o_proj", (H, nq_l * D)),
            (p + "post_attention_layernorm", (H,)),
        ]
        if cfg.is_moe:
            E, Fe = cfg.num_experts, cfg.moe_intermediate_size
            if E % ep_size:
                raise ValueError(f"ep_size={ep_size} does not divide num_experts={E}")
            El = E // ep_size  # this expert-parallel rank's experts
            shapes += [
                (p + "router", (E, H)),
                (p + "experts.w1", (El, 2 * Fe // tp_size, H)),
                (p + "experts.w2", (El, H, Fe // tp_size)),
            ]
        else:
            F = cfg.intermediate_size // tp_size
            shapes += [(p + "gate_up_proj", (2 * F, H)), (p + "down_proj", (H, F))]
    shapes.append(("norm", (H,)))
    if not cfg.tie_word_embeddings:
        shapes.append(("lm_head", (V_l, H)))
    return shapes


class ParamLayout:
    """Offsets of every parameter inside the flat buffer (256-byte aligned)."""

    ALIGN = 128  # elements; keeps every view 16-byte aligned for TMA in bf16 and fp32

    def __init__(self, shapes: List[Tuple[str, Tuple[int, ...]]]):
        self.shapes = dict(shapes)
        self.order = [n for n, _ in shapes]
        self.offsets: Dict[str, int] = {}
        off = 0
        for name, shape in shapes:
            self.offsets[name] = off
            n = math.prod(shape)
            off += (n + self.ALIGN - 1) // self.ALIGN * self.ALIGN
        self.numel = off

    def views(self, flat: torch.Tensor) -> Dict[str, torch.Tensor]:
        out = {}
        for name in self.order:
            shape = self.shapes[name]
            off = self.offsets[name]
            out[name] = flat[off:off + math.prod(shape)].view(shape)
        return out

    def shift(self, names: List[str], delta: int) -> None:
        """Move the named parameters ``delta`` elements further into the buffer
        (a multiple of ALIGN; used to start a segment on a shard boundary)."""
        if delta % self.ALIGN:
            raise ValueError("layout shifts must keep the alignment")
        for n in names:
            self.offsets[n] += delta
        self.numel += delta

    def segment(self, name: str) -> Tuple[int, int]:
        off = self.offsets[name]
        return off, off + math.prod(self.shapes[name])


def init_params(cfg: Qwen3Config, views: Dict[str, torch.Tensor], seed: int = 0, expert_offset: int = 0) -> None:
    """Random init in place: N(0, initializer_range) for matrices, 1 for norms,
    N(0, router_init_std) for MoE routers (router logits ~ N(0,1) scale).

    Dense parameters draw from one stream in layout order; every expert's
    weights draw from a stream of their own keyed by (layer, global expert id),
    so an expert-parallel rank holding experts ``expert_offset ..`` gets exactly
    the weights the unsharded model has for them."""
    gen_device = next(iter(views.values())).device
    g = torch.Generator(device=gen_device)
    g.manual_seed(seed)
    ge = torch.Generator(device=gen_device)
    with torch.no_grad():
        for name, t in views.items():
            if t.dim() == 1:
                t.fill_(1.0)
            elif name.endswith("router"):
                t.normal_(0.0, cfg.router_init_std / math.sqrt(cfg.hidden_size), generator=g)
            elif is_expert_param(name):
                layer = int(name.split(".")[1])
                which = 1 if name.endswith("w1") else 2
                for e in range(t.shape[0]):
                    ge.manual_seed(((seed * 1000003 + layer) * 4099 + expert_offset + e) * 3 + which)
                    t[e].normal_(0.0, cfg.initializer_range, generator=ge)
            else:
                t.normal_(0.0, cfg.initializer_range, generator=g)


# ---------------------------------------------------------------------------
# packed batch
# ---------------------------------------------------------------------------

@dataclass
class PackedBatch:
    """Sequences packed into one stream.

    tokens/positions: [T]; cu_seqlens: [B+1] int32; max_seqlen: int.
    action_rows: indices t whose next token tokens[t+1] is scored (loss rows);
    action_targets: tokens[t+1] for those rows.
    """

    tokens: torch.Tensor
    positions: torch.Tensor
    cu_seqlens: torch.Tensor
    max_seqlen: int
    action_rows: torch.Tensor
    action_targets: torch.Tensor
    seq_index: Optional[torch.Tensor] = None  # sequence id of each action row
    attn_tiles: Optional[torch.Tensor] = None  # int32 [n, 2] (sequence, 128-row q tile), heaviest first
    attn_kv_tiles: Optional[torch.Tensor] = None  # int32 [n, 2] (sequence, 128-row kv tile), heaviest first

    def to(self, device, non_blocking: bool = True) -> "PackedBatch":
        mv = lambda t: None if t is None else t.to(device, non_blocking=non_blocking)  # noqa: E731
        return PackedBatch(mv(self.tokens), mv(self.positions), mv(self.cu_seqlens), self.max_seqlen,
                           mv(self.action_rows), mv(self.action_targets), mv(self.seq_index), mv(self.attn_tiles),
                           mv(self.attn_kv_tiles))

    @property
    def tiles(self):
        return (self.attn_tiles, self.attn_kv_tiles)

    @property
    def num_tokens(self) -> int:
        return int(self.tokens.numel())


def pack_sequences(seqs: List[torch.Tensor], masks: Optional[List[torch.Tensor]] = None,
                   pin: bool = False, pad_multiple: int = 1) -> PackedBatch:
    """Pack 1-D token tensors; ``masks[i][t] = 1`` marks tokens[t] as an action token
    (its logprob is computed from the row t-1).  ``pad_multiple > 1`` appends
    one padding sequence (token 0, no action rows) so the token count is a
    multiple of it (sequence parallelism splits the rows evenly)."""
    total = sum(int(s.numel()) for s in seqs)
    if pad_multiple > 1 and total % pad_multiple:
        pad = pad_multiple - total % pad_multiple
        seqs = list(seqs) + [torch.zeros(pad, dtype=torch.long)]
        if masks is not None:
            masks = list(masks) + [torch.zeros(pad, dtype=torch.bool)]
        else:
            masks = [torch.ones(int(s.numel()), dtype=torch.bool) for s in seqs[:-1]] + \
                [torch.zeros(pad, dtype=torch.bool)]
    lens = [int(s.numel()) for s in seqs]
    cu = torch.zeros(len(seqs) + 1, dtype=torch.int32)
    cu[1:] = torch.tensor(lens, dtype=torch.int32).cumsum(0)
    tokens = torch.cat([s.reshape(-1).long() for s in seqs]) if seqs else torch.zeros(0, dtype=torch.long)
    positions = torch.cat([torch.arange(n, dtype=torch.int32) for n in lens]) if seqs else torch.zeros(0, dtype=torch.int32)
    rows, targets, sidx = [], [], []
    for i, s in enumerate(seqs):
        start = int(cu[i])
        m = masks[i].reshape(-1) if masks is not None else torch.ones(lens[i], dtype=torch.bool)
        idx = torch.nonzero(m[1:].bool(), as_tuple=False).reshape(-1)  # positions t+1 that are actions
        rows.append(idx + start)
        targets.append(s.reshape(-1)[idx + 1].long())
        sidx.append(torch.full((idx.numel(),), i, dtype=torch.int32))
    action_rows = torch.cat(rows) if rows else torch.zeros(0, dtype=torch.long)
    action_targets = torch.cat(targets) if targets else torch.zeros(0, dtype=torch.long)
    seq_index = torch.cat(sidx) if sidx else torch.zeros(0, dtype=torch.int32)
    from libra_b200.ops.attention import attn_tiles

    cul = cu.tolist()
    batch = PackedBatch(tokens, positions, cu, max(lens) if lens else 0, action_rows.long(), action_targets, seq_index,
                        attn_tiles(cul, causal=True), attn_tiles(cul, causal=True, kv=True))
    if pin:
        batch = PackedBatch(*(t.pin_memory() if isinstance(t, torch.Tensor) else t for t in
                              (batch.tokens, batch.positions, batch.cu_seqlens, batch.max_seqlen, batch.action_rows,
                               batch.action_targets, batch.seq_index, batch.attn_tiles, batch.attn_kv_tiles)))
    return batch


# ---------------------------------------------------------------------------
# model
# ---------------------------------------------------------------------------

class Qwen3Model(nn.Module):
    """Stateless-compute model over externally owned parameter views.

    ``params`` maps canonical names to tensors (views into a flat buffer); the
    module never allocates parameters itself, which lets the engine place them
    in a flat buffer or in peer-visible memory.
    """

    def __init__(self, cfg: Qwen3Config, params: Dict[str, torch.Tensor], recompute: bool = False,
                 tp_group=None, tp_size: int = 1, tp_rank: int = 0, ep_group=None, ep_size: int = 1,
                 ep_exchange=None, sequence_parallel: bool = False):
        super().__init__()
        self.cfg = cfg
        self.p = params
        self.recompute = recompute
        self.tp_group, self.tp_size, self.tp_rank = tp_group, tp_size, tp_rank
        # sequence parallelism: the residual stream holds T / tp token rows per rank (the packed batch's
        # token count must divide evenly: pack with pad_multiple = sp_multiple(tp, device))
        self.sp = bool(sequence_parallel) and tp_size > 1 and not cfg.is_moe
        # expert parallelism: this rank holds num_experts / ep_size experts; tokens travel to their
        # experts' owners through ``ep_exchange`` (peer-memory kernels) or all-to-all over ``ep_group``
        self.ep_group, self.ep_size, self.ep_exchange = ep_group, ep_size, ep_exchange
        dev = next(iter(params.values())).device
        cos, sin = ops.ref.rope_tables(cfg.max_position_embeddings, cfg.head_dim, cfg.rope_theta, dev)
        self.register_buffer("rope_cos", cos, persistent=False)
        self.register_buffer("rope_sin", sin, persistent=False)
        self.nq_local = cfg.num_attention_heads // tp_size
        self.nkv_local = max(1, cfg.num_key_value_heads // tp_size)

    # -- blocks ------------------------------------------------------------
    def _attention_block(self, i: int, x, pos, cu, max_len, tiles=None):
        p, cfg = self.p, self.cfg
        pre = f"layers.{i}."
        if self.sp:
            from libra_b200.parallel.sequence_parallel import sp_column_parallel_linear

            qkv = sp_column_parallel_linear(ops.rmsnorm(x, p[pre + "input_layernorm"], cfg.rms_norm_eps),
                                            p[pre + "qkv_proj"], self.tp_group)
        else:
            h = self._tp_in(ops.rmsnorm(x, p[pre + "input_layernorm"], cfg.rms_norm_eps))
            qkv = ops.linear(h, p[pre + "qkv_proj"])
        q, k, v = ops.qk_norm_rope(qkv, p[pre + "q_norm"], p[pre + "k_norm"], pos, self.rope_cos, self.rope_sin,
                                   self.nq_local, self.nkv_local, cfg.rms_norm_eps)
        attn = ops.varlen_causal_attention(q, k, v, cu, max_len, tiles=tiles)
        return self._row_parallel(attn.reshape(attn.shape[0], -1), p[pre + "o_proj"], x)

    def _mlp_block(self, i: int, x):
        p, cfg = self.p, self.cfg
        pre = f"layers.{i}."
        h = ops.rmsnorm(x, p[pre + "post_attention_layernorm"], cfg.rms_norm_eps)
        if cfg.is_moe:
            if self.ep_size > 1:
                from libra_b200.parallel.expert_parallel import ep_moe_mlp

                return ep_moe_mlp(h, x, p[pre + "router"], p[pre + "experts.w1"], p[pre + "experts.w2"], cfg,
                                  self.ep_group, self.ep_exchange)
            from libra_b200.models.moe import moe_mlp

            return moe_mlp(h, x, p[pre + "router"], p[pre + "experts.w1"], p[pre + "experts.w2"], cfg)
        if self.sp:
            from libra_b200.parallel.sequence_parallel import sp_gather

            a = ops.linear_swiglu(sp_gather(h, self.tp_group), p[pre + "gate_up_proj"])
        else:
            a = ops.linear_swiglu(self._tp_in(h), p[pre + "gate_up_proj"])
        return self._row_parallel(a, p[pre + "down_proj"], x)

    def _tp_in(self, h):
        """Replicated input of a column-parallel linear (gradient all-reduced over TP)."""
        if self.tp_size == 1:
            return h
        from libra_b200.parallel.tensor_parallel import copy_to_tp

        return copy_to_tp(h, self.tp_group)

    def _row_parallel(self, a, w, residual):
        if self.tp_size == 1:
            return ops.linear(a, w, residual=residual)
        if self.sp:
            from libra_b200.parallel.sequence_parallel import sp_row_parallel_linear

            return sp_row_parallel_linear(a, w, residual, self.tp_group)
        from libra_b200.parallel.tensor_parallel import row_parallel_linear

        return row_parallel_linear(a, w, residual, self.tp_group)

    def _layer(self, i, x, pos, cu, max_len, tiles=None):
        x = self._attention_block(i, x, pos, cu, max_len, tiles)
        return self._mlp_block(i, x)

    # -- public ------------------------------------------------------------
    def embed(self, tokens):
        w = self.p["embed_tokens"]
        if self.tp_size == 1:
            return _Embedding.apply(tokens, w)
        from libra_b200.parallel.tensor_parallel import vocab_parallel_embedding

        return vocab_parallel_embedding(tokens, w, self.tp_group, self.tp_rank)

    def hidden_states(self, batch: PackedBatch) -> torch.Tensor:
        if self.sp:
            from libra_b200.parallel.sequence_parallel import sp_scatter
            from libra_b200.parallel.tensor_parallel import vocab_parallel_embedding

            if batch.num_tokens % self.tp_size:
                raise ValueError(f"sequence parallelism needs a token count divisible by tp={self.tp_size} "
                                 f"(pack with pad_multiple); got {batch.num_tokens}")
            # per-rank partial embedding (its vocab shard), reduce-scattered into this rank's token rows
            x = sp_scatter(vocab_parallel_embedding(batch.tokens, self.p["embed_tokens"], self.tp_group,
                                                    self.tp_rank, reduce=False), self.tp_group)
        else:
            x = self.embed(batch.tokens)
        for i in range(self.cfg.num_hidden_layers):
            if self.recompute and torch.is_grad_enabled():
                x = torch.utils.checkpoint.checkpoint(self._layer, i, x, batch.positions, batch.cu_seqlens,
                                                      batch.max_seqlen, batch.tiles, use_reentrant=False)
            else:
                x = self._layer(i, x, batch.positions, batch.cu_seqlens, batch.max_seqlen, batch.tiles)
        h = ops.rmsnorm(x, self.p["norm"], self.cfg.rms_norm_eps)
        if self.sp:
            from libra_b200.parallel.sequence_parallel import sp_gather_to_replicated

            # every rank scores its vocab shard for all rows; the vocab-parallel logprob hands back the
            # complete row gradient on every rank
            h = sp_gather_to_replicated(h, self.tp_group)
        return h

    @property
    def lm_head_weight(self):
        return self.p["embed_tokens"] if self.cfg.tie_word_embeddings else self.p["lm_head"]

    def action_logprobs(self, batch: PackedBatch, temperature: float = 1.0, entropy_out=None) -> torch.Tensor:
        """Logprob of every action token (rows ``batch.action_rows``)."""
        h = self.hidden_states(batch)
        rows = h.index_select(0, batch.action_rows)
        if self.tp_size == 1:
            return ops.lm_head_logprob(rows, self.lm_head_weight, batch.action_targets, temperature, entropy_out)
        from libra_b200.parallel.tensor_parallel import vocab_parallel_logprob

        return vocab_parallel_logprob(rows, self.lm_head_weight, batch.action_targets, temperature, self.tp_group,
                                      self.tp_rank, entropy_out)

    def logits(self, batch: PackedBatch) -> torch.Tensor:
        """Full logits [T, V] (inference/sampling helper)."""
        h = self.hidden_states(batch)
        return ops.linear(h, self.lm_head_weight)


class _Embedding(torch.autograd.Function):
    @staticmethod
    def forward(ctx, tokens, w):
        ctx.save_for_backward(tokens)
        ctx.wref = w
        return w.index_select(0, tokens)

    @staticmethod
    def backward(ctx, g):
        (tokens,) = ctx.saved_tensors
        w = ctx.wref
        main = getattr(w, "main_grad", None)
        if main is not None:
            main.index_add_(0, tokens, g.float())
            return None, None
        out = torch.zeros(w.shape, dtype=torch.float32, device=w.device)
        out.index_add_(0, tokens, g.float())
        return None, out.to(w.dtype)


def config_from_arch(arch) -> Qwen3Config:
    """Build a model config from the planner's ``ModelArchConfig`` section."""
    return Qwen3Config(
        vocab_size=int(arch.vocab_size), hidden_size=int(arch.d_model), intermediate_size=int(arch.intermediate_size),
        num_hidden_layers=int(arch.n_layers), num_attention_heads=int(arch.n_heads),
        num_key_value_heads=int(arch.n_kv_heads), head_dim=int(arch.head_dim),
        tie_word_embeddings=float(arch.num_params) < 8e9 and not arch.is_moe,
        num_experts=int(arch.num_experts) if arch.is_moe else 0,
        num_experts_per_tok=int(arch.num_activated_experts),
        moe_intermediate_size=int(arch.expert_intermediate_size),
    )
