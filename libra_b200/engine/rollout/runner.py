"""Forward pass of the rollout engine over a paged KV cache.

One ``step`` runs a mixed batch: sequences that append several tokens
(prefill of a new prompt, or the tool-return tokens of the next turn of an
agentic episode) and sequences that decode one token.  All new tokens are
packed into one stream, so the GEMMs (tcgen05 kernel) see every token of the
step at once; attention is split:

* decode rows -> ``paged_decode_attention`` (sm_100a kernel, KV read in place);
* extend rows -> causal varlen attention (tcgen05 flash kernel) with the
  queries aligned to the end of each sequence's key range.  The gather plan is
  built once per step (``_ExtendPlan``): when every extending sequence is a
  fresh prefill its keys are this step's K/V rows and nothing is copied from
  the cache; otherwise one flat slot index gathers every sequence's whole key
  range from the paged pool with one ``index_select`` per layer.
* CPU tensors use the fp32 reference for both.

Only the last position of each sequence goes through the final norm and the
LM head.  Weights are the training engine's parameter views when rollout and
training share a process (zero-copy weight updates), or this instance's own
buffer otherwise.
"""

from __future__ import annotations

import math
from dataclasses import dataclass
from typing import Dict, List, Optional, Sequence

import torch

from libra_b200 import ops
from libra_b200.engine.rollout.kv_cache import PagedKVCache
from libra_b200.models.qwen3 import Qwen3Config


@dataclass
class WorkItem:
    seq_id: str
    tokens: List[int]   # full token list of the sequence after this step's tokens are appended
    start: int          # number of tokens whose KV is already in the cache


def _extend_attention_ref(q, k, v, q_start: int):
    """q [n, Hq, D] at positions q_start..; k/v [L, Hkv, D] (positions 0..L-1)."""
    n, hq, d = q.shape
    L, hkv = k.shape[0], k.shape[1]
    kk = k.float().transpose(0, 1).repeat_interleave(hq // hkv, 0)
    vv = v.float().transpose(0, 1).repeat_interleave(hq // hkv, 0)
    s = (q.float().transpose(0, 1) @ kk.transpose(-1, -2)) / math.sqrt(d)
    qpos = torch.arange(q_start, q_start + n, device=q.device).unsqueeze(1)
    kpos = torch.arange(L, device=q.device).unsqueeze(0)
    s = s.masked_fill(kpos > qpos, float("-inf"))
    return (s.softmax(-1) @ vv).transpose(0, 1).to(q.dtype)


def _to_device(values: List[int], dtype, device) -> torch.Tensor:
    """Small host list -> device tensor without a stream synchronisation (a
    pinned staging copy on CUDA)."""
    t = torch.tensor(values, dtype=dtype)
    if torch.device(device).type == "cuda":
        return t.pin_memory().to(device, non_blocking=True)
    return t


@dataclass
class _ExtendPlan:
    """How one step's extend attention finds its queries and keys.

    ``items`` are the indices of the work items with more than one new token.
    Their queries are rows ``q_rows`` of the step's token stream, or the
    leading ``n_q`` rows when ``q_rows`` is None.  Keys come from this step's
    K/V at the query rows when ``key_slots`` is None (every such item starts at
    position 0), else from the paged cache at the flat slots ``key_slots`` (the
    whole range 0..len of each item, in item order)."""

    items: List[int]
    n_q: int
    q_rows: Optional[torch.Tensor]
    key_slots: Optional[torch.Tensor]
    cu_q: List[int]
    cu_k: List[int]
    cu_q_dev: Optional[torch.Tensor] = None
    cu_k_dev: Optional[torch.Tensor] = None
    tiles: Optional[torch.Tensor] = None

    def queries(self, q: torch.Tensor) -> torch.Tensor:
        return q[:self.n_q] if self.q_rows is None else q.index_select(0, self.q_rows)

    def keys(self, kv: PagedKVCache, layer: int, k: torch.Tensor, v: torch.Tensor):
        if self.key_slots is None:
            return self.queries(k), self.queries(v)
        kf = kv.k[layer].view(-1, kv.kv_heads, kv.head_dim)
        vf = kv.v[layer].view(-1, kv.kv_heads, kv.head_dim)
        return kf.index_select(0, self.key_slots), vf.index_select(0, self.key_slots)


def build_extend_plan(items: Sequence[WorkItem], offsets: List[int], kv: PagedKVCache, device) -> Optional[_ExtendPlan]:
    """The extend-attention gather plan of one step (host work once per step,
    not once per layer)."""
    ext = [i for i, it in enumerate(items) if len(it.tokens) - it.start > 1]
    if not ext:
        return None
    cu_q, cu_k, rows = [0], [0], []
    for i in ext:
        it = items[i]
        n_new = len(it.tokens) - it.start
        cu_q.append(cu_q[-1] + n_new)
        cu_k.append(cu_k[-1] + len(it.tokens))
        rows.extend(range(offsets[i], offsets[i] + n_new))
    n_q = cu_q[-1]
    contiguous = rows == list(range(n_q))
    q_rows = None if contiguous else _to_device(rows, torch.long, device)
    fresh = all(items[i].start == 0 for i in ext)
    key_slots = None
    if not fresh:
        key_slots = torch.cat([kv.slot_mapping(items[i].seq_id, 0, len(items[i].tokens)) for i in ext])
        key_slots = key_slots.to(device, non_blocking=True)
    plan = _ExtendPlan(ext, n_q, q_rows, key_slots, cu_q, cu_k)
    if torch.device(device).type == "cuda":
        from libra_b200.ops.attention import attn_tiles

        plan.cu_q_dev = _to_device(cu_q, torch.int32, device)
        plan.cu_k_dev = _to_device(cu_k, torch.int32, device)
        plan.tiles = attn_tiles(cu_q, True, device)
    return plan


class InferenceRunner:
    def __init__(self, cfg: Qwen3Config, params: Dict[str, torch.Tensor], kv_cache: PagedKVCache,
                 tp_group=None, tp_size: int = 1, max_step_tokens: int = 0):
        self.cfg, self.p, self.kv = cfg, params, kv_cache
        self.device = next(iter(params.values())).device
        self.tp_group, self.tp_size = tp_group, tp_size
        self.peer_ar = self._make_peer_allreduce(max_step_tokens)
        self.nq = cfg.num_attention_heads // tp_size
        self.nkv = max(1, cfg.num_key_value_heads // tp_size)
        cos, sin = ops.ref.rope_tables(cfg.max_position_embeddings, cfg.head_dim, cfg.rope_theta, self.device)
        self.cos, self.sin = cos, sin
        self.scale = 1.0 / math.sqrt(cfg.head_dim)

    def _make_peer_allreduce(self, max_rows: int):
        """Tensor-parallel ranks on NCCL (one box) reduce the row-parallel GEMM
        outputs over NVLink peer memory, fused with the residual add and the
        next RMSNorm (``PeerAllReduce``).  ``LIBRA_TP_PEER_AR=0`` keeps the NCCL
        all-reduce; gloo ranks and mixture-of-experts layers always do."""
        import os

        import torch.distributed as dist

        if (self.tp_size <= 1 or self.device.type != "cuda" or self.cfg.is_moe or max_rows <= 0
                or os.environ.get("LIBRA_TP_PEER_AR", "1") == "0"
                or dist.get_backend(self.tp_group) != "nccl"):
            return None
        from libra_b200.parallel.peer_allreduce import PeerAllReduce

        return PeerAllReduce(self.tp_group, max_rows, self.cfg.hidden_size, self.device)

    @property
    def lm_head(self):
        return self.p["embed_tokens"] if self.cfg.tie_word_embeddings else self.p["lm_head"]

    def _attention(self, layer: int, q, k, v, items: Sequence[WorkItem], offsets: List[int]):
        dev = q.device
        plan = self._ext_plan
        if plan is not None and plan.n_q == q.shape[0] and plan.q_rows is None:
            out = None  # every row extends: the kernel's output is the whole result
        else:
            out = torch.empty_like(q)
        dec = self._dec
        if dec:
            rows = self._dec_rows
            if dev.type == "cuda" and self.cfg.head_dim == 128:
                ids = [items[i].seq_id for i in dec]
                tbl = self._tables.get(tuple(ids))
                if tbl is None:
                    tbl = self.kv.block_table(ids, dev)
                    self._tables[tuple(ids)] = tbl
                lens = self._lens_dec
                o = ops.ext().paged_decode_attention(q.index_select(0, rows).contiguous(), self.kv.k[layer],
                                                     self.kv.v[layer], tbl, lens, self._max_len_dec, self.scale)
                out.index_copy_(0, rows, o)
            else:
                for i in dec:
                    kk, vv = self.kv.gather(layer, items[i].seq_id, len(items[i].tokens))
                    out[offsets[i]:offsets[i] + 1] = _extend_attention_ref(q[offsets[i]:offsets[i] + 1], kk, vv,
                                                                           len(items[i].tokens) - 1)
        if plan is None:
            return out
        qe = plan.queries(q)
        ke, ve = plan.keys(self.kv, layer, k, v)
        if dev.type == "cuda" and self.cfg.head_dim == 128:
            # queries are the new suffix of each sequence; keys span the whole (cached) prefix
            o, _ = ops.ext().flash_fwd(qe.contiguous(), ke.contiguous(), ve.contiguous(), plan.cu_q_dev,
                                       plan.tiles, self.scale, True, ops.error_flag(dev), plan.cu_k_dev)
        else:
            o = torch.empty_like(qe)
            for j, i in enumerate(plan.items):
                a, b, c, d = plan.cu_q[j], plan.cu_q[j + 1], plan.cu_k[j], plan.cu_k[j + 1]
                o[a:b] = _extend_attention_ref(qe[a:b], ke[c:d], ve[c:d], items[i].start)
        if out is None:
            return o
        if plan.q_rows is None:
            out[:plan.n_q] = o
        else:
            out.index_copy_(0, plan.q_rows, o)
        return out

    @torch.no_grad()
    def step(self, items: Sequence[WorkItem]) -> torch.Tensor:
        """Write KV for every new token and return last-position logits [B, V]."""
        cfg, p, dev = self.cfg, self.p, self.device
        toks, pos, slots, offsets = [], [], [], []
        off = 0
        for it in items:
            self.kv.reserve(it.seq_id, len(it.tokens))
            new = it.tokens[it.start:]
            offsets.append(off)
            toks.extend(new)
            pos.extend(range(it.start, len(it.tokens)))
            slots.append(self.kv.slot_mapping(it.seq_id, it.start, len(it.tokens)))
            off += len(new)
        tok_t = torch.tensor(toks, dtype=torch.long).to(dev, non_blocking=True)
        pos_t = torch.tensor(pos, dtype=torch.int32).to(dev, non_blocking=True)
        slot_t = torch.cat(slots).to(dev, non_blocking=True)
        last_rows = torch.tensor([o + len(it.tokens) - it.start - 1 for o, it in zip(offsets, items)],
                                 dtype=torch.long).to(dev, non_blocking=True)
        self._tables = {}
        self._ext_plan = build_extend_plan(items, offsets, self.kv, dev)
        # per-step host tables, copied once (asynchronously) rather than once per layer
        self._dec = [i for i, it in enumerate(items) if len(it.tokens) - it.start == 1]
        self._dec_rows = _to_device([offsets[i] for i in self._dec], torch.long, dev)
        self._lens_dec = _to_device([len(items[i].tokens) for i in self._dec], torch.int32, dev)
        self._max_len_dec = max((len(items[i].tokens) for i in self._dec), default=1)
        if self.tp_size > 1:
            from libra_b200.parallel.tensor_parallel import vocab_parallel_embedding
            import torch.distributed as dist

            x = vocab_parallel_embedding(tok_t, self.p["embed_tokens"], self.tp_group, dist.get_rank(self.tp_group))
        else:
            x = self.p["embed_tokens"].index_select(0, tok_t)
        peer = self.peer_ar if self.peer_ar is not None and x.shape[0] <= self.peer_ar.max_rows else None
        L = cfg.num_hidden_layers
        if peer is not None:
            # fused path: each row-parallel GEMM writes its partial into the peer buffer; one kernel sums
            # the TP partials over NVLink, adds the residual and applies the next RMSNorm
            h = ops.rmsnorm(x, p["layers.0.input_layernorm"], cfg.rms_norm_eps)
            for layer in range(L):
                pre = f"layers.{layer}."
                qkv = ops.linear(h, p[pre + "qkv_proj"])
                q, k, v = ops.qk_norm_rope(qkv, p[pre + "q_norm"], p[pre + "k_norm"], pos_t, self.cos, self.sin,
                                           self.nq, self.nkv, cfg.rms_norm_eps)
                self.kv.write(layer, slot_t, k, v)
                attn = self._attention(layer, q, k, v, items, offsets)
                ops.gemm(attn.reshape(attn.shape[0], -1), p[pre + "o_proj"], out=peer.partial(x.shape[0]))
                x, h = peer.reduce_add_rmsnorm(x, p[pre + "post_attention_layernorm"], cfg.rms_norm_eps)
                ops.gemm(ops.linear_swiglu(h, p[pre + "gate_up_proj"]), p[pre + "down_proj"],
                         out=peer.partial(x.shape[0]))
                nxt = p[f"layers.{layer + 1}.input_layernorm"] if layer + 1 < L else p["norm"]
                x, h = peer.reduce_add_rmsnorm(x, nxt, cfg.rms_norm_eps)
            last = h.index_select(0, last_rows)
            return self._finish_step(items, last)
        for layer in range(L):
            pre = f"layers.{layer}."
            h = ops.rmsnorm(x, p[pre + "input_layernorm"], cfg.rms_norm_eps)
            qkv = ops.linear(h, p[pre + "qkv_proj"])
            q, k, v = ops.qk_norm_rope(qkv, p[pre + "q_norm"], p[pre + "k_norm"], pos_t, self.cos, self.sin,
                                       self.nq, self.nkv, cfg.rms_norm_eps)
            self.kv.write(layer, slot_t, k, v)
            attn = self._attention(layer, q, k, v, items, offsets)
            x = self._row_parallel(attn.reshape(attn.shape[0], -1), p[pre + "o_proj"], x)
            h = ops.rmsnorm(x, p[pre + "post_attention_layernorm"], cfg.rms_norm_eps)
            if cfg.is_moe:
                from libra_b200.models.moe import moe_mlp

                x = moe_mlp(h, x, p[pre + "router"], p[pre + "experts.w1"], p[pre + "experts.w2"], cfg)
            else:
                x = self._row_parallel(ops.linear_swiglu(h, p[pre + "gate_up_proj"]), p[pre + "down_proj"], x)
        last = ops.rmsnorm(x.index_select(0, last_rows), p["norm"], cfg.rms_norm_eps)
        return self._finish_step(items, last)

    def _finish_step(self, items: Sequence[WorkItem], last: torch.Tensor) -> torch.Tensor:
        logits = ops.linear(last, self.lm_head)
        if self.tp_size > 1:
            from libra_b200.parallel.tensor_parallel import gather_vocab_logits

            logits = gather_vocab_logits(logits, self.tp_group)
        for it in items:
            self.kv.commit(it.seq_id, it.tokens)
        return logits

    def _row_parallel(self, a, w, residual):
        if self.tp_size == 1:
            return ops.linear(a, w, residual=residual)
        from libra_b200.parallel.tensor_parallel import row_parallel_linear_allreduce

        return row_parallel_linear_allreduce(a, w, residual, self.tp_group)
