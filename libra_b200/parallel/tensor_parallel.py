"""Tensor-parallel building blocks (Megatron-style, without sequence parallelism).

Reference: own TP layers ``engine/qwen3d_modules.py:149-269`` and the MCore
path.  Column-parallel linears (QKV, gate/up, expert w1) take a replicated
input through ``copy_to_tp`` (identity forward, all-reduce of the input
gradient backward); row-parallel linears (o-proj, down) all-reduce their
partial outputs (``reduce_from_tp``, identity backward) before the residual
add.  The embedding and LM head are split over the vocabulary; the token
logprob combines per-shard (max, sum-exp, target logit) statistics with three
tiny all-reduces instead of gathering [rows, V] logits (reference
``engine/megatron_core_train_engine.py:905-948``).

On CUDA the local math runs through the tcgen05 GEMM and the fused logprob
kernel (vocab offset = shard start); on CPU through torch (gloo tests).
"""

from __future__ import annotations

import torch
import torch.distributed as dist

from libra_b200 import ops


def _ws(group) -> int:
    return dist.get_world_size(group) if dist.is_initialized() else 1


def _rank(group) -> int:
    return dist.get_rank(group) if dist.is_initialized() else 0


class _CopyToTP(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, group):
        ctx.group = group
        return x

    @staticmethod
    def backward(ctx, g):
        g = g.contiguous()
        if _ws(ctx.group) > 1:
            dist.all_reduce(g, group=ctx.group)
        return g, None


class _ReduceFromTP(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, group):
        x = x.contiguous()
        if _ws(group) > 1:
            dist.all_reduce(x, group=group)
        return x

    @staticmethod
    def backward(ctx, g):
        return g, None


def copy_to_tp(x, group):
    return _CopyToTP.apply(x, group)


def reduce_from_tp(x, group):
    return _ReduceFromTP.apply(x, group)


def row_parallel_linear(a, w_local, residual, group):
    """residual + all_reduce(a_local @ w_local^T) with autograd.

    On CUDA with peer buffers registered for the group
    (``peer_gemm.enable_fused_row_parallel``) this is one fused GEMM +
    peer-memory all-reduce kernel; otherwise our GEMM followed by NCCL."""
    if _ws(group) > 1 and a.is_cuda:
        from libra_b200.parallel.peer_gemm import fused_for, row_parallel_fused

        fused = fused_for(group, w_local.shape[0], a.numel() // a.shape[-1])
        if fused is not None:
            return row_parallel_fused(a, w_local, residual, fused)
    y = reduce_from_tp(ops.linear(a, w_local), group)
    return y + residual if residual is not None else y


@torch.no_grad()
def row_parallel_linear_allreduce(a, w_local, residual, group):
    """Inference version (rollout): no autograd bookkeeping."""
    y = ops.linear(a, w_local).contiguous()
    if _ws(group) > 1:
        dist.all_reduce(y, group=group)
    return y + residual if residual is not None else y


class _VocabParallelEmbedding(torch.autograd.Function):
    @staticmethod
    def forward(ctx, tokens, w_local, group, rank, reduce=True):
        V_l = w_local.shape[0]
        lo = rank * V_l
        local = (tokens >= lo) & (tokens < lo + V_l)
        idx = torch.where(local, tokens - lo, torch.zeros_like(tokens))
        out = w_local.index_select(0, idx) * local.unsqueeze(-1).to(w_local.dtype)
        out = out.contiguous()
        if reduce and _ws(group) > 1:
            dist.all_reduce(out, group=group)
        ctx.save_for_backward(idx, local)
        ctx.wref = w_local
        return out

    @staticmethod
    def backward(ctx, g):
        idx, local = ctx.saved_tensors
        w = ctx.wref
        gl = g.float() * local.unsqueeze(-1).float()
        main = getattr(w, "main_grad", None)
        if main is not None:
            main.index_add_(0, idx, gl)
            return None, None, None, None, None
        out = torch.zeros(w.shape, dtype=torch.float32, device=w.device)
        out.index_add_(0, idx, gl)
        return None, out.to(w.dtype), None, None, None


def vocab_parallel_embedding(tokens, w_local, group, rank, reduce: bool = True):
    """Embedding rows of this rank's vocab shard (zero elsewhere), summed over
    the group (``reduce``) or left partial for a reduce-scatter."""
    return _VocabParallelEmbedding.apply(tokens, w_local, group, rank, reduce)


class PeerLogprobExchange:
    """The vocab-parallel log-softmax's per-row (max, sum-exp, target logit)
    exchange in one kernel over NVLink peer memory (``vocab_stats_exchange`` in
    ``ops/csrc/vocab_exchange.cu``) instead of two NCCL all-reduces.  Each rank
    of the TP group maps every rank's exchange area (CUDA IPC); calls are
    collective and in the same order on every rank."""

    MAX_RANKS, MAX_CTAS = 8, 256

    def __init__(self, group, max_rows: int, device):
        from libra_b200.parallel.peer_grad_reduce import map_peer_tensors

        self.group = group
        self.n, self.me = _ws(group), _rank(group)
        if self.n > self.MAX_RANKS:
            raise ValueError(f"at most {self.MAX_RANKS} ranks")
        self.max_rows = int(max_rows)
        self.data = torch.zeros(2 * self.MAX_RANKS * self.max_rows * 4, dtype=torch.float32, device=device)
        self.flags = torch.zeros(self.MAX_CTAS * self.MAX_RANKS, dtype=torch.int32, device=device)
        (self.data_ptrs, self.flag_ptrs), self._opened = map_peer_tensors(group, [self.data, self.flags], self.n,
                                                                          self.me)
        self.calls = 0
        if self.n > 1:
            torch.cuda.synchronize(device)
            dist.barrier(group=group)

    def close(self) -> None:
        for b in self._opened:
            ops.ext().ipc_close(b)
        self._opened = []

    def __call__(self, stats_m, stats_s, zt):
        lse, z = ops.ext().vocab_stats_exchange(self.data_ptrs, self.flag_ptrs, self.me, self.max_rows,
                                                stats_m.float().contiguous(), stats_s.float().contiguous(),
                                                zt.float().contiguous(), self.calls + 1, ops.error_flag(zt.device))
        self.calls += 1
        return lse, z


_LOGPROB_EXCHANGE: dict = {}


def enable_peer_logprob_exchange(group, max_rows: int, device) -> None:
    """Collective over the TP group: route the vocab-parallel logprob's shard
    statistics through the peer-memory exchange for up to ``max_rows`` rows."""
    if id(group) not in _LOGPROB_EXCHANGE:
        _LOGPROB_EXCHANGE[id(group)] = PeerLogprobExchange(group, max_rows, device)


def disable_peer_logprob_exchange() -> None:
    for x in _LOGPROB_EXCHANGE.values():
        x.close()
    _LOGPROB_EXCHANGE.clear()


def _combine(stats_m, stats_s, zt, group):
    """Global (lse, target logit) from per-shard (max, sum-exp, target logit)."""
    x = _LOGPROB_EXCHANGE.get(id(group)) if stats_m.is_cuda else None
    if x is not None and stats_m.numel() <= x.max_rows:
        return x(stats_m, stats_s, zt)
    M = stats_m.clone()
    if _ws(group) > 1:
        dist.all_reduce(M, op=dist.ReduceOp.MAX, group=group)
    S = stats_s * torch.exp(stats_m - M)
    both = torch.stack([S, zt])
    if _ws(group) > 1:
        dist.all_reduce(both, group=group)
    return M + torch.log(both[0]), both[1]


class _VocabParallelLogprob(torch.autograd.Function):
    @staticmethod
    def forward(ctx, h, w_local, targets, temperature, group, rank, entropy_out):
        V_l = w_local.shape[0]
        v0 = rank * V_l
        inv_t = 1.0 / temperature
        if h.is_cuda:
            logits = ops.gemm(h, w_local)
            _, ent, stats, zt = ops.ext().logprob_fwd(logits, targets, v0, temperature, entropy_out is not None)
            m, s = stats[:, 0].contiguous(), stats[:, 1].contiguous()
        else:
            logits = torch.nn.functional.linear(h.float(), w_local.float())
            z = logits * inv_t
            m = z.max(-1).values
            s = torch.exp(z - m[:, None]).sum(-1)
            tl = targets - v0
            ok = (tl >= 0) & (tl < V_l)
            zt = torch.where(ok, z.gather(-1, tl.clamp(0, V_l - 1)[:, None]).squeeze(-1), torch.zeros_like(m))
            ent = None
        lse, zt_g = _combine(m, s, zt.float(), group)
        if entropy_out is not None:
            z = (logits.float() * inv_t)
            t_local = (torch.exp(z - m[:, None]) * z).sum(-1)
            T = t_local * torch.exp(m - lse)  # this shard's part of E[z]
            if _ws(group) > 1:
                dist.all_reduce(T, group=group)
            entropy_out.copy_(lse - T)
        ctx.save_for_backward(h, w_local, targets, lse)
        ctx.logits = logits
        ctx.v0, ctx.temperature, ctx.group = v0, temperature, group
        return zt_g - lse

    @staticmethod
    def backward(ctx, g):
        h, w, targets, lse = ctx.saved_tensors
        logits, v0, temp = ctx.logits, ctx.v0, ctx.temperature
        g = g.contiguous().float()
        main = getattr(w, "main_grad", None)
        if h.is_cuda:
            ops.ext().logprob_bwd_(logits, targets, v0, temp, lse.contiguous(), g)
            dh = ops.gemm(logits, w, b_mn=True)
            if main is not None:
                ops.gemm(logits, h, a_mn=True, b_mn=True, out=main, epi=ops.EPI_ACC_F32)
                dw = None
            else:
                dw = torch.zeros(w.shape, dtype=torch.float32, device=w.device)
                ops.gemm(logits, h, a_mn=True, b_mn=True, out=dw, epi=ops.EPI_ACC_F32)
                dw = dw.to(w.dtype)
        else:
            V_l = w.shape[0]
            p = torch.exp(logits / temp - lse[:, None])
            tl = targets - v0
            onehot = torch.zeros_like(p)
            ok = (tl >= 0) & (tl < V_l)
            onehot[ok, tl[ok]] = 1.0
            dz = g[:, None] * (onehot - p) / temp
            dh = dz @ w.float()
            dwf = dz.t() @ h.float()
            if main is not None:
                main.add_(dwf)
                dw = None
            else:
                dw = dwf.to(w.dtype)
            dh = dh.to(h.dtype)
        dh = dh.contiguous()
        if _ws(ctx.group) > 1:
            dist.all_reduce(dh, group=ctx.group)
        return dh, dw, None, None, None, None, None


def vocab_parallel_logprob(h, w_local, targets, temperature, group, rank, entropy_out=None):
    """Token logprobs under a vocab-sharded LM head (h replicated over the TP group)."""
    return _VocabParallelLogprob.apply(h.contiguous(), w_local, targets.contiguous(), float(temperature), group, rank,
                                       entropy_out)


@torch.no_grad()
def gather_vocab_logits(logits_local, group):
    """[rows, V/tp] shards -> [rows, V] on every rank (rollout sampling)."""
    n = _ws(group)
    if n == 1:
        return logits_local
    parts = [torch.empty_like(logits_local) for _ in range(n)]
    dist.all_gather(parts, logits_local.contiguous(), group=group)
    return torch.cat(parts, dim=-1)


def shard_full_params(full: dict, cfg, tp_size: int, tp_rank: int) -> dict:
    """Slice full (TP=1) parameters into one TP rank's local shards.

    QKV rows are taken per head group: this rank's q heads, then its k and v
    heads; gate/up keeps the [gate; up] halves; expert w1 likewise per expert.
    """
    if tp_size == 1:
        return dict(full)
    H, D = cfg.hidden_size, cfg.head_dim
    nq, nkv = cfg.num_attention_heads, cfg.num_key_value_heads
    nq_l, kv_l = nq // tp_size, max(1, nkv // tp_size)
    kv0 = tp_rank * nkv // tp_size  # with tp > nkv, neighbouring ranks share (replicate) a kv head
    out = {}
    for name, t in full.items():
        if name.endswith("qkv_proj"):
            q = t[:nq * D].view(nq, D, H)[tp_rank * nq_l:(tp_rank + 1) * nq_l].reshape(-1, H)
            k = t[nq * D:(nq + nkv) * D].view(nkv, D, H)[kv0:kv0 + kv_l].reshape(-1, H)
            v = t[(nq + nkv) * D:].view(nkv, D, H)[kv0:kv0 + kv_l].reshape(-1, H)
            out[name] = torch.cat([q, k, v])
        elif name.endswith("o_proj"):
            out[name] = t[:, tp_rank * nq_l * D:(tp_rank + 1) * nq_l * D]
        elif name.endswith("gate_up_proj"):
            F = t.shape[0] // 2
            Fl = F // tp_size
            out[name] = torch.cat([t[tp_rank * Fl:(tp_rank + 1) * Fl], t[F + tp_rank * Fl:F + (tp_rank + 1) * Fl]])
        elif name.endswith("down_proj"):
            Fl = t.shape[1] // tp_size
            out[name] = t[:, tp_rank * Fl:(tp_rank + 1) * Fl]
        elif name.endswith("experts.w1"):
            F = t.shape[1] // 2
            Fl = F // tp_size
            out[name] = torch.cat([t[:, tp_rank * Fl:(tp_rank + 1) * Fl], t[:, F + tp_rank * Fl:F + (tp_rank + 1) * Fl]],
                                  dim=1)
        elif name.endswith("experts.w2"):
            Fl = t.shape[2] // tp_size
            out[name] = t[:, :, tp_rank * Fl:(tp_rank + 1) * Fl]
        elif name in ("embed_tokens", "lm_head"):
            Vl = t.shape[0] // tp_size
            out[name] = t[tp_rank * Vl:(tp_rank + 1) * Vl]
        else:
            out[name] = t
    return {k: v.contiguous() for k, v in out.items()}


def merge_tp_shards(parts: list, cfg, tp_size: int) -> dict:
    """Inverse of ``shard_full_params``: full (TP=1) tensors from the TP ranks'
    local dicts (``parts[r]`` = rank r's).  KV heads replicated over several
    ranks (tp > kv heads) are taken once."""
    if tp_size == 1:
        return dict(parts[0])
    D = cfg.head_dim
    nq, nkv = cfg.num_attention_heads, cfg.num_key_value_heads
    nq_l, kv_l = nq // tp_size, max(1, nkv // tp_size)
    owners = []  # first rank holding each kv group
    for r in range(tp_size):
        kv0 = r * nkv // tp_size
        if not owners or owners[-1][0] != kv0:
            owners.append((kv0, r))
    out = {}
    for name in parts[0]:
        ts = [p[name] for p in parts]
        if name.endswith("qkv_proj"):
            q = torch.cat([t[:nq_l * D] for t in ts])
            k = torch.cat([ts[r][nq_l * D:(nq_l + kv_l) * D] for _, r in owners])
            v = torch.cat([ts[r][(nq_l + kv_l) * D:] for _, r in owners])
            out[name] = torch.cat([q, k, v])
        elif name.endswith("o_proj") or name.endswith("down_proj"):
            out[name] = torch.cat(ts, dim=1)
        elif name.endswith("gate_up_proj"):
            F = ts[0].shape[0] // 2
            out[name] = torch.cat([t[:F] for t in ts] + [t[F:] for t in ts])
        elif name.endswith("experts.w1"):
            F = ts[0].shape[1] // 2
            out[name] = torch.cat([t[:, :F] for t in ts] + [t[:, F:] for t in ts], dim=1)
        elif name.endswith("experts.w2"):
            out[name] = torch.cat(ts, dim=2)
        elif name in ("embed_tokens", "lm_head"):
            out[name] = torch.cat(ts)
        else:
            out[name] = ts[0]  # replicated
    return out


def tp_partial_grad_params(names, sequence_parallel: bool = False) -> list:
    """Replicated parameters whose gradient differs per TP rank and must be
    all-reduced over the TP group: the per-head q/k norms (local heads only)
    and, with sequence parallelism, every RMSNorm weight of the residual stream
    (local token rows only)."""
    out = [n for n in names if n.endswith("q_norm") or n.endswith("k_norm")]
    if sequence_parallel:
        out += [n for n in names if n == "norm" or n.endswith("layernorm")]
    return out
