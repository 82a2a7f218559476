"""Top-k routed expert MLP (Qwen3-MoE) for single-GPU / expert-replicated use.

Router: logits = h W_r^T in fp32, softmax over experts, top-k, renormalised over
the selected experts (``norm_topk_prob``), as in the Qwen3-MoE block the
reference trains through Megatron-Core's alltoall dispatcher and grouped GEMM
(engine/megatron_core_train_engine.py:299-308, engine/megatron_core_moe_mapping.py).

Expert weights are stored expert-major: ``w1`` [E, 2*Fe, H] (gate rows then up
rows) and ``w2`` [E, H, Fe]; that is the per-expert slicing of Megatron's
GroupedMLP ``weight1``/``weight2`` (reference
engine/megatron_core_moe_mapping.py:11-70) transposed to K-major rows so every
expert GEMM is a K-major tcgen05 GEMM.

The expert-parallel path (tokens dispatched to peers) lives in
``libra_b200.parallel.expert_parallel``; this module handles the local groups.
"""

from __future__ import annotations

import torch

from libra_b200 import ops


class GroupedLinear(torch.autograd.Function):
    """y[rows of group e] = x[rows of group e] W[e]^T for contiguous row groups."""

    @staticmethod
    def forward(ctx, x, w, counts_host, dest=None):
        E, N, _ = w.shape
        if dest is not None:
            # ``dest`` = (tensor,): caller-provided [rows, N] memory (e.g. a peer-visible send slot).  The
            # output aliases its storage without being an autograd view of it, so the gradient history
            # starts here rather than at the buffer the slot is carved from.
            d = dest[0]
            y = torch.empty(0, dtype=d.dtype, device=d.device).set_(d.untyped_storage(), d.storage_offset(),
                                                                     d.shape, d.stride())
        else:
            y = torch.empty(x.shape[0], N, dtype=x.dtype, device=x.device)
        s = 0
        for e in range(E):
            c = int(counts_host[e])
            if c:
                ops.gemm(x[s:s + c], w[e], out=y[s:s + c]) if x.is_cuda else y[s:s + c].copy_(
                    torch.nn.functional.linear(x[s:s + c].float(), w[e].float()))
            s += c
        ctx.save_for_backward(x, w)
        ctx.counts = list(int(c) for c in counts_host)
        return y

    @staticmethod
    def backward(ctx, dy):
        x, w = ctx.saved_tensors
        dy = dy.contiguous()
        dx = torch.empty_like(x)
        main = getattr(w, "main_grad", None)
        dw = None if main is not None else torch.zeros(w.shape, dtype=torch.float32, device=w.device)
        target = main if main is not None else dw
        s = 0
        for e, c in enumerate(ctx.counts):
            if c:
                if x.is_cuda:
                    ops.gemm(dy[s:s + c], w[e], b_mn=True, out=dx[s:s + c])
                    ops.gemm(dy[s:s + c], x[s:s + c], a_mn=True, b_mn=True, out=target[e], epi=ops.EPI_ACC_F32)
                else:
                    dx[s:s + c] = (dy[s:s + c].float() @ w[e].float()).to(dx.dtype)
                    target[e] += dy[s:s + c].float().t() @ x[s:s + c].float()
            s += c
        return dx, (None if main is not None else dw.to(w.dtype)), None, None


def route(h, router_w, top_k: int, normalize: bool = True):
    """Returns (weights [T, k] fp32, experts [T, k] int64, router probs [T, E])."""
    logits = torch.nn.functional.linear(h.float(), router_w.float())
    probs = logits.softmax(dim=-1)
    weights, experts = probs.topk(top_k, dim=-1)
    if normalize:
        weights = weights / weights.sum(-1, keepdim=True)
    return weights, experts, probs


GROUP_ALIGN = 128  # rows: every expert's group starts on a tensor-core tile boundary


def expert_layout(experts: torch.Tensor, num_experts: int, align: int = GROUP_ALIGN):
    """Padded grouped layout of the (token, k) assignments, computed on the device.

    Returns ``offs`` (int32 [E+1]: group e owns rows [offs[e], offs[e+1]), each
    start a multiple of ``align``) and ``rows`` (int64 [T*k]: the row of
    assignment j = t*k + kk).  Nothing is read back to the host: the counts come
    from a scatter-add, not a bincount whose size depends on the data."""
    flat = experts.reshape(-1)
    counts = torch.zeros(num_experts, dtype=torch.int64, device=flat.device)
    counts.scatter_add_(0, flat, torch.ones_like(flat))
    padded = (counts + align - 1) // align * align
    offs = torch.zeros(num_experts + 1, dtype=torch.int64, device=flat.device)
    offs[1:] = padded.cumsum(0)
    order = torch.argsort(flat, stable=True)
    g = flat[order]
    first = counts.cumsum(0) - counts
    rank = torch.arange(flat.numel(), device=flat.device) - first[g]
    rows = torch.empty_like(flat)
    rows[order] = offs[g] + rank
    return offs.to(torch.int32), rows


def grouped_capacity(tokens: int, k: int, num_groups: int, align: int = GROUP_ALIGN) -> int:
    """Rows that always hold the padded layout of ``tokens * k`` assignments over ``num_groups`` groups."""
    return tokens * k + (align - 1) * num_groups + align


def moe_mlp(h, residual, router_w, w1, w2, cfg):
    """residual + sum_k w_k * Expert_{e_k}(h), with every expert's rows in one
    padded buffer and both expert GEMMs as single grouped launches (no host
    synchronisation, no per-expert loop)."""
    T, H = h.shape
    E, k = cfg.num_experts, cfg.num_experts_per_tok
    weights, experts, _ = route(h, router_w, k, cfg.norm_topk_prob)
    offs, rows = expert_layout(experts, E)
    cap = grouped_capacity(T, k, E)
    xs = h.new_zeros(cap, H).index_copy(0, rows, h.repeat_interleave(k, dim=0))
    a = ops.grouped_swiglu(xs, w1, offs)
    ys = ops.grouped_linear(a, w2, offs)
    picked = ys.index_select(0, rows).view(T, k, H)
    out = (picked.float() * weights.unsqueeze(-1)).sum(1) + residual.float()
    return out.to(h.dtype)


def moe_mlp_looped(h, residual, router_w, w1, w2, cfg):
    """Per-expert loop with host-side counts: the oracle for ``moe_mlp``."""
    T, H = h.shape
    E, k = cfg.num_experts, cfg.num_experts_per_tok
    weights, experts, _ = route(h, router_w, k, cfg.norm_topk_prob)
    flat_e = experts.reshape(-1)
    order = torch.argsort(flat_e, stable=True)
    token_of = order // k
    counts = torch.bincount(flat_e, minlength=E).cpu()
    xs = h.index_select(0, token_of)
    gu = GroupedLinear.apply(xs, w1, counts)
    a = ops.swiglu(gu)
    ys = GroupedLinear.apply(a, w2, counts)
    wsel = weights.reshape(-1).index_select(0, order).unsqueeze(1)
    out = torch.zeros(T, H, dtype=torch.float32, device=h.device)
    out = out.index_add(0, token_of, ys.float() * wsel)
    return (out + residual.float()).to(h.dtype)
