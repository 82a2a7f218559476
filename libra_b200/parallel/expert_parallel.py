"""Expert parallelism for MoE layers: token dispatch / combine all-to-all.

Reference: MCore's MoE token dispatcher + grouped GEMM
(``engine/megatron_core_train_engine.py:299-308``; Qwen3-30B-A3B: 128 experts,
top-8).  The EP group owns ``E / ep`` experts per rank.  Forward:
route (fp32 softmax top-k, renormalised) -> sort the (token, k) assignments by
destination rank -> ``all_to_all_single`` the rows and their local expert ids
-> per-local-expert SwiGLU MLP (tcgen05 GEMMs through ``models.moe``) ->
all-to-all back -> weighted sum into the residual.  Autograd runs the same
exchanges in reverse.
"""

from __future__ import annotations

from typing import List

import torch
import torch.distributed as dist

from libra_b200 import ops


def _all_to_all(x: torch.Tensor, send_counts: List[int], recv_counts: List[int], group) -> torch.Tensor:
    out = torch.empty((sum(recv_counts),) + tuple(x.shape[1:]), dtype=x.dtype, device=x.device)
    dist.all_to_all_single(out, x.contiguous(), recv_counts, send_counts, group=group)
    return out


class _AllToAll(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, send_counts, recv_counts, group):
        ctx.sc, ctx.rc, ctx.group = send_counts, recv_counts, group
        return _all_to_all(x, send_counts, recv_counts, group)

    @staticmethod
    def backward(ctx, g):
        return _all_to_all(g, ctx.rc, ctx.sc, ctx.group), None, None, None


def ep_moe_mlp(h, residual, router, w1_local, w2_local, cfg, group):
    """MoE block with experts sharded over ``group``; returns residual + MoE(h)."""
    ep = dist.get_world_size(group) if dist.is_initialized() else 1
    E_l = w1_local.shape[0]
    T, H = h.shape
    k = cfg.num_experts_per_tok
    from libra_b200.models.moe import route

    weights, experts, _ = route(h, router, k, cfg.norm_topk_prob)
    flat_e = experts.reshape(-1)
    order = torch.argsort(flat_e, stable=True)
    dest = flat_e[order] // E_l
    send_counts = torch.bincount(dest, minlength=ep)
    counts = send_counts.clone()
    recv = torch.empty_like(counts)
    if ep > 1:
        dist.all_to_all_single(recv, counts, group=group)
    else:
        recv = counts
    sc, rc = send_counts.tolist(), recv.tolist()
    tok = order // k
    x_send = h.index_select(0, tok)
    e_send = (flat_e[order] % E_l).to(torch.int32)
    x_recv = _AllToAll.apply(x_send, sc, rc, group) if ep > 1 else x_send
    e_recv = _all_to_all(e_send, sc, rc, group) if ep > 1 else e_send
    # local experts on the received rows
    y_recv = torch.zeros_like(x_recv)
    for e in range(E_l):
        sel = (e_recv == e).nonzero(as_tuple=True)[0]
        if sel.numel() == 0:
            continue
        xe = x_recv.index_select(0, sel)
        gu = ops.linear(xe, w1_local[e])
        a = ops.swiglu(gu)
        y_recv = y_recv.index_add(0, sel, ops.linear(a, w2_local[e]))
    y_send = _AllToAll.apply(y_recv, rc, sc, group) if ep > 1 else y_recv
    wsel = weights.reshape(-1)[order].unsqueeze(1)
    out = torch.zeros((T, H), dtype=torch.float32, device=h.device)
    out = out.index_add(0, tok, y_send.float() * wsel)
    return (out + residual.float()).to(h.dtype)
