"""Expert parallelism for MoE layers: token dispatch / combine all-to-all.

Reference: MCore's MoE token dispatcher + grouped GEMM
(``engine/megatron_core_train_engine.py:299-308``; Qwen3-30B-A3B: 128 experts,
top-8).  The EP group owns ``E / ep`` experts per rank.  Forward:
route (fp32 softmax top-k, renormalised) -> sort the (token, k) assignments by
destination rank -> ``all_to_all_single`` the rows and their local expert ids
-> per-local-expert SwiGLU MLP (tcgen05 GEMMs through ``models.moe``) ->
all-to-all back -> weighted sum into the residual.  Autograd runs the same
exchanges in reverse.

With a ``PeerExpertExchange`` the two all-to-alls become one kernel each over
NVLink peer memory (``ops/csrc/ep_exchange.cu``): dispatch stores every
(token, k) row straight into the expert owner's receive slot, combine loads the
k expert outputs of each token from the owners and sums them with the routing
weights and the residual in the same pass.  The routing plan places received
rows grouped by local expert, so the expert MLP is a grouped GEMM with no
per-expert gather/scatter.
"""

from __future__ import annotations

from dataclasses import dataclass
from typing import List, Optional

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


def ep_moe_mlp(h, residual, router, w1_local, w2_local, cfg, group, exchange: Optional["PeerExpertExchange"] = None):
    """MoE block with experts sharded over ``group``; returns residual + MoE(h).
    With ``exchange`` the dispatch and combine run as peer-memory kernels."""
    if exchange is not None:
        return _ep_moe_mlp_peer(h, residual, router, w1_local, w2_local, cfg, exchange)
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


# ----------------------------------------------------------------------------- peer-memory dispatch / combine

CTAS_PER_SM = 4  # grid = 4 x SMs, the same on every rank: arrival counters count CTAs


@dataclass
class RoutePlan:
    """Where each (token, k) assignment j = t * k + kk lives on the expert side."""

    dst_rank: torch.Tensor  # int32 [T*k]: rank owning the assignment's expert
    dst_row: torch.Tensor  # int32 [T*k]: row in that rank's receive slot
    offs: torch.Tensor  # int32 [E_l + 1] on the device: this rank's padded group of each local expert
    valid: torch.Tensor  # bf16 [recv_total, 1]: 1 on received rows, 0 on group padding
    recv_total: int  # rows of this rank's padded receive layout
    k: int


def route_plan(experts: torch.Tensor, counts_all: torch.Tensor, me: int, align: int = 128) -> RoutePlan:
    """Destination of every assignment, from all ranks' per-expert counts.

    ``experts`` [T, k] global expert ids of this rank's tokens; ``counts_all``
    [n, E] the number of assignments each rank sends to each expert.  The
    receive slot of rank d holds one group per local expert, each starting at a
    multiple of ``align`` rows (so the expert GEMM runs as one grouped launch
    over tile-aligned groups), ordered inside by (source rank, source order):
    row = (start of the expert's group on d) + (rows of this expert from lower
    ranks) + (position among this rank's rows for the expert).  One number is
    read back to the host: this rank's padded receive total, which sizes its
    buffers.
    """
    n, E = counts_all.shape
    E_l = E // n
    T, k = experts.shape
    flat = experts.reshape(-1)
    order = torch.argsort(flat, stable=True)
    g = flat[order]
    cnt = counts_all.to(torch.int64)
    per_dest = cnt.sum(0).view(n, E_l)
    padded = (per_dest + align - 1) // align * align
    base = (padded.cumsum(1) - padded).reshape(-1)
    lower = (cnt.cumsum(0) - cnt)[me]
    start = cnt[me].cumsum(0) - cnt[me]
    i = torch.arange(flat.numel(), device=flat.device)
    row_sorted = base[g] + lower[g] + i - start[g]
    dst_rank = torch.empty(flat.numel(), dtype=torch.int32, device=flat.device)
    dst_row = torch.empty_like(dst_rank)
    dst_rank[order] = (g // E_l).to(torch.int32)
    dst_row[order] = row_sorted.to(torch.int32)
    offs = torch.zeros(E_l + 1, dtype=torch.int64, device=flat.device)
    offs[1:] = padded[me].cumsum(0)
    total = int(offs[-1])
    r = torch.arange(total, device=flat.device)
    grp = torch.searchsorted(offs[1:], r, right=True).clamp_(max=E_l - 1)
    valid = ((r - offs[grp]) < per_dest[me][grp]).to(torch.bfloat16).unsqueeze(1)
    return RoutePlan(dst_rank, dst_row, offs.to(torch.int32), valid, total, k)


class PeerExpertExchange:
    """Symmetric receive / send slots shared over CUDA IPC by the EP group.

    Per rank: ``rx`` (2 slots of [max_rows, H] bf16, written by peers' dispatch),
    ``tx`` (2 slots, read by peers' combine) and 16 int32 arrival counters.
    Calls are collective: every rank makes the same push / pull calls in the
    same order (forward: dispatch then combine; backward in reverse).
    """

    def __init__(self, group, max_rows: int, hidden: int, device):
        from libra_b200.parallel.peer_gemm import MAX_RANKS

        self.grid = CTAS_PER_SM * torch.cuda.get_device_properties(torch.device(device)).multi_processor_count

        self.group = group
        self.n = dist.get_world_size(group) if dist.is_initialized() and group is not None else 1
        self.me = dist.get_rank(group) if dist.is_initialized() and group is not None else 0
        if self.n > MAX_RANKS:
            raise ValueError(f"at most {MAX_RANKS} ranks")
        if hidden % 8:
            raise ValueError("hidden size must be a multiple of 8")
        self.max_rows, self.H = int(max_rows), int(hidden)
        self.slot_bytes = (self.max_rows * self.H * 2 + 255) // 256 * 256
        self.buf = torch.zeros(4 * self.slot_bytes + 256, dtype=torch.uint8, device=device)
        bases = [int(self.buf.data_ptr())]
        self._opened = []
        if self.n > 1:
            C = ops.ext()
            handles = [None] * self.n
            dist.all_gather_object(handles, C.ipc_export(self.buf), group=self.group)
            bases = []
            with torch.cuda.device(self.buf.device):
                for r, (h, off) in enumerate(handles):
                    if r == self.me:
                        bases.append(int(self.buf.data_ptr()))
                    else:
                        base = C.ipc_open(h)
                        self._opened.append(base)
                        bases.append(base + int(off))
        self.rx = bases
        self.tx = [b + 2 * self.slot_bytes for b in bases]
        self.flags = [b + 4 * self.slot_bytes for b in bases]
        self.push_calls = 0
        self.pull_calls = 0
        if self.n > 1:
            torch.cuda.synchronize(self.buf.device)
            dist.barrier(group=self.group)

    def close(self) -> None:
        for base in self._opened:
            ops.ext().ipc_close(base)
        self._opened = []

    def _slot_view(self, area: int, slot: int, rows: int) -> torch.Tensor:
        off = (2 * area + slot) * self.slot_bytes
        return self.buf[off:off + rows * self.H * 2].view(torch.bfloat16).view(rows, self.H)

    def plan(self, experts: torch.Tensor, num_experts: int) -> RoutePlan:
        cnt = torch.bincount(experts.reshape(-1), minlength=num_experts).to(torch.int32)
        if self.n > 1:
            parts = [torch.empty_like(cnt) for _ in range(self.n)]
            dist.all_gather(parts, cnt, group=self.group)
            counts_all = torch.stack(parts)
        else:
            counts_all = cnt[None]
        # rows beyond max_rows are refused by the dispatch kernel (error word), not checked here
        return route_plan(experts, counts_all, self.me)

    def push(self, x: torch.Tensor, plan: RoutePlan, scale: Optional[torch.Tensor] = None) -> torch.Tensor:
        """Rows x[j // k] (times scale[j]) to their owners; returns this rank's received rows."""
        slot = self.push_calls & 1
        self.push_calls += 1
        x = x.contiguous()
        ops.ext().ep_push(self.rx, self.flags, self.me, slot * self.slot_bytes, x,
                          None if scale is None else scale.reshape(-1).float().contiguous(),
                          plan.dst_rank, plan.dst_row, plan.k, self.max_rows, self.push_calls, self.grid,
                          ops.error_flag(x.device))
        # group padding rows hold whatever the slot held before: zero them for the grouped GEMMs
        return self._slot_view(0, slot, plan.recv_total) * plan.valid

    def send_view(self, rows: int) -> torch.Tensor:
        """The slot the next ``pull`` publishes: a producer that writes its [rows, H] output
        here saves the copy into the slot."""
        return self._slot_view(1, self.pull_calls & 1, rows)

    def pull(self, y: torch.Tensor, plan: RoutePlan, weight: Optional[torch.Tensor] = None,
             residual: Optional[torch.Tensor] = None, T: int = 0, save_rows: bool = False):
        """Publishes this rank's rows ``y`` [recv_total, H]; returns (out [T, H], gathered rows or None)
        with out[t] = residual[t] + sum_kk weight[t, kk] * (row of assignment (t, kk))."""
        slot = self.pull_calls & 1
        self.pull_calls += 1
        dst = self._slot_view(1, slot, y.shape[0])
        if y.shape[0] and y.data_ptr() != dst.data_ptr():
            dst.copy_(y)
        out = torch.empty(T, self.H, dtype=torch.bfloat16, device=self.buf.device)
        gath = torch.empty(T * plan.k, self.H, dtype=torch.bfloat16, device=out.device) if save_rows else None
        ops.ext().ep_pull(self.tx, self.flags, self.me, slot * self.slot_bytes,
                          None if weight is None else weight.reshape(-1).float().contiguous(),
                          None if residual is None else residual.contiguous(), plan.dst_rank, plan.dst_row,
                          plan.k, self.max_rows, out, gath, self.pull_calls, self.grid, ops.error_flag(out.device))
        return out, gath


class _PeerDispatch(torch.autograd.Function):
    @staticmethod
    def forward(ctx, h, plan, xchg):
        ctx.plan, ctx.xchg, ctx.T = plan, xchg, h.shape[0]
        return xchg.push(h, plan)

    @staticmethod
    def backward(ctx, g):
        dh, _ = ctx.xchg.pull(g.contiguous(), ctx.plan, T=ctx.T)
        return dh, None, None


class _PeerCombine(torch.autograd.Function):
    @staticmethod
    def forward(ctx, y, weights, residual, plan, xchg):
        out, gath = xchg.pull(y, plan, weight=weights, residual=residual, T=residual.shape[0],
                              save_rows=weights.requires_grad)
        ctx.plan, ctx.xchg = plan, xchg
        ctx.save_for_backward(weights, gath if gath is not None else weights.new_empty(0))
        return out

    @staticmethod
    def backward(ctx, g):
        weights, gath = ctx.saved_tensors
        g = g.contiguous()
        dy = ctx.xchg.push(g, ctx.plan, scale=weights)  # padding rows zeroed like the forward dispatch
        dw = None
        if ctx.needs_input_grad[1]:
            T, k = weights.shape
            dw = torch.einsum("th,tkh->tk", g.float(), gath.view(T, k, -1).float())
        return dy, dw, g, None, None


def _ep_moe_mlp_peer(h, residual, router, w1_local, w2_local, cfg, xchg: PeerExpertExchange):
    from libra_b200.models.moe import route

    weights, experts, _ = route(h, router, cfg.num_experts_per_tok, cfg.norm_topk_prob)
    plan = xchg.plan(experts, cfg.num_experts)
    x_recv = _PeerDispatch.apply(h, plan, xchg)
    # both expert projections are single grouped launches over the padded per-expert groups; the second
    # writes straight into the send slot that the combine kernels on the other ranks read
    a = ops.grouped_swiglu(x_recv, w1_local, plan.offs)
    y_recv = ops.grouped_linear(a, w2_local, plan.offs, out=xchg.send_view(plan.recv_total))
    return _PeerCombine.apply(y_recv, weights, residual, plan, xchg)


def _bench(argv=None) -> None:
    """Device time of MoE dispatch + combine, peer-memory kernels against NCCL all-to-all.

    torchrun --nproc-per-node 2 --master-addr 127.0.0.1 -m libra_b200.parallel.expert_parallel
    Prints one JSON line (rank 0) with the max over ranks of the mean time per dispatch + combine.
    """
    import argparse
    import datetime
    import json
    import os

    p = argparse.ArgumentParser()
    p.add_argument("--tokens", type=int, default=8192)
    p.add_argument("--hidden", type=int, default=2048)
    p.add_argument("--experts", type=int, default=128)
    p.add_argument("--topk", type=int, default=8)
    p.add_argument("--iters", type=int, default=10)
    a = p.parse_args(argv)
    rank, world = int(os.environ.get("RANK", 0)), int(os.environ.get("WORLD_SIZE", 1))
    torch.cuda.set_device(int(os.environ.get("LOCAL_RANK", 0)))
    dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                            device_id=torch.device("cuda", torch.cuda.current_device()))
    grp = dist.group.WORLD
    T, H, E, k = a.tokens, a.hidden, a.experts, a.topk
    g = torch.Generator(device="cuda").manual_seed(rank)
    h = torch.randn(T, H, device="cuda", generator=g).bfloat16()
    res = torch.randn(T, H, device="cuda", generator=g).bfloat16()
    experts = torch.stack([torch.randperm(E, device="cuda", generator=g)[:k] for _ in range(T)])
    weights = torch.rand(T, k, device="cuda", generator=g)
    xchg = PeerExpertExchange(grp, max_rows=2 * T * k, hidden=H, device="cuda")
    plan = xchg.plan(experts, E)

    def peer():
        x_recv = xchg.push(h, plan)
        return xchg.pull(x_recv, plan, weight=weights, residual=res, T=T)[0]

    def dispatch():
        return xchg.push(h, plan)

    def combine():  # expert outputs already in the send slot, as the MoE block leaves them
        y = xchg.send_view(plan.recv_total)
        return xchg.pull(y, plan, weight=weights, residual=res, T=T)[0]

    flat = experts.reshape(-1)
    order = torch.argsort(flat, stable=True)
    sc = torch.bincount(flat // (E // world), minlength=world)
    rc = torch.empty_like(sc)
    dist.all_to_all_single(rc, sc, group=grp)
    sc, rc = sc.tolist(), rc.tolist()
    tok = order // k
    wsel = weights.reshape(-1)[order].unsqueeze(1)

    def nccl():
        x_recv = _all_to_all(h.index_select(0, tok), sc, rc, grp)
        y = _all_to_all(x_recv, rc, sc, grp)
        return (res.float().index_add(0, tok, y.float() * wsel)).bfloat16()

    torch.testing.assert_close(peer().float(), nccl().float(), rtol=2e-2, atol=5e-2)
    out = {}
    for name, fn in (("peer", peer), ("nccl", nccl), ("peer_dispatch", dispatch), ("peer_combine", combine)):
        for _ in range(3):
            fn()
        dist.barrier()
        torch.cuda.synchronize()
        t0, t1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        t0.record()
        for _ in range(a.iters):
            fn()
        t1.record()
        torch.cuda.synchronize()
        ms = torch.tensor([t0.elapsed_time(t1) / a.iters], device="cuda")
        dist.all_reduce(ms, op=dist.ReduceOp.MAX, group=grp)
        out[name + "_ms"] = round(float(ms), 4)
    cross = T * k * H * 2 * (world - 1) / world  # bytes leaving this rank per direction, dispatch alone
    out.update(tokens_per_rank=T, hidden=H, experts=E, topk=k, ranks=world,
               peer_dispatch_combine_gbs_per_direction=round(2 * cross / out["peer_ms"] / 1e6, 1))
    if rank == 0:
        print(json.dumps(out))
    xchg.close()
    dist.barrier()
    dist.destroy_process_group()


if __name__ == "__main__":
    _bench()
