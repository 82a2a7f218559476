"""Sequence parallelism for the tensor-parallel training model.

Megatron's sequence parallelism (enabled by the reference's MCore engine with
``sequence_parallel``, engine/megatron_core_train_engine.py:286-288) keeps the
residual stream split along tokens over the TP group: RMSNorm and the residual
adds run on ``T / tp`` rows per rank, a column-parallel linear all-gathers its
input rows first, and a row-parallel linear reduce-scatters its output instead
of all-reducing it.  Activation memory outside attention and the MLP drops by
``tp``, and the per-layer collective volume stays that of one all-reduce.

Collectives here:

* ``sp_gather`` / ``sp_scatter`` are the autograd pair all-gather <->
  reduce-scatter over the token dimension (NCCL; gloo ranks use all-reduce
  and slicing, since gloo has no reduce-scatter of tensors);
* ``sp_row_parallel_linear`` runs the fused GEMM + reduce-scatter kernel over
  NVLink peer memory (``PeerGemmAllReduce.reduce_scatter``) when peer buffers
  are registered for the group and output width, and our GEMM + NCCL
  reduce-scatter otherwise; its backward all-gathers the output gradient once
  and reuses it for both the input and the weight gradient;
* ``sp_column_parallel_linear`` runs the fused all-gather + GEMM kernel
  (``PeerAllGatherGemm``) when one is registered for the shard shape, else
  all-gather + GEMM.

The token count of a packed batch is padded to a multiple of ``sp_multiple``
so every rank holds the same number of rows (256 x tp on CUDA, the fused
kernels' row block; tp on CPU).
"""

from __future__ import annotations

from typing import Dict, Optional, Tuple

import torch
import torch.distributed as dist

from libra_b200 import ops


def _ws(group) -> int:
    return dist.get_world_size(group) if dist.is_initialized() else 1


def _rank(group) -> int:
    return dist.get_rank(group) if dist.is_initialized() else 0


def _gloo(group) -> bool:
    return dist.get_backend(group) == "gloo"


def sp_multiple(tp: int, device) -> int:
    return 256 * tp if torch.device(device).type == "cuda" else tp


def all_gather_rows(x: torch.Tensor, group) -> torch.Tensor:
    n = _ws(group)
    if n == 1:
        return x
    x = x.contiguous()
    if _gloo(group):
        parts = [torch.empty_like(x) for _ in range(n)]
        dist.all_gather(parts, x, group=group)
        return torch.cat(parts)
    out = torch.empty((n * x.shape[0],) + tuple(x.shape[1:]), dtype=x.dtype, device=x.device)
    dist.all_gather_into_tensor(out, x, group=group)
    return out


def reduce_scatter_rows(x: torch.Tensor, group) -> torch.Tensor:
    n = _ws(group)
    if n == 1:
        return x
    x = x.contiguous()
    rows = x.shape[0] // n
    if _gloo(group):
        y = x.clone()
        dist.all_reduce(y, group=group)
        r = _rank(group)
        return y[r * rows:(r + 1) * rows].contiguous()
    out = torch.empty((rows,) + tuple(x.shape[1:]), dtype=x.dtype, device=x.device)
    dist.reduce_scatter_tensor(out, x, group=group)
    return out


class _Gather(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, group):
        ctx.group = group
        return all_gather_rows(x, group)

    @staticmethod
    def backward(ctx, g):
        return reduce_scatter_rows(g, ctx.group), None


class _Scatter(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, group):
        ctx.group = group
        return reduce_scatter_rows(x, group)

    @staticmethod
    def backward(ctx, g):
        return all_gather_rows(g, ctx.group), None


class _GatherToReplicated(torch.autograd.Function):
    """All-gather whose consumer returns the complete gradient on every rank
    (the vocab-parallel logprob all-reduces its input gradient): the backward
    keeps this rank's rows instead of summing them again."""

    @staticmethod
    def forward(ctx, x, group):
        ctx.group, ctx.rows = group, x.shape[0]
        return all_gather_rows(x, group)

    @staticmethod
    def backward(ctx, g):
        r = _rank(ctx.group)
        return g[r * ctx.rows:(r + 1) * ctx.rows], None


def sp_gather_to_replicated(x_local: torch.Tensor, group) -> torch.Tensor:
    return _GatherToReplicated.apply(x_local, group)


def sp_gather(x_local: torch.Tensor, group) -> torch.Tensor:
    """[T/tp, ...] -> [T, ...] (backward: reduce-scatter of the gradient)."""
    return _Gather.apply(x_local, group)


def sp_scatter(x_full: torch.Tensor, group) -> torch.Tensor:
    """Partial [T, ...] summed over the group, keep this rank's rows (backward: all-gather)."""
    return _Scatter.apply(x_full, group)


# ------------------------------------------------------------------ fused kernels (peer memory)
_AG_REGISTRY: Dict[Tuple[int, int, int], object] = {}


def enable_fused_sequence_parallel(group, max_rows: int, row_widths, gather_shapes, device) -> None:
    """Register the peer buffers of the fused SP kernels for one TP group:
    GEMM + reduce-scatter for every row-parallel output width in
    ``row_widths`` (up to ``max_rows`` full rows), and all-gather + GEMM for
    every (shard rows, K) in ``gather_shapes``.  Collective over the group."""
    from libra_b200.parallel.peer_gemm import PeerAllGatherGemm, enable_fused_row_parallel

    enable_fused_row_parallel(group, max_rows, row_widths, device)
    for rows, k in sorted(set((int(r), int(c)) for r, c in gather_shapes)):
        key = (id(group), rows, k)
        if key not in _AG_REGISTRY:
            _AG_REGISTRY[key] = PeerAllGatherGemm(group, rows, k, device)


def disable_fused_sequence_parallel() -> None:
    from libra_b200.parallel.peer_gemm import disable_fused_row_parallel

    for f in _AG_REGISTRY.values():
        f.close()
    _AG_REGISTRY.clear()
    disable_fused_row_parallel()


class _RowParallelRS(torch.autograd.Function):
    """y_local = reduce_scatter(a @ w^T) + residual_local; ``fused`` is a
    PeerGemmAllReduce (one kernel) or None (GEMM + NCCL)."""

    @staticmethod
    def forward(ctx, a, w, residual, group, fused):
        a2 = a.reshape(-1, a.shape[-1])
        if not a2.is_contiguous():
            a2 = a2.contiguous()
        if fused is not None:
            y = fused.reduce_scatter(a2, w, residual)
        else:
            y = reduce_scatter_rows(ops.linear(a2, w), group)
            if residual is not None:
                y = y + residual
        ctx.save_for_backward(a2, w)
        ctx.group, ctx.in_shape, ctx.has_residual = group, a.shape, residual is not None
        return y

    @staticmethod
    def backward(ctx, dy_local):
        a2, w = ctx.saved_tensors
        dy = all_gather_rows(dy_local.contiguous(), ctx.group)
        da = None
        if ctx.needs_input_grad[0]:
            # CPU ranks keep the activation dtype (the reference GEMM would round to bf16)
            da = ops.gemm(dy, w, b_mn=True) if dy.is_cuda else (dy.float() @ w.float()).to(a2.dtype)
            da = da.view(ctx.in_shape)
        dw = ops._accumulate_wgrad(w, dy, a2) if ctx.needs_input_grad[1] else None
        return da, dw, (dy_local if ctx.has_residual else None), None, None


def sp_row_parallel_linear(a: torch.Tensor, w_local: torch.Tensor, residual_local: Optional[torch.Tensor], group):
    """Row-parallel linear with a sequence-parallel output: this rank's token
    rows of sum_r a_r w_r^T, plus the local residual rows."""
    fused = None
    if _ws(group) > 1 and a.is_cuda:
        from libra_b200.parallel.peer_gemm import ROW_BLOCK, fused_for

        rows = a.numel() // a.shape[-1]
        f = fused_for(group, w_local.shape[0], rows)
        if f is not None and rows % (ROW_BLOCK * _ws(group)) == 0:
            fused = f
    return _RowParallelRS.apply(a, w_local, residual_local, group, fused)


class _AGColumnParallel(torch.autograd.Function):
    """y = all_gather(h_local) @ w^T in one kernel; backward: dh = reduce_scatter(dy @ w),
    dw += dy^T all_gather(h_local) (gathered again, as Megatron does, instead of
    keeping the full input alive between forward and backward)."""

    @staticmethod
    def forward(ctx, h_local, w, group, ag):
        h_local = h_local.contiguous()
        y = ag(h_local, w)
        ctx.save_for_backward(h_local, w)
        ctx.group = group
        return y

    @staticmethod
    def backward(ctx, dy):
        h_local, w = ctx.saved_tensors
        h_full = all_gather_rows(h_local, ctx.group)
        dy = dy.contiguous()
        dh = reduce_scatter_rows(ops.gemm(dy, w, b_mn=True), ctx.group) if ctx.needs_input_grad[0] else None
        dw = ops._accumulate_wgrad(w, dy, h_full) if ctx.needs_input_grad[1] else None
        return dh, dw, None, None


def sp_gathered_input(h_local: torch.Tensor, group) -> torch.Tensor:
    """All-gathered input rows of a column-parallel linear (autograd)."""
    return sp_gather(h_local, group)


def sp_column_parallel_linear(h_local: torch.Tensor, w_local: torch.Tensor, group) -> torch.Tensor:
    """Column-parallel linear whose input rows are sequence-sharded."""
    if _ws(group) > 1 and h_local.is_cuda:
        ag = _AG_REGISTRY.get((id(group), h_local.shape[0], h_local.shape[1]))
        if ag is not None:
            return _AGColumnParallel.apply(h_local, w_local, group, ag)
    return ops.linear(sp_gather(h_local, group), w_local)
