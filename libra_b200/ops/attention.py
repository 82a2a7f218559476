"""Causal GQA attention over packed (variable-length) sequences.

q [T, Hq, 128], k/v [T, Hkv, 128], ``cu_seqlens`` [B+1] int32.  Forward and
backward are our tcgen05 kernels (``csrc/flash_attn.cu``, ``csrc/flash_attn_bwd.cu``);
the forward returns the output and the natural-log softmax denominators ``lse``
[Hq, T], which the backward reuses.  Stands in for the reference's SDPA-flash
call (engine/megatron_core_attention.py:447-456).

The kernels walk tile tables of (sequence, 128-row tile) pairs, heaviest
causal tiles first: q tiles for the forward and the dQ pass, kv tiles for the
dK/dV pass.  Build them once per packed batch with :func:`attn_tiles` (from the
host copy of ``cu_seqlens``) and reuse them for every layer.
"""

from __future__ import annotations

import math
from typing import Optional, Sequence

import torch

BLOCK = 128
HEAD_DIM = 128


def attn_tiles(cu_seqlens_host: Sequence[int], causal: bool = True, device=None, kv: bool = False) -> torch.Tensor:
    """int32 [n, 2] (sequence, tile) ordered by decreasing work.

    q tiles (``kv=False``): causal work of q tile t is t + 1 kv blocks.
    kv tiles (``kv=True``): causal work of kv tile t is n - t q blocks."""
    cu = [int(x) for x in cu_seqlens_host]
    items = []
    for b in range(len(cu) - 1):
        n = (cu[b + 1] - cu[b] + BLOCK - 1) // BLOCK
        for t in range(n):
            work = ((n - t) if kv else (t + 1)) if causal else n
            items.append((work, b, t))
    items.sort(key=lambda x: -x[0])
    tab = torch.tensor([[b, t] for _, b, t in items] or [[0, 0]], dtype=torch.int32)
    if not items:
        tab = tab[:0]
    if device is not None and torch.device(device).type == "cuda":
        tab = tab.pin_memory().to(device, non_blocking=True)
    return tab


class _FlashAttnFn(torch.autograd.Function):
    @staticmethod
    def forward(ctx, q, k, v, cu, tiles, kv_tiles, max_seqlen, scale):
        from libra_b200 import ops

        o, lse = ops.ext().flash_fwd(q, k, v, cu, tiles, scale, True, ops.error_flag(q.device))
        ctx.save_for_backward(q, k, v, o, lse, cu, tiles, kv_tiles)
        ctx.max_seqlen, ctx.scale = max_seqlen, scale
        return o

    @staticmethod
    def backward(ctx, do):
        from libra_b200 import ops

        q, k, v, o, lse, cu, tiles, kv_tiles = ctx.saved_tensors
        dq, dk, dv = ops.ext().flash_bwd(do.contiguous(), q, k, v, o, lse, cu, tiles, kv_tiles, ctx.scale, True,
                                         ops.error_flag(q.device))
        return dq, dk, dv, None, None, None, None, None


def flash_varlen_causal(q, k, v, cu_seqlens, max_seqlen: int, scale: Optional[float] = None,
                        tiles: Optional[torch.Tensor] = None, kv_tiles: Optional[torch.Tensor] = None):
    if scale is None:
        scale = 1.0 / math.sqrt(q.shape[-1])
    cu = cu_seqlens.to(device=q.device, dtype=torch.int32)
    if q.shape[-1] != HEAD_DIM:
        from torch.nn.attention.varlen import varlen_attn

        return varlen_attn(q, k, v, cu, cu, int(max_seqlen), int(max_seqlen), scale=scale, window_size=(-1, 0))
    if tiles is None:
        tiles = attn_tiles(cu.tolist(), True, q.device)
    if kv_tiles is None:
        kv_tiles = attn_tiles(cu.tolist(), True, q.device, kv=True) if torch.is_grad_enabled() else tiles
    return _FlashAttnFn.apply(q.contiguous(), k.contiguous(), v.contiguous(), cu, tiles, kv_tiles, int(max_seqlen),
                              float(scale))
