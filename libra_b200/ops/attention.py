"""Causal GQA attention over packed (variable-length) sequences.

q [T, Hq, 128], k/v [T, Hkv, 128], ``cu_seqlens`` [B+1] int32.  The forward
pass is our tcgen05 kernel (``csrc/flash_attn.cu``); it returns the output and
the natural-log softmax denominators ``lse`` [Hq, T].  The backward pass feeds
that output and ``lse`` to PyTorch's bundled flash-attention backward; this
library kernel stays on the hot path until the tcgen05 backward replaces it.
Stands in for the reference's SDPA-flash call
(engine/megatron_core_attention.py:447-456).

The kernel walks a tile table of (sequence, 128-row q tile) pairs, heaviest
causal tiles first.  Build it once per packed batch with :func:`attn_tiles`
(from the host copy of ``cu_seqlens``) and reuse it for every layer.
"""

from __future__ import annotations

import math
from typing import Optional, Sequence

import torch

BLOCK = 128
HEAD_DIM = 128


def attn_tiles(cu_seqlens_host: Sequence[int], causal: bool = True, device=None) -> torch.Tensor:
    """int32 [n, 2] (sequence, q tile) ordered by decreasing work."""
    cu = [int(x) for x in cu_seqlens_host]
    items = []
    for b in range(len(cu) - 1):
        n = (cu[b + 1] - cu[b] + BLOCK - 1) // BLOCK
        nblk = n
        for t in range(n):
            work = (t + 1) if causal else nblk
            items.append((work, b, t))
    items.sort(key=lambda x: -x[0])
    tab = torch.tensor([[b, t] for _, b, t in items] or [[0, 0]], dtype=torch.int32)
    if not items:
        tab = tab[:0]
    if device is not None and torch.device(device).type == "cuda":
        tab = tab.pin_memory().to(device, non_blocking=True)
    return tab


def _torch_flash_fwd(q, k, v, cu, max_seqlen, scale):
    out = torch.ops.aten._flash_attention_forward(q, k, v, cu, cu, max_seqlen, max_seqlen, 0.0, True, False,
                                                  scale=scale)
    return out[0], out[1]


class _FlashAttnFn(torch.autograd.Function):
    @staticmethod
    def forward(ctx, q, k, v, cu, tiles, max_seqlen, scale):
        from libra_b200 import ops

        o, lse = ops.ext().flash_fwd(q, k, v, cu, tiles, scale, True, ops.error_flag(q.device))
        ctx.save_for_backward(q, k, v, o, lse, cu)
        ctx.max_seqlen, ctx.scale = max_seqlen, scale
        return o

    @staticmethod
    def backward(ctx, do):
        q, k, v, o, lse, cu = ctx.saved_tensors
        rng = torch.zeros(2, dtype=torch.uint64, device=q.device)
        unused = torch.empty(0, device=q.device)
        dq, dk, dv = torch.ops.aten._flash_attention_backward(
            do.contiguous(), q, k, v, o, lse, cu, cu, ctx.max_seqlen, ctx.max_seqlen, 0.0, True, rng, unused,
            scale=ctx.scale)
        return dq, dk, dv, None, None, None, None


def flash_varlen_causal(q, k, v, cu_seqlens, max_seqlen: int, scale: Optional[float] = None,
                        tiles: Optional[torch.Tensor] = None):
    if scale is None:
        scale = 1.0 / math.sqrt(q.shape[-1])
    cu = cu_seqlens.to(device=q.device, dtype=torch.int32)
    if q.shape[-1] != HEAD_DIM:
        from torch.nn.attention.varlen import varlen_attn

        return varlen_attn(q, k, v, cu, cu, int(max_seqlen), int(max_seqlen), scale=scale, window_size=(-1, 0))
    if tiles is None:
        tiles = attn_tiles(cu.tolist(), True, q.device)
    return _FlashAttnFn.apply(q.contiguous(), k.contiguous(), v.contiguous(), cu, tiles, int(max_seqlen), float(scale))
