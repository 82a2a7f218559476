"""Causal GQA attention over packed (variable-length) sequences.

The training and prefill paths call :func:`flash_varlen_causal` with
q [T, Hq, D], k/v [T, Hkv, D] and ``cu_seqlens`` [B+1] int32.  The current
implementation routes to PyTorch's bundled flash-attention varlen kernel with a
(-1, 0) window (causal).  It is the one library kernel left on the training hot
path; it stands in for the reference's SDPA-flash call
(engine/megatron_core_attention.py:447-456) until the tcgen05 attention kernel
replaces it.
"""

from __future__ import annotations

import torch


def flash_varlen_causal(q, k, v, cu_seqlens, max_seqlen: int, scale=None):
    from torch.nn.attention.varlen import varlen_attn

    cu = cu_seqlens.to(device=q.device, dtype=torch.int32)
    return varlen_attn(q, k, v, cu, cu, int(max_seqlen), int(max_seqlen), scale=scale, window_size=(-1, 0))
