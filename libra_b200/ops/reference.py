"""Plain PyTorch fp32 implementations of every fused op.

These are the numerics oracle for the CUDA kernels (tests compare against
them) and the execution path for CPU tensors (gloo plumbing runs, unit tests).
They follow the maths of the reference's library calls:

* RMSNorm / q-k norm / RoPE / SwiGLU as in the HF/Megatron Qwen3 block.
* token logprob = log_softmax(logits)[target] (reference
  ``engine/train_engine.py:35`` ``_selected_token_logprobs`` and
  ``engine/megatron_core_train_engine.py:905-948``).
* GRPO loss (reference ``engine/megatron_core_train_engine.py:950-986``).
"""

from __future__ import annotations

import math

import torch
import torch.nn.functional as F


def rmsnorm(x: torch.Tensor, w: torch.Tensor, eps: float) -> torch.Tensor:
    xf = x.float()
    rstd = torch.rsqrt(xf.pow(2).mean(-1, keepdim=True) + eps)
    return (xf * rstd * w.float()).to(x.dtype)


def rope_tables(max_positions: int, head_dim: int, theta: float, device=None):
    """cos/sin tables [P, D/2] in fp32, computed in float64."""
    inv = 1.0 / (theta ** (torch.arange(0, head_dim, 2, dtype=torch.float64) / head_dim))
    pos = torch.arange(max_positions, dtype=torch.float64)
    ang = torch.outer(pos, inv)
    return ang.cos().float().to(device), ang.sin().float().to(device)


def apply_rope(x: torch.Tensor, cos: torch.Tensor, sin: torch.Tensor, pos: torch.Tensor) -> torch.Tensor:
    """x: [T, heads, D]; rotate-half convention."""
    half = x.shape[-1] // 2
    c = cos[pos.long()].unsqueeze(1)
    s = sin[pos.long()].unsqueeze(1)
    x1, x2 = x[..., :half], x[..., half:]
    return torch.cat([x1 * c - x2 * s, x2 * c + x1 * s], dim=-1)


def qk_norm_rope(qkv, qw, kw, pos, cos, sin, nq, nkv, eps):
    T = qkv.shape[0]
    D = qkv.shape[1] // (nq + 2 * nkv)
    x = qkv.float().view(T, nq + 2 * nkv, D)
    q, k, v = x[:, :nq], x[:, nq:nq + nkv], x[:, nq + nkv:]
    q = rmsnorm(q, qw, eps).float()
    k = rmsnorm(k, kw, eps).float()
    q = apply_rope(q, cos, sin, pos)
    k = apply_rope(k, cos, sin, pos)
    dt = qkv.dtype
    return q.to(dt).contiguous(), k.to(dt).contiguous(), v.to(dt).contiguous()


def swiglu(gu: torch.Tensor) -> torch.Tensor:
    g, u = gu.float().chunk(2, dim=-1)
    return (F.silu(g) * u).to(gu.dtype)


def varlen_causal_attention(q, k, v, cu_seqlens, scale=None):
    """q [T, Hq, D], k/v [T, Hkv, D]; packed sequences delimited by cu_seqlens."""
    T, hq, d = q.shape
    hkv = k.shape[1]
    scale = scale if scale is not None else 1.0 / math.sqrt(d)
    out = torch.empty_like(q)
    bounds = cu_seqlens.tolist()
    for s, e in zip(bounds[:-1], bounds[1:]):
        if e <= s:
            continue
        qs = q[s:e].float().transpose(0, 1)
        ks = k[s:e].float().transpose(0, 1).repeat_interleave(hq // hkv, dim=0)
        vs = v[s:e].float().transpose(0, 1).repeat_interleave(hq // hkv, dim=0)
        att = (qs @ ks.transpose(-1, -2)) * scale
        L = e - s
        mask = torch.ones(L, L, dtype=torch.bool, device=q.device).triu(1)
        att = att.masked_fill(mask, float("-inf")).softmax(-1)
        out[s:e] = (att @ vs).transpose(0, 1).to(q.dtype)
    return out


def token_logprobs(logits: torch.Tensor, targets: torch.Tensor, temperature: float = 1.0):
    z = logits.float() / temperature
    lp = torch.log_softmax(z, dim=-1)
    sel = lp.gather(-1, targets.long().unsqueeze(-1)).squeeze(-1)
    ent = -(lp.exp() * lp).sum(-1)
    return sel, ent


def grpo_loss(logp, old_logp, mask, adv, clip_eps: float, kl_coef: float):
    """PPO-clip with log-ratio clamped to [-20, 20] and the k3 KL estimator.

    All inputs are per-token vectors of the same shape except ``adv`` which is
    broadcast per token already.
    """
    log_ratio = logp - old_logp
    ratio = torch.exp(log_ratio.clamp(-20.0, 20.0))
    clipped = ratio.clamp(1.0 - clip_eps, 1.0 + clip_eps)
    pg = torch.maximum(-adv * ratio, -adv * clipped)
    count = mask.sum().clamp(min=1.0)
    pg_loss = (pg * mask).sum() / count
    kl = (((ratio - 1.0) - log_ratio) * mask).sum() / count
    return pg_loss + kl_coef * kl, pg_loss, kl
