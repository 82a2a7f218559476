"""Token sampling: temperature, top-k and top-p (nucleus), with the sampled
token's logprob under the temperature-scaled distribution (what the rollout
returns as ``token_logprobs``; reference ``engine/rollout_engine.py:255``)."""

from __future__ import annotations

from dataclasses import dataclass, field
from typing import List, Optional

import torch


@dataclass
class SamplingParams:
    max_tokens: int = 1024
    temperature: float = 1.0
    top_p: float = 1.0
    top_k: int = -1
    stop_token_ids: List[int] = field(default_factory=list)
    seed: Optional[int] = None
    logprobs: bool = True


def sample(logits: torch.Tensor, temperature: torch.Tensor, top_p: torch.Tensor, top_k: torch.Tensor,
           generators: Optional[List[Optional[torch.Generator]]] = None):
    """logits [B, V] (any float dtype) -> (tokens [B] int64, logprobs [B] fp32).

    temperature 0 means greedy.  Filtering is applied per row.
    """
    x = logits.float()
    greedy = temperature <= 0
    t = torch.where(greedy, torch.ones_like(temperature), temperature).unsqueeze(1)
    x = x / t
    logp_full = torch.log_softmax(x, dim=-1)
    B, V = x.shape
    need_filter = bool(((top_k > 0) & (top_k < V)).any()) or bool((top_p < 1.0).any())
    probs_logits = x
    if need_filter:
        sorted_x, idx = torch.sort(x, dim=-1, descending=True)
        ranks = torch.arange(V, device=x.device).unsqueeze(0)
        k = torch.where(top_k > 0, top_k, torch.full_like(top_k, V)).unsqueeze(1)
        drop = ranks >= k
        cum = torch.softmax(sorted_x, dim=-1).cumsum(-1)
        drop |= (cum - torch.softmax(sorted_x, dim=-1)) > top_p.unsqueeze(1)
        sorted_x = sorted_x.masked_fill(drop, float("-inf"))
        probs_logits = torch.full_like(x, float("-inf")).scatter(1, idx, sorted_x)
    probs = torch.softmax(probs_logits, dim=-1)
    if generators is not None and any(g is not None for g in generators):
        toks = torch.stack([torch.multinomial(probs[i], 1, generator=g).squeeze(0) if g is not None
                            else torch.multinomial(probs[i], 1).squeeze(0) for i, g in enumerate(generators)])
    else:
        toks = torch.multinomial(probs, 1).squeeze(1)
    toks = torch.where(greedy, x.argmax(-1), toks)
    return toks, logp_full.gather(1, toks.unsqueeze(1)).squeeze(1)
