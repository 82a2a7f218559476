"""Synthetic GRPO workloads with the shapes of the benchmark configurations.

There is no dataset or checkpoint access on the benchmark machines, so every
benchmark runs on seeded synthetic prompts/responses of the stated length
distributions with random-init weights.  A trajectory dict has the same keys
as the reference's (``workflow/r2e_gym.py:290-304``): ``input_ids``,
``attention_mask``, ``loss_mask``, ``logprobs``, ``rewards``, ``advantages``,
``grpo_group_id``, ``rollout_index``, ``version``.
"""

from __future__ import annotations

import math
from dataclasses import dataclass
from typing import Dict, List, Optional

import numpy as np
import torch


@dataclass
class LengthDist:
    """Lognormal with a given median, clipped to [lo, hi]."""

    median: float
    sigma: float
    lo: int
    hi: int

    def sample(self, rng: np.random.Generator, n: int) -> np.ndarray:
        x = rng.lognormal(mean=math.log(self.median), sigma=self.sigma, size=n)
        return np.clip(np.round(x), self.lo, self.hi).astype(np.int64)


@dataclass
class GRPOWorkload:
    """Prompts x group size per step, with prompt/response length distributions."""

    name: str
    vocab_size: int
    prompts_per_step: int
    group_size: int
    prompt: LengthDist
    response: LengthDist
    reward_p: float = 0.4
    seed: int = 0
    token_lo: int = 4

    def trajectories(self, step: int, rank: int = 0, prompts: Optional[int] = None,
                     pin: bool = False) -> List[Dict[str, torch.Tensor]]:
        n_prompts = self.prompts_per_step if prompts is None else prompts
        rng = np.random.default_rng([self.seed, rank, step])
        plens = self.prompt.sample(rng, n_prompts)
        out: List[Dict[str, torch.Tensor]] = []
        for p in range(n_prompts):
            prompt = torch.from_numpy(rng.integers(self.token_lo, self.vocab_size, size=int(plens[p])))
            rlens = self.response.sample(rng, self.group_size)
            rewards = (rng.random(self.group_size) < self.reward_p).astype(np.float32)
            for g in range(self.group_size):
                resp = torch.from_numpy(rng.integers(self.token_lo, self.vocab_size, size=int(rlens[g])))
                ids = torch.cat([prompt, resp]).view(1, -1)
                L = ids.shape[1]
                mask = torch.zeros(1, L, dtype=torch.float32)
                mask[:, int(plens[p]):] = 1.0
                logprobs = torch.from_numpy(-rng.random((1, L), dtype=np.float32) * 2.0)
                logprobs[:, :int(plens[p])] = 0.0
                traj = {
                    "input_ids": ids,
                    "attention_mask": torch.ones(1, L, dtype=torch.long),
                    "loss_mask": mask,
                    "logprobs": logprobs,
                    "rewards": torch.tensor([float(rewards[g])]),
                    "grpo_group_id": f"r{rank}:s{step}:p{p}",
                    "rollout_index": g,
                    "version": step,
                }
                if pin:
                    for k, v in list(traj.items()):
                        if isinstance(v, torch.Tensor):
                            traj[k] = v.pin_memory()
                out.append(traj)
        group_normalize(out)
        return out


@dataclass
class RolloutRequest:
    """One GRPO sample to generate: the group's prompt, the response length to
    generate (the workload's length distribution; generation ignores stop
    tokens) and its Bernoulli reward."""

    group_id: str
    rollout_index: int
    prompt: List[int]
    response_len: int
    reward: float


def rollout_requests(wl: GRPOWorkload, step: int, rank: int = 0, prompts: Optional[int] = None) -> List[RolloutRequest]:
    """The generation side of a synthetic GRPO step: ``prompts`` x group size
    requests with the workload's prompt/response length distributions."""
    n_prompts = wl.prompts_per_step if prompts is None else prompts
    rng = np.random.default_rng([wl.seed, rank, step, 17])
    plens = wl.prompt.sample(rng, n_prompts)
    out: List[RolloutRequest] = []
    for p in range(n_prompts):
        prompt = rng.integers(wl.token_lo, wl.vocab_size, size=int(plens[p])).tolist()
        rlens = wl.response.sample(rng, wl.group_size)
        rewards = (rng.random(wl.group_size) < wl.reward_p).astype(np.float32)
        for g in range(wl.group_size):
            out.append(RolloutRequest(f"r{rank}:s{step}:p{p}", g, prompt, max(1, int(rlens[g])), float(rewards[g])))
    return out


def rollout_trajectory(req: RolloutRequest, output_tokens: List[int], output_logprobs: List[float], version: int,
                       pin: bool = False) -> Dict[str, torch.Tensor]:
    """Trajectory dict (reference schema) from a generated response."""
    P, R = len(req.prompt), len(output_tokens)
    ids = torch.tensor(req.prompt + list(output_tokens), dtype=torch.long).view(1, -1)
    mask = torch.zeros(1, P + R, dtype=torch.float32)
    mask[:, P:] = 1.0
    lps = torch.zeros(1, P + R, dtype=torch.float32)
    if R:
        lps[0, P:] = torch.tensor(output_logprobs, dtype=torch.float32)
    traj = {"input_ids": ids, "attention_mask": torch.ones(1, P + R, dtype=torch.long), "loss_mask": mask,
            "logprobs": lps, "rewards": torch.tensor([req.reward]), "grpo_group_id": req.group_id,
            "rollout_index": req.rollout_index, "version": version, "prompt_len": P, "output_len": R}
    if pin:
        for k, v in list(traj.items()):
            if isinstance(v, torch.Tensor):
                traj[k] = v.pin_memory()
    return traj


def group_normalize(trajectories: List[Dict]) -> None:
    """GRPO advantages: (r - mean) / (std + 1e-6) per group; zero-variance -> 0;
    singleton groups keep the raw reward (reference
    ``trainer/async_rl_trainer.py:557-598``)."""
    groups: Dict[str, List[Dict]] = {}
    for i, t in enumerate(trajectories):
        groups.setdefault(str(t.get("grpo_group_id", f"singleton:{i}")), []).append(t)
    for members in groups.values():
        scores = torch.stack([m["rewards"].reshape(-1).float()[0] for m in members])
        if len(members) == 1:
            adv = scores
        else:
            std = scores.std()
            adv = torch.zeros_like(scores) if (not torch.isfinite(std) or std <= 1e-6) else (scores - scores.mean()) / (std + 1e-6)
        for m, a in zip(members, adv):
            m["advantages"] = a.reshape(1)


WORKLOADS = {
    # CPU/gloo plumbing run: tiny model, 8 prompts x 4, prompt 16-48, response <= 32
    "tiny-cpu": GRPOWorkload("tiny-cpu", vocab_size=1024, prompts_per_step=8, group_size=4,
                             prompt=LengthDist(32, 0.3, 16, 48), response=LengthDist(24, 0.3, 1, 32)),
    # Qwen3-4B async GRPO: 64 prompts x 8; prompt median 300 (64-1024), response median 1500 (<= 4096)
    "qwen3-4b-grpo": GRPOWorkload("qwen3-4b-grpo", vocab_size=151936, prompts_per_step=64, group_size=8,
                                  prompt=LengthDist(300, 0.5, 64, 1024), response=LengthDist(1500, 0.75, 1, 4096)),
    # Qwen3-30B-A3B: 32 prompts x 8, prompt 512, response uniform-ish 512-4096 (lognormal proxy)
    "qwen3-30b-a3b-grpo": GRPOWorkload("qwen3-30b-a3b-grpo", vocab_size=151936, prompts_per_step=32, group_size=8,
                                       prompt=LengthDist(512, 0.0, 512, 512),
                                       response=LengthDist(1800, 0.6, 512, 4096)),
}
