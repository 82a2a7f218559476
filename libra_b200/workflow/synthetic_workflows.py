"""Synthetic workflows for the benchmark configurations.

``TargetTokenWorkflow`` — single turn: the prompt is a list of random token
ids, the policy samples a response, reward 1.0 if the response contains the
prompt's seeded target token id, else 0.0.

``SyntheticAgenticWorkflow`` — multi-turn: each turn generates up to
``turn_max_tokens`` tokens, then a synthetic tool return of random tokens
(lognormal length) is appended after a simulated tool latency (asyncio sleep);
the number of turns is geometric.  It drives the C-MLFQ request lifecycle
(begin -> route tool return -> finish / cancel) exactly like the reference's
R2E-Gym workflow (``workflow/r2e_gym.py:151-278``) and records tool events
(``payload_tokens``, ``token_position``, ``remaining_length``) for the prefix
tree and the planner.

Both return the reference trajectory schema: ``input_ids``, ``attention_mask``,
``loss_mask`` (1 on policy tokens only), ``logprobs`` (rollout logprobs aligned
to token positions), ``rewards``, ``versions``, ``prompt_len``/``output_len``.
"""

from __future__ import annotations

import asyncio
import math
import random
from dataclasses import dataclass
from typing import Any, Dict, List, Optional

import torch


def make_trajectory(prompt: List[int], segments: List[tuple], reward: float, version: int,
                    extra: Optional[Dict[str, Any]] = None) -> Dict[str, Any]:
    """segments: list of (token_ids, logprobs or None); logprobs None => not trained (tool tokens)."""
    ids = list(prompt)
    mask = [0.0] * len(prompt)
    lps = [0.0] * len(prompt)
    out_len = 0
    for toks, lp in segments:
        ids.extend(toks)
        if lp is None:
            mask.extend([0.0] * len(toks))
            lps.extend([0.0] * len(toks))
        else:
            mask.extend([1.0] * len(toks))
            lps.extend(float(x) for x in lp)
            out_len += len(toks)
    L = len(ids)
    traj = {"input_ids": torch.tensor(ids, dtype=torch.long).view(1, L),
            "attention_mask": torch.ones(1, L, dtype=torch.long),
            "loss_mask": torch.tensor(mask, dtype=torch.float32).view(1, L),
            "logprobs": torch.tensor(lps, dtype=torch.float32).view(1, L),
            "rewards": torch.tensor([float(reward)]), "versions": torch.tensor([int(version)]),
            "prompt_len": len(prompt), "output_len": L - len(prompt), "policy_tokens": out_len}
    if extra:
        traj.update(extra)
    return traj


class TargetTokenWorkflow:
    def __init__(self, max_new_tokens: int = 32, temperature: float = 1.0, top_p: float = 1.0):
        self.max_new_tokens, self.temperature, self.top_p = max_new_tokens, temperature, top_p

    async def run_episode(self, engine, data: Dict[str, Any], version: int = 0, rollout_index: int = 0) -> Dict:
        prompt = [int(t) for t in data["prompt_ids"]]
        seed = hash((data.get("prompt_id", ""), rollout_index, version)) & 0x7FFFFFFF
        res = await engine.generate(prompt, max_new_tokens=self.max_new_tokens, temperature=self.temperature,
                                    top_p=self.top_p, seed=seed, prompt_id=str(data.get("prompt_id", "")))
        out = list(res.get("token_ids") or [int(t) for t in res.get("tokens", [])])
        reward = 1.0 if int(data["target"]) in out else 0.0
        return make_trajectory(prompt, [(out, res.get("logprobs") or [0.0] * len(out))], reward, version,
                               {"prompt_id": data.get("prompt_id", "")})

    async def evaluate(self, engine, dataset, max_samples=None, concurrency: int = 16,
                       accuracy_threshold: float = 1.0, max_new_tokens=None, **kw) -> Dict[str, Any]:
        from libra_b200.workflow.evaluation import evaluate_workflow

        return await evaluate_workflow(self, engine, dataset, max_samples, concurrency, accuracy_threshold,
                                       max_new_tokens, **kw)


class GRPOLengthWorkflow:
    """Single turn with prescribed response lengths: rollout ``i`` of a group
    generates ``data["response_lens"][i]`` tokens at temperature 1.0 and gets
    reward ``data["rewards"][i]`` (the synthetic GRPO benchmark workload:
    random prompts, lognormal lengths, Bernoulli rewards)."""

    def __init__(self, temperature: float = 1.0):
        self.temperature = temperature

    async def run_episode(self, engine, data: Dict[str, Any], version: int = 0, rollout_index: int = 0) -> Dict:
        prompt = [int(t) for t in data["prompt_ids"]]
        n = int(data["response_lens"][rollout_index % len(data["response_lens"])])
        res = await engine.generate(prompt, max_new_tokens=n, temperature=self.temperature,
                                    prompt_id=str(data.get("prompt_id", "")))
        out = list(res.get("token_ids") or [])
        reward = float(data["rewards"][rollout_index % len(data["rewards"])])
        return make_trajectory(prompt, [(out, res.get("logprobs") or [0.0] * len(out))], reward, version,
                               {"prompt_id": data.get("prompt_id", "")})


def grpo_length_dataset(requests) -> List[Dict[str, Any]]:
    """Group ``workflow.synthetic.rollout_requests`` output by prompt into dataset items."""
    items: Dict[str, Dict[str, Any]] = {}
    for r in requests:
        it = items.setdefault(r.group_id, {"prompt_id": r.group_id, "prompt_ids": r.prompt, "response_lens": [],
                                           "rewards": []})
        it["response_lens"].append(r.response_len)
        it["rewards"].append(r.reward)
    return list(items.values())


def target_token_dataset(n_prompts: int, vocab: int = 1024, lo: int = 16, hi: int = 48, seed: int = 0,
                         token_lo: int = 4) -> List[Dict[str, Any]]:
    rng = random.Random(seed)
    out = []
    for i in range(n_prompts):
        L = rng.randint(lo, hi)
        out.append({"prompt_id": f"p{i}", "prompt_ids": [rng.randrange(token_lo, vocab) for _ in range(L)],
                    "target": rng.randrange(token_lo, vocab)})
    return out


@dataclass
class AgenticSpec:
    turn_max_tokens: int = 512
    turn_geometric_p: float = 0.3
    max_turns: int = 8
    tool_len_median: float = 400.0
    tool_len_sigma: float = 0.6
    tool_len_max: int = 2048
    tool_latency_median_s: float = 2.0
    tool_latency_sigma: float = 0.5
    context_cap: int = 16384
    vocab: int = 151936
    token_lo: int = 4


class SyntheticAgenticWorkflow:
    def __init__(self, spec: AgenticSpec = AgenticSpec(), temperature: float = 1.0, reward_p: float = 0.4,
                 latency_scale: float = 1.0):
        self.spec, self.temperature, self.reward_p = spec, temperature, reward_p
        self.latency_scale = latency_scale

    def _turns(self, rng: random.Random) -> int:
        n = 1
        while n < self.spec.max_turns and rng.random() > self.spec.turn_geometric_p:
            n += 1
        return n

    async def run_episode(self, engine, data: Dict[str, Any], version: int = 0, rollout_index: int = 0) -> Dict:
        s = self.spec
        rng = random.Random(hash((data.get("prompt_id", ""), rollout_index, version)) & 0x7FFFFFFF)
        prompt = [int(t) for t in data["prompt_ids"]]
        pid = str(data.get("prompt_id", ""))
        hetero = hasattr(engine, "begin_cmlfq_request")
        rid = engine.begin_cmlfq_request(pid, len(prompt)) if hetero else ""
        segments, events, context = [], [], list(prompt)
        generated = 0
        try:
            for turn in range(self._turns(rng)):
                budget = min(s.turn_max_tokens, s.context_cap - len(context))
                if budget <= 0:
                    break
                res = await engine.generate(context, max_new_tokens=budget, temperature=self.temperature,
                                            seed=rng.randrange(1 << 30), prompt_id=pid, request_id=rid)
                out = list(res.get("token_ids") or [])
                segments.append((out, res.get("logprobs") or [0.0] * len(out)))
                context += out
                generated += len(out)
                if len(context) >= s.context_cap:
                    break
                n_tool = int(min(s.tool_len_max, max(1, round(rng.lognormvariate(math.log(s.tool_len_median),
                                                                                 s.tool_len_sigma)))))
                n_tool = min(n_tool, s.context_cap - len(context))
                if n_tool <= 0:
                    break
                latency = rng.lognormvariate(math.log(s.tool_latency_median_s), s.tool_latency_sigma)
                await asyncio.sleep(latency * self.latency_scale)
                tool = [rng.randrange(s.token_lo, s.vocab) for _ in range(n_tool)]
                events.append({"turn": turn, "tool_type": "synthetic_tool", "payload_tokens": n_tool,
                               "token_position": generated, "latency_s": latency})
                if hetero and rid:
                    engine.route_cmlfq_tool_return(rid, {"tool_type": "synthetic_tool", "payload_tokens": n_tool,
                                                         "output": ""}, generated)
                segments.append((tool, None))
                context += tool
            if hetero and rid:
                engine.finish_cmlfq_request(rid, generated)
        except BaseException:
            if hetero and rid:
                engine.cancel_cmlfq_request(rid)
            raise
        for e in events:
            e["remaining_length"] = max(0, generated - e["token_position"])
        reward = 1.0 if rng.random() < self.reward_p else 0.0
        return make_trajectory(prompt, segments, reward, version,
                               {"prompt_id": pid, "tool_events": events, "num_turns": len(events) + 1,
                                "total_output_tokens": generated})
