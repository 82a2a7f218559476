"""Shared multi-turn episode machinery of the workflows.

Every workflow of the reference (``workflow/{rlvr,agentic,r2e_gym,search_r1,
dapo_math,code_agent}.py``) runs the same loop: generate a turn, maybe call a
tool/validator, append its output as untrained tokens, route the tool return
through C-MLFQ, repeat; then score and emit one trajectory.  Here that loop is
written once; each workflow supplies its prompt, its tool step and its reward.

Trajectory keys (reference schema): ``input_ids``/``attention_mask``/
``loss_mask``/``logprobs`` [1, L], ``rewards``/``versions`` [1], plus
``input_len``/``prompt_len``, ``output_len``, ``rollout_index``,
``prompt_id``, ``tool_events``, ``num_turns``.
"""

from __future__ import annotations

import asyncio
import hashlib
from typing import Any, Callable, Dict, List, Optional, Tuple

import torch

Segment = Tuple[List[int], List[float], int]  # tokens, logprobs, trained (1) or not (0)


class MultiTurnWorkflow:
    tool_type = "tool"
    stop: Optional[List[str]] = None

    def __init__(self, reward_fn: Optional[Callable[..., float]], tokenizer, max_turns: int = 1,
                 max_new_tokens: int = 1024, max_seq_length: int = 8192, max_prompt_tokens: Optional[int] = None,
                 temperature: float = 1.0, top_p: float = 1.0, n_samples: int = 1):
        self.reward_fn, self.tokenizer = reward_fn, tokenizer
        self.max_turns = max(1, int(max_turns))
        self.max_new_tokens = max(1, int(max_new_tokens))
        self.max_seq_length = max(64, int(max_seq_length))
        if max_prompt_tokens is None:
            max_prompt_tokens = min(8192, max(64, self.max_seq_length // 2))
        self.max_prompt_tokens = max(16, min(int(max_prompt_tokens), self.max_seq_length - 16))
        self.temperature, self.top_p, self.n_samples = temperature, top_p, n_samples

    # ------------------------------------------------------------------ text helpers
    def encode(self, text: str) -> List[int]:
        return list(self.tokenizer.encode(text or "", add_special_tokens=False))

    def decode(self, ids: List[int]) -> str:
        return self.tokenizer.decode(ids, skip_special_tokens=True)

    def truncate(self, text: str, max_tokens: int) -> str:
        """Keep the head and the tail when a text exceeds ``max_tokens``."""
        ids = self.encode(text)
        if len(ids) <= max_tokens:
            return text
        head = max_tokens // 2
        return self.decode(ids[:head] + ids[len(ids) - (max_tokens - head):])

    def budget(self, prompt_tokens: int, used: int, turn: int, reserve: int) -> int:
        per_request = self.max_seq_length - prompt_tokens - 16
        per_turn = (self.max_seq_length - used - reserve) // max(1, self.max_turns - turn)
        return max(1, min(self.max_new_tokens, per_request, per_turn))

    def clip(self, tokens: List[int], lps: List[float], used: int) -> Tuple[List[int], List[float]]:
        room = self.max_seq_length - used
        return (tokens[:room], lps[:room]) if room > 0 else ([], [])

    @staticmethod
    def prompt_id(data: Dict[str, Any]) -> str:
        return str(data.get("prompt_id") or data.get("id") or data.get("question", "")[:64])

    # ------------------------------------------------------------------ per-workflow hooks
    def initial_prompt(self, data: Dict[str, Any]) -> str:
        raise NotImplementedError

    async def tool_step(self, engine, data: Dict[str, Any], output_text: str, turn: int
                        ) -> Optional[Tuple[str, Dict[str, Any]]]:
        """Feedback text + tool-event fields, or None to end the episode."""
        return None

    def score(self, data: Dict[str, Any], prompt: str, completion: str, segments: List[Segment]) -> float:
        row = {k: v for k, v in data.items() if k not in ("prompt", "completion")}
        return float(self.reward_fn(prompt=prompt, completion=completion, **row)) if self.reward_fn else 0.0

    # ------------------------------------------------------------------ episode
    def _seed(self, pid: str, version: int, idx: int, turn: int) -> int:
        h = hashlib.sha256(f"{pid}:{version}:{idx}:{turn}".encode()).digest()
        return int.from_bytes(h[:8], "big") % (2 ** 31 - 1)

    async def run_episode(self, engine, data: Dict[str, Any], version: int = 0, rollout_index: int = 0
                          ) -> Dict[str, Any]:
        prompt = self.initial_prompt(data)
        p_ids = self.encode(prompt)
        segments: List[Segment] = [(p_ids, [0.0] * len(p_ids), 0)]
        pid = self.prompt_id(data)
        begin = getattr(engine, "begin_cmlfq_request", None)
        rid = begin(pid, len(p_ids)) if callable(begin) else ""
        events: List[Dict[str, Any]] = []
        context, completion, turns = prompt, "", 0
        try:
            for turn in range(self.max_turns):
                turns = turn + 1
                used = sum(len(s[0]) for s in segments)
                ctx = self.truncate(context, max(16, self.max_seq_length - 32))
                ctx_ids = len(self.encode(ctx))
                kw = dict(prompt=ctx, max_new_tokens=self.budget(ctx_ids, used, turn, 128 if turn < self.max_turns - 1
                                                                  else 0),
                          temperature=self.temperature, top_p=self.top_p, n=1, input_tokens=ctx_ids,
                          seed=self._seed(pid, version, rollout_index, turn))
                if self.stop:
                    kw["stop"] = list(self.stop)
                if rid:
                    kw.update(request_id=rid, prompt_id=pid)
                resp = await engine.generate(**kw)
                text = resp.get("text", "") or ""
                out = [int(t) for t in (resp.get("token_ids") or [])] or self.encode(text)
                lps = [float(x) for x in (resp.get("logprobs") or [])]
                if len(lps) != len(out):
                    lps = [0.0] * len(out)
                out, lps = self.clip(out, lps, used)
                if out:
                    segments.append((out, lps, 1))
                completion += text
                if turn == self.max_turns - 1 or not out:
                    break
                step = await self.tool_step(engine, data, text, turn)
                if step is None:
                    break
                fb_text, event = step
                used = sum(len(s[0]) for s in segments)
                fb, _ = self.clip(self.encode(fb_text), [], used)
                if not fb:
                    break
                segments.append((fb, [0.0] * len(fb), 0))
                generated = sum(len(s[0]) for s in segments[1:])
                event = {"tool_type": self.tool_type, "output": fb_text, "status": "success", **event,
                         "payload_tokens": len(fb), "token_position": generated, "turn": turn}
                events.append(event)
                route = getattr(engine, "route_cmlfq_tool_return", None)
                if rid and callable(route):
                    route(rid, event, generated)
                context += text + fb_text
                completion += fb_text
            finish = getattr(engine, "finish_cmlfq_request", None)
            if rid and callable(finish):
                finish(rid, sum(len(s[0]) for s in segments[1:] if s[2]))
        except BaseException:
            cancel = getattr(engine, "cancel_cmlfq_request", None)
            if rid and callable(cancel):
                cancel(rid)
            raise
        reward = self.score(data, prompt, completion, segments)
        ids, lp, mask = [], [], []
        for toks, l, m in segments:
            ids += toks
            lp += l
            mask += [m] * len(toks)
        generated = sum(len(s[0]) for s in segments[1:])
        for e in events:
            e["remaining_length"] = max(0, generated - e["token_position"])
        L = len(ids)
        return {"input_ids": torch.tensor(ids, dtype=torch.long).view(1, L),
                "attention_mask": torch.ones(1, L, dtype=torch.long),
                "loss_mask": torch.tensor(mask, dtype=torch.float32).view(1, L),
                "logprobs": torch.tensor(lp, dtype=torch.float32).view(1, L),
                "rewards": torch.tensor([reward], dtype=torch.float32),
                "versions": torch.tensor([int(version)], dtype=torch.long),
                "input_len": len(p_ids), "prompt_len": len(p_ids), "output_len": L - len(p_ids),
                "rollout_index": rollout_index, "prompt_id": pid, "tool_events": events, "num_turns": turns,
                "completion": completion}

    async def run_batch(self, engine, batch: List[Dict[str, Any]], version: int = 0) -> List[Dict[str, Any]]:
        res = await asyncio.gather(*(self.run_episode(engine, d, version, i) for i, d in enumerate(batch)),
                                   return_exceptions=True)
        return [r for r in res if not isinstance(r, BaseException)]

    async def evaluate(self, engine, dataset, max_samples: Optional[int] = None, concurrency: int = 16,
                       accuracy_threshold: float = 1.0, max_new_tokens: Optional[int] = None,
                       strategy: str = "first", seed: int = 0, record_limit: int = 8) -> Dict[str, Any]:
        """Greedy evaluation over ``dataset`` (see ``workflow.evaluation``)."""
        from libra_b200.workflow.evaluation import evaluate_workflow

        return await evaluate_workflow(self, engine, dataset, max_samples, concurrency, accuracy_threshold,
                                       max_new_tokens, strategy, seed, record_limit)
