"""DAPO-Math: multi-turn math with validator feedback (reference ``workflow/dapo_math.py``).

After each attempt the validator scores the boxed answer; a correct answer or
the last turn ends the episode, otherwise its report is appended as an
untrained tool return and the model revises.
"""

from __future__ import annotations

from typing import Any, Dict

from libra_b200.env.prompts import MATH_SYSTEM, chat
from libra_b200.env.rewards import dapo_math_reward_fn, evaluate_math_completion, math_validator_feedback
from libra_b200.workflow.base import MultiTurnWorkflow


def _question(row: Dict[str, Any]) -> str:
    for k in ("question", "problem", "prompt"):
        v = row.get(k)
        if isinstance(v, list) and v and isinstance(v[0], dict):  # chat-formatted rows
            return str(v[-1].get("content", ""))
        if v:
            return str(v)
    return ""


def _answer(row: Dict[str, Any]):
    rm = row.get("reward_model")
    if isinstance(rm, dict) and rm.get("ground_truth") is not None:
        return rm["ground_truth"]
    return row.get("ground_truth") or row.get("answer") or row.get("solution") or ""


class DAPOMathWorkflow(MultiTurnWorkflow):
    tool_type = "math_validator"

    def __init__(self, reward_fn=dapo_math_reward_fn, tokenizer=None, max_turns: int = 2, **kw):
        super().__init__(reward_fn, tokenizer, max_turns=max_turns, **kw)

    def initial_prompt(self, data):
        q = self.truncate(_question(data), self.max_prompt_tokens)
        return chat(self.tokenizer, [{"role": "system", "content": MATH_SYSTEM}, {"role": "user", "content": q}])

    async def tool_step(self, engine, data, output_text, turn):
        m = evaluate_math_completion(output_text, _answer(data))
        if m["accuracy"] >= 1.0:
            return None
        return "\n" + math_validator_feedback(m) + "\n", {"reward": m["reward"], "status": "failure"}

    def score(self, data, prompt, completion, segments):
        last = self.decode(segments[-1][0]) if segments[-1][2] else completion
        for toks, _, trained in reversed(segments):
            if trained:
                last = self.decode(toks)
                break
        return float(self.reward_fn(prompt=prompt, completion=last, ground_truth=_answer(data)))
