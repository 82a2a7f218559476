"""Single-turn RL with a verifiable reward (reference ``workflow/rlvr.py``)."""

from __future__ import annotations

from typing import Any, Dict

from libra_b200.env.prompts import MATH_SYSTEM, chat
from libra_b200.env.rewards import rlvr_math_reward_fn
from libra_b200.workflow.base import MultiTurnWorkflow


class RLVRWorkflow(MultiTurnWorkflow):
    def __init__(self, reward_fn=rlvr_math_reward_fn, tokenizer=None, max_new_tokens: int = 1024,
                 temperature: float = 1.0, n_samples: int = 4, max_seq_length: int = 8192, **kw):
        super().__init__(reward_fn, tokenizer, max_turns=1, max_new_tokens=max_new_tokens,
                         max_seq_length=max_seq_length, temperature=temperature, n_samples=n_samples, **kw)

    def initial_prompt(self, data: Dict[str, Any]) -> str:
        q = self.truncate(str(data.get("question") or data.get("problem") or data.get("prompt", "")),
                          self.max_prompt_tokens)
        return chat(self.tokenizer, [{"role": "system", "content": MATH_SYSTEM}, {"role": "user", "content": q}])
