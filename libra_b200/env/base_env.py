"""Chain-of-thought step environment (reference ``env/base_env.py``, legacy).

A problem is revealed one reasoning step at a time: ``reset`` builds the
query, ``step(action)`` appends a step and reports done/reward when the
action contains a final answer (``\\boxed{}`` or the stop string).  Used by
tree-search style data generation, not by the GRPO workflows.
"""

from __future__ import annotations

import copy
from typing import Any, Dict, List, Optional, Sequence

from libra_b200.env.math_grader import extract_answer, math_equal


class NoLegalActionException(Exception):
    pass


class ResetException(Exception):
    pass


class CoTEnv:
    sep = "\n\n"

    def __init__(self, problems: Sequence[Dict[str, Any]], task_desc: str = "", max_steps: int = 16,
                 stop_str: str = "The answer is"):
        self.problems, self.task_desc, self.max_steps, self.stop_str = list(problems), task_desc, max_steps, stop_str
        self.idx = 0
        self.steps: List[str] = []

    def set_problem(self, idx: int) -> None:
        if not 0 <= idx < len(self.problems):
            raise ResetException(f"problem index {idx} out of range")
        self.idx = idx

    @property
    def question(self) -> str:
        return str(self.problems[self.idx].get("question", ""))

    @property
    def answer(self) -> str:
        return str(self.problems[self.idx].get("answer", ""))

    def build_query_str(self) -> str:
        head = (self.task_desc + self.sep) if self.task_desc else ""
        return head + self.question + self.sep + self.sep.join(self.steps)

    def reset(self, idx: Optional[int] = None) -> str:
        if idx is not None:
            self.set_problem(idx)
        self.steps = []
        return self.build_query_str()

    def _final(self, action: str) -> bool:
        return "\\boxed" in action or self.stop_str in action

    def step(self, action: str):
        if len(self.steps) >= self.max_steps:
            raise NoLegalActionException("step budget exhausted")
        self.steps.append(action.strip())
        done = self._final(action) or len(self.steps) >= self.max_steps
        reward = 0.0
        if done:
            pred = extract_answer(action)
            reward = 1.0 if pred and math_equal(pred, self.answer) else 0.0
        return self.build_query_str(), reward, done, {"num_steps": len(self.steps)}

    def copy(self) -> "CoTEnv":
        return copy.deepcopy(self)
