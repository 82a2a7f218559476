"""R2E-Gym issue generation with validator feedback (reference ``workflow/r2e_gym.py:27-499``).

The model drafts a GitHub issue inside [ISSUE]...[/ISSUE]; the validator
scores it (lexical F1 against the real issue, coverage of the failing tests
and modified files, format) and, unless the score reaches ``stop_reward`` or
the turn budget is spent, its report comes back as a tool return that C-MLFQ
routes.
"""

from __future__ import annotations

from libra_b200.env.prompts import R2E_ISSUE_SYSTEM, chat
from libra_b200.env.rewards import evaluate_issue, issue_validator_feedback, r2e_gym_reward_fn
from libra_b200.workflow.base import MultiTurnWorkflow


def target_issue(row) -> str:
    return str(row.get("target_issue") or row.get("task_text") or row.get("problem_statement") or "")


class R2EGymWorkflow(MultiTurnWorkflow):
    tool_type = "r2e_issue_validator"
    stop = ["[/ISSUE]"]

    def __init__(self, reward_fn=r2e_gym_reward_fn, tokenizer=None, max_turns: int = 3, max_new_tokens: int = 2048,
                 max_seq_length: int = 8192, stop_reward: float = 0.5, **kw):
        if not 0.0 <= stop_reward <= 1.0:
            raise ValueError("stop_reward must be between 0 and 1")
        super().__init__(reward_fn, tokenizer, max_turns=max_turns, max_new_tokens=max_new_tokens,
                         max_seq_length=max_seq_length, **kw)
        self.stop_reward = float(stop_reward)

    @staticmethod
    def prompt_id(data) -> str:
        return str(data.get("prompt_id") or f"{data.get('repo_name', 'repo')}:{data.get('commit_hash', '')}")

    def initial_prompt(self, data):
        task = self.truncate(str(data.get("prompt") or data.get("problem_statement") or data.get("task_text") or ""),
                             self.max_prompt_tokens)
        return chat(self.tokenizer, [{"role": "system", "content": R2E_ISSUE_SYSTEM}, {"role": "user", "content": task}])

    async def tool_step(self, engine, data, output_text, turn):
        m = evaluate_issue(output_text, target_issue(data), data.get("expected_output_json"),
                           data.get("modified_files"))
        if m["reward"] >= self.stop_reward:
            return None
        return "\n" + issue_validator_feedback(m) + "\n", {"reward": m["reward"], "status": "failure"}

    def score(self, data, prompt, completion, segments):
        last = ""
        for toks, _, trained in reversed(segments):
            if trained:
                last = self.decode(toks)
                break
        return float(self.reward_fn(prompt=prompt, completion=last, target_issue=target_issue(data),
                                    expected_output_json=data.get("expected_output_json"),
                                    modified_files=data.get("modified_files")))
