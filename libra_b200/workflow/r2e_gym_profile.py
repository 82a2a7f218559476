"""Startup length profile for R2E-Gym (reference ``workflow/r2e_gym_profile.py``).

Prompt lengths are the tokenized initial prompts the workflow will send;
output lengths are estimated from the real target issues wrapped in the
workflow's [ISSUE] delimiters, capped at the generation budget.  The records
feed the planner's startup history.
"""

from __future__ import annotations

from typing import Any, Dict, List, Optional

from libra_b200.infra.cost_model.startup_profile import build_length_profile
from libra_b200.workflow.r2e_gym import R2EGymWorkflow, target_issue


def estimate_issue_tokens(tokenizer, row: Dict[str, Any]) -> int:
    issue = target_issue(row).strip()
    if not issue:
        return 1
    if not issue.startswith("[ISSUE]"):
        issue = "[ISSUE]\n" + issue
    if "[/ISSUE]" not in issue:
        issue = issue.rstrip() + "\n[/ISSUE]"
    return len(tokenizer.encode(issue, add_special_tokens=False))


def build_r2e_gym_length_profile(rows: List[Dict[str, Any]], *, tokenizer, sample_size: int, strategy: str = "spread",
                                 seed: int = 0, samples_per_prompt: int = 1, max_turns: int = 3,
                                 max_new_tokens: int = 2048, max_seq_length: int = 8192,
                                 max_prompt_tokens: Optional[int] = None) -> List[Dict[str, Any]]:
    wf = R2EGymWorkflow(tokenizer=tokenizer, max_turns=max_turns, max_new_tokens=max_new_tokens,
                        max_seq_length=max_seq_length, max_prompt_tokens=max_prompt_tokens)
    return build_length_profile(rows, prompt_length_fn=lambda r: len(wf.encode(wf.initial_prompt(r))),
                                output_length_fn=lambda r: estimate_issue_tokens(tokenizer, r),
                                sample_size=sample_size, strategy=strategy, seed=seed,
                                samples_per_prompt=samples_per_prompt, max_output_len=max_new_tokens)
