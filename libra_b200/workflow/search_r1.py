"""Search-R1: interleaved reasoning and retrieval (reference ``workflow/search_r1.py``).

A turn that emits ``<search>query</search>`` (or ``<tool_call>query</tool_call>``)
without an answer runs the search tool; the results return inside
``<information>...</information>`` as untrained tokens.  An ``<answer>`` or the
turn budget ends the episode.
"""

from __future__ import annotations

import re

from libra_b200.env.prompts import SEARCH_R1_SYSTEM, chat
from libra_b200.env.rewards import combined_search_r1_reward_fn
from libra_b200.env.search_tool import SearchTool
from libra_b200.workflow.base import MultiTurnWorkflow

_QUERY = re.compile(r"<(search|tool_call)>(.*?)</\1>", re.DOTALL)


class SearchR1Workflow(MultiTurnWorkflow):
    tool_type = "web_search"
    stop = ["</search>", "</tool_call>", "</answer>"]

    def __init__(self, reward_fn=combined_search_r1_reward_fn, tokenizer=None, search_tool=None, max_turns: int = 5,
                 **kw):
        super().__init__(reward_fn, tokenizer, max_turns=max_turns, **kw)
        self.search_tool = search_tool or SearchTool()

    @staticmethod
    def extract_query(text: str):
        m = _QUERY.findall(text or "")
        return m[-1][1].strip() if m and m[-1][1].strip() else None

    def initial_prompt(self, data):
        return chat(self.tokenizer, [{"role": "system", "content": SEARCH_R1_SYSTEM},
                                     {"role": "user", "content": str(data.get("question", ""))}])

    async def tool_step(self, engine, data, output_text, turn):
        if "<answer>" in output_text and "</answer>" in output_text:
            return None
        q = self.extract_query(output_text)
        if q is None:
            return None
        try:
            res, status = await self.search_tool.search(q), "success"
        except Exception as exc:  # noqa: BLE001 - the model sees the error
            res, status = f"Error: {exc}", "failure"
        return f"\n<information>{res}</information>\n", {"status": status, "query": q}

    def score(self, data, prompt, completion, segments):
        gt = data.get("golden_answers") or data.get("ground_truth") or data.get("answer") or ""
        return float(self.reward_fn(prompt=prompt, completion=completion, ground_truth=gt))
