"""Generic tool-calling agent (reference ``workflow/agentic.py``).

Tools are ``{"name": str, "function": async callable}``.  A turn calls tools
with ``<tool_call>{"name": ..., "arguments": {...}}</tool_call>`` (JSON); the
results return as ``<tool_response>`` blocks.  A turn without a tool call is
the final answer.  ``discount_factor`` scales the reward by gamma^(tool turns).
"""

from __future__ import annotations

import json
import re

from libra_b200.env.prompts import chat
from libra_b200.workflow.base import MultiTurnWorkflow

_CALL = re.compile(r"<tool_call>(.*?)</tool_call>", re.DOTALL)


class AgenticWorkflow(MultiTurnWorkflow):
    tool_type = "agent_tool"

    def __init__(self, reward_fn, tokenizer, tools=None, max_turns: int = 5, max_new_tokens: int = 512,
                 temperature: float = 1.0, discount_factor: float = 0.9, **kw):
        super().__init__(reward_fn, tokenizer, max_turns=max_turns, max_new_tokens=max_new_tokens,
                         temperature=temperature, **kw)
        self.tools = {t["name"]: t for t in (tools or [])}
        self.discount_factor = discount_factor

    def initial_prompt(self, data):
        msgs = list(data.get("messages") or [{"role": "user", "content": str(data.get("question", ""))}])
        if self.tools:
            spec = ", ".join(sorted(self.tools))
            msgs = [{"role": "system", "content": f"Tools: {spec}. Call one as <tool_call>{{\"name\": ..., "
                                                  f"\"arguments\": {{...}}}}</tool_call>."}] + msgs
        return chat(self.tokenizer, msgs)

    @staticmethod
    def parse_calls(text: str):
        calls = []
        for raw in _CALL.findall(text or ""):
            try:
                obj = json.loads(raw)
                calls.append({"name": str(obj.get("name", "")), "arguments": dict(obj.get("arguments") or {})})
            except (ValueError, AttributeError):
                calls.append({"name": raw.strip(), "arguments": {}})
        return calls

    async def tool_step(self, engine, data, output_text, turn):
        calls = self.parse_calls(output_text)
        if not calls:
            return None
        outs, status = [], "success"
        for c in calls:
            tool = self.tools.get(c["name"])
            if tool is None:
                outs.append(f"Tool not found: {c['name']}")
                status = "failure"
                continue
            try:
                outs.append(str(await tool["function"](**c["arguments"])))
            except Exception as exc:  # noqa: BLE001 - the model sees the error
                outs.append(f"Error: {exc}")
                status = "failure"
        return "".join(f"\n<tool_response>{o}</tool_response>" for o in outs) + "\n", {"status": status,
                                                                                       "n_calls": len(calls)}

    def score(self, data, prompt, completion, segments):
        r = super().score(data, prompt, completion, segments)
        tool_turns = sum(1 for s in segments[1:] if not s[2])
        return r * (self.discount_factor ** tool_turns) if self.discount_factor < 1.0 else r
