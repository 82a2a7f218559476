"""Code agent: write, run, revise, submit (reference ``workflow/code_agent.py``).

A turn with a ```python block and no ``<submit>`` runs the code in the sandbox
(on the row's first test input when there is one); stdout/stderr return as a
tool result.  ``<submit>`` or the turn budget ends the episode; the reward is
the test pass rate of the last code block.
"""

from __future__ import annotations

from libra_b200.env.code_executor import CodeExecutor
from libra_b200.env.prompts import CODE_AGENT_SYSTEM, chat
from libra_b200.env.rewards import extract_code_block, make_code_reward_fn
from libra_b200.workflow.base import MultiTurnWorkflow


class CodeAgentWorkflow(MultiTurnWorkflow):
    tool_type = "code_execution"

    def __init__(self, reward_fn=None, tokenizer=None, executor=None, max_turns: int = 4, **kw):
        self.executor = executor or CodeExecutor(mode="local", timeout=10)
        super().__init__(reward_fn or make_code_reward_fn(self.executor), tokenizer, max_turns=max_turns, **kw)

    def initial_prompt(self, data):
        task = str(data.get("question") or data.get("prompt") or "")
        if data.get("starter_code"):
            task += "\n\nStarter code:\n```python\n" + str(data["starter_code"]) + "\n```"
        return chat(self.tokenizer, [{"role": "system", "content": CODE_AGENT_SYSTEM},
                                     {"role": "user", "content": self.truncate(task, self.max_prompt_tokens)}])

    async def tool_step(self, engine, data, output_text, turn):
        if "<submit>" in output_text:
            return None
        code = extract_code_block(output_text)
        if not code:
            return None
        tc = data.get("test_cases") or {}
        stdin = str((tc.get("inputs") or [""])[0]) if not tc.get("fn_name") else ""
        r = await self.executor.run(code, stdin)
        body = (r.get("stdout", "")[-2000:] + ("\n[stderr]\n" + r["stderr"][-1000:] if r.get("stderr") else ""))
        return f"\n<execution status={r['status']}>\n{body}\n</execution>\n", {"status": r["status"]}

    def score(self, data, prompt, completion, segments):
        return float(self.reward_fn(prompt=prompt, completion=completion, **{k: v for k, v in data.items()
                                                                             if k not in ("prompt", "completion")}))
