"""Workflows and environment rewards/tools on CPU with a scripted engine."""

import asyncio
import json

import pytest

from libra_b200.engine.tokenizer import ByteTokenizer
from libra_b200.env.code_executor import CodeExecutor, run_sync
from libra_b200.env.math_grader import extract_answer, last_boxed, math_equal
from libra_b200.env.rewards import (code_reward_fn, combined_search_r1_reward_fn, dapo_math_reward_fn,
                                    evaluate_issue, r2e_gym_reward_fn, rlvr_math_reward_fn)
from libra_b200.env.search_tool import BM25Corpus, SearchTool
from libra_b200.workflow.agentic import AgenticWorkflow
from libra_b200.workflow.code_agent import CodeAgentWorkflow
from libra_b200.workflow.dapo_math import DAPOMathWorkflow
from libra_b200.workflow.r2e_gym import R2EGymWorkflow
from libra_b200.workflow.rlvr import RLVRWorkflow
from libra_b200.workflow.search_r1 import SearchR1Workflow


class ScriptedEngine:
    """Returns the scripted texts in order and records the C-MLFQ lifecycle."""

    def __init__(self, tok, texts):
        self.tok, self.texts, self.calls, self.events = tok, list(texts), [], []

    async def generate(self, prompt, max_new_tokens=16, **kw):
        self.calls.append({"prompt": prompt, "max_new_tokens": max_new_tokens, **kw})
        text = self.texts.pop(0)
        ids = self.tok.encode(text, add_special_tokens=False)[:max_new_tokens]
        return {"text": self.tok.decode(ids), "token_ids": ids, "logprobs": [-0.5] * len(ids)}

    def begin_cmlfq_request(self, pid, n):
        self.events.append(("begin", pid, n))
        return "rid-1"

    def route_cmlfq_tool_return(self, rid, event, pos):
        self.events.append(("tool", event["tool_type"], pos))

    def finish_cmlfq_request(self, rid, n):
        self.events.append(("finish", n))

    def cancel_cmlfq_request(self, rid):
        self.events.append(("cancel",))


TOK = ByteTokenizer()


def _check_traj(t):
    L = t["input_ids"].shape[1]
    assert t["loss_mask"].shape == (1, L) and t["logprobs"].shape == (1, L)
    trained = t["loss_mask"][0].bool()
    assert (t["logprobs"][0][trained] == -0.5).all() and (t["logprobs"][0][~trained] == 0).all()
    assert t["prompt_len"] + t["output_len"] == L


def test_math_grader_and_rewards():
    assert last_boxed(r"x \boxed{\frac{3}{4}} y") == r"\frac{3}{4}"
    assert math_equal(r"\frac{3}{4}", "0.75") and math_equal("75%", "0.75") and not math_equal("2", "3")
    assert extract_answer("so the answer is 17") == "17"
    assert dapo_math_reward_fn(completion=r"reasoning ... \boxed{4}", ground_truth="4") == 1.0
    wrong = dapo_math_reward_fn(completion=r"a long enough reasoning chain here \boxed{5}", ground_truth="4")
    assert wrong == pytest.approx(0.05)
    assert rlvr_math_reward_fn(completion="<answer>12</answer>", answer="12") == 1.0
    assert combined_search_r1_reward_fn(completion="<think>t</think><answer>the Eiffel Tower</answer>",
                                        ground_truth=["Eiffel Tower"]) == pytest.approx(1.0 + 0.15 * 0.15)
    m = evaluate_issue("[ISSUE]\nTitle: parse_date crashes\nExpected: a date. Actual: TypeError[/ISSUE]",
                       "parse_date raises TypeError on iso strings",
                       json.dumps({"tests/test_dates.py::test_parse_date_iso": "FAILED"}), ["src/dates/parse_date.py"])
    assert m["format_score"] == 1.0 and m["missing_sections"] == [] and 0 < m["reward"] <= 1
    assert m["reward"] == pytest.approx(0.55 * m["lexical_f1"] + 0.2 * m["test_coverage"] + 0.1 * m["file_coverage"]
                                        + 0.15)


def test_code_sandbox_pass_fail_timeout():
    ex = CodeExecutor(timeout=3)
    rate, meta = run_sync(ex.execute("print(sum(map(int, input().split())))", {"inputs": ["1 2", "5 5"],
                                                                                 "outputs": ["3", "11"]}))
    assert rate == 0.5 and meta["passed"] == 1
    rate, _ = run_sync(ex.execute("def add(a, b):\n    return a + b", {"fn_name": "add", "inputs": [[1, 2]],
                                                                       "outputs": [3]}))
    assert rate == 1.0
    rate, meta = run_sync(ex.execute("import time\ntime.sleep(30)", {"inputs": [""], "outputs": [""]}))
    assert rate == 0.0 and meta["results"] == [-1]
    assert code_reward_fn(completion="no code here", test_cases={"inputs": ["1"], "outputs": ["1"]}) == 0.0


def test_local_search_backend():
    corpus = BM25Corpus([{"title": "Paris", "text": "Paris is the capital of France."},
                         {"title": "Berlin", "text": "Berlin is the capital of Germany."}])
    out = asyncio.run(SearchTool(corpus=corpus, max_results=1).search("capital of France"))
    assert "Paris" in out and "Berlin" not in out
    assert "empty query" in asyncio.run(SearchTool(corpus=corpus).search(""))


def test_rlvr_single_turn():
    eng = ScriptedEngine(TOK, [r"2+2 is \boxed{4}"])
    wf = RLVRWorkflow(tokenizer=TOK, max_new_tokens=64)
    t = asyncio.run(wf.run_episode(eng, {"question": "2+2?", "answer": "4", "prompt_id": "p0"}, version=3))
    _check_traj(t)
    assert float(t["rewards"][0]) == 1.0 and int(t["versions"][0]) == 3 and len(eng.calls) == 1


def test_dapo_math_revises_after_validator():
    eng = ScriptedEngine(TOK, [r"first try \boxed{5}", r"fixed \boxed{4}"])
    wf = DAPOMathWorkflow(tokenizer=TOK, max_turns=3, max_new_tokens=64)
    t = asyncio.run(wf.run_episode(eng, {"question": "2+2?", "ground_truth": "4", "prompt_id": "p"}))
    _check_traj(t)
    assert len(eng.calls) == 2 and t["num_turns"] == 2 and float(t["rewards"][0]) == 1.0
    assert [e[0] for e in eng.events] == ["begin", "tool", "finish"]
    assert t["tool_events"][0]["tool_type"] == "math_validator"


def test_r2e_gym_stops_when_validator_is_satisfied():
    good = "[ISSUE]\nTitle: parse_date TypeError\nExpected a date, actual TypeError in parse_date[/ISSUE]"
    eng = ScriptedEngine(TOK, ["[ISSUE]nothing[/ISSUE]", good, "unused"])
    wf = R2EGymWorkflow(tokenizer=TOK, max_turns=3, stop_reward=0.3, max_new_tokens=256)
    row = {"prompt": "commit details", "target_issue": "parse_date raises TypeError", "repo_name": "r",
           "commit_hash": "c"}
    t = asyncio.run(wf.run_episode(eng, row))
    _check_traj(t)
    assert len(eng.calls) == 2 and eng.calls[0]["stop"] == ["[/ISSUE]"] and t["prompt_id"] == "r:c"
    assert t["tool_events"][0]["remaining_length"] > 0 and float(t["rewards"][0]) >= 0.3


def test_search_r1_calls_tool_then_answers():
    corpus = BM25Corpus([{"title": "Paris", "text": "Paris is the capital of France."}])
    eng = ScriptedEngine(TOK, ["<think>need facts</think><search>capital of France</search>",
                               "<answer>Paris</answer>"])
    wf = SearchR1Workflow(tokenizer=TOK, search_tool=SearchTool(corpus=corpus), max_turns=4, max_new_tokens=128)
    t = asyncio.run(wf.run_episode(eng, {"question": "Capital of France?", "golden_answers": ["Paris"]}))
    _check_traj(t)
    assert "<information>" in eng.calls[1]["prompt"] and float(t["rewards"][0]) > 1.0
    assert t["tool_events"][0]["query"] == "capital of France"


def test_code_agent_runs_code_and_scores_submission():
    eng = ScriptedEngine(TOK, ["```python\nprint(int(input())*2)\n```", "```python\nprint(int(input())*2)\n``` <submit>"])
    wf = CodeAgentWorkflow(tokenizer=TOK, executor=CodeExecutor(timeout=5), max_turns=3, max_new_tokens=128)
    row = {"question": "double it", "test_cases": {"inputs": ["3", "5"], "outputs": ["6", "10"]}}
    t = asyncio.run(wf.run_episode(eng, row))
    _check_traj(t)
    assert "<execution status=success>" in eng.calls[1]["prompt"] and float(t["rewards"][0]) == pytest.approx(1.0)


def test_agentic_tools_and_discount():
    async def lookup(key=""):
        return {"a": "alpha"}.get(key, "?")

    eng = ScriptedEngine(TOK, ['<tool_call>{"name": "lookup", "arguments": {"key": "a"}}</tool_call>', "done: alpha"])
    wf = AgenticWorkflow(lambda prompt, completion, **kw: 1.0 if "alpha" in completion else 0.0, TOK,
                         tools=[{"name": "lookup", "function": lookup}], max_turns=3, discount_factor=0.5,
                         max_new_tokens=128)
    t = asyncio.run(wf.run_episode(eng, {"question": "what is a?"}))
    assert "<tool_response>alpha</tool_response>" in eng.calls[1]["prompt"]
    assert float(t["rewards"][0]) == pytest.approx(0.5)


def test_engine_failure_cancels_cmlfq_request():
    class Boom(ScriptedEngine):
        async def generate(self, prompt, **kw):
            raise RuntimeError("instance died")

    eng = Boom(TOK, [])
    with pytest.raises(RuntimeError):
        asyncio.run(DAPOMathWorkflow(tokenizer=TOK).run_episode(eng, {"question": "q", "ground_truth": "1"}))
    assert eng.events[-1] == ("cancel",)


def test_r2e_length_profile():
    from libra_b200.workflow.r2e_gym_profile import build_r2e_gym_length_profile

    rows = [{"prompt": "x" * (50 * i + 10), "target_issue": "y" * (20 * i + 5), "prompt_id": f"p{i}"} for i in range(6)]
    recs = build_r2e_gym_length_profile(rows, tokenizer=TOK, sample_size=4, max_new_tokens=64)
    assert len(recs) == 4
    assert all(r["output_len"] <= 64 and r["input_len"] > 0 for r in recs)


def test_dataset_evaluation_greedy_and_failures():
    import asyncio

    import torch

    from libra_b200.workflow.evaluation import eval_indices, evaluate_workflow

    assert eval_indices(10, 4, "first") == [0, 1, 2, 3]
    assert eval_indices(10, 4, "spread") == [0, 2, 5, 7]
    assert eval_indices(10, 20, "random") == list(range(10))
    r = eval_indices(10, 3, "random", seed=1)
    assert len(r) == 3 and r == sorted(r) and r == eval_indices(10, 3, "random", seed=1)

    class Wf:
        temperature, top_p, max_new_tokens = 1.0, 0.9, 64
        seen = []

        async def run_episode(self, engine, row, version=0, rollout_index=0):
            Wf.seen.append((self.temperature, self.top_p, self.max_new_tokens))
            if row["x"] == 3:
                raise ValueError("bad row")
            return {"rewards": torch.tensor([row["x"] / 4.0]), "prompt_id": str(row["x"]), "output_len": 2,
                    "completion": "c"}

    wf = Wf()
    ds = [{"x": i} for i in range(5)]
    out = asyncio.run(evaluate_workflow(wf, None, ds, max_samples=0, concurrency=2, accuracy_threshold=0.5,
                                        max_new_tokens=7, record_limit=2))
    assert wf.temperature == 1.0  # the caller's workflow is untouched
    assert set(Wf.seen) == {(0.0, 1.0, 7)}
    assert out["eval_samples"] == 5 and out["eval_failures"] == 1 and "bad row" in out["eval_first_error"]
    # rewards 0, .25, .5, fail(0), 1.0 -> accurate at >= .5: rows 2 and 4
    assert abs(out["eval_accuracy"] - 0.4) < 1e-9
    assert abs(out["eval_reward_mean"] - 1.75 / 5) < 1e-9 and out["eval_reward_max"] == 1.0
    assert len(out["eval_records"]) == 2 and out["eval_records"][1]["accurate"] is False


def test_rollout_index_gives_distinct_reproducible_seeds():
    """The GRPO group's members (rollout_index) sample with distinct seeds; the
    same (prompt, version, index, turn) always gets the same seed."""
    eng = ScriptedEngine(TOK, ["[ISSUE]a[/ISSUE]"] * 3)
    wf = R2EGymWorkflow(tokenizer=TOK, max_turns=1, max_new_tokens=32, temperature=0.8, top_p=0.95)
    row = {"prompt": "commit details", "target_issue": "x", "repo_name": "r", "commit_hash": "c"}
    for idx in (0, 1, 0):
        asyncio.run(wf.run_episode(eng, row, version=3, rollout_index=idx))
    first, second, again = [c["seed"] for c in eng.calls]
    assert first != second and first == again
    assert all(c["temperature"] == 0.8 and c["top_p"] == 0.95 for c in eng.calls)
