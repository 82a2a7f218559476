"""Reward functions of the workflows.

All share the reference call convention ``fn(prompt=..., completion=..., **row)
-> float`` (``workflow/rlvr.py:80-86``).  Component weights are the reference's
(``env/dapo_math_reward.py:45-65``, ``env/search_r1_reward.py:57-90``,
``env/r2e_gym_reward.py:119-124``, ``env/code_reward.py:35-138``) so rewards are
comparable between the two frameworks; the code is our own.
"""

from __future__ import annotations

import ast
import json
import re
import string
from typing import Any, Dict, Iterable, List, Optional, Sequence, Union

from libra_b200.env.math_grader import extract_answer, last_boxed, math_equal

Answers = Union[str, Sequence[str]]


def _answers(gt: Answers) -> List[str]:
    if gt is None or gt == "":
        return []
    return [str(a) for a in gt] if isinstance(gt, (list, tuple)) else [str(gt)]


def _squash(s: str, drop_articles: bool = False) -> str:
    s = str(s or "").lower()
    s = "".join(ch for ch in s if ch not in string.punctuation.replace("/", "") or ch == "/")
    if drop_articles:
        s = re.sub(r"\b(a|an|the)\b", " ", s)
    return " ".join(s.split())


def _matches(pred: str, gt: Answers, drop_articles: bool = False) -> bool:
    for a in _answers(gt):
        if math_equal(pred, a, timeout=True) or _squash(pred, drop_articles) == _squash(a, drop_articles):
            return True
    return False


# ----------------------------------------------------------------------------- math (DAPO / RLVR)
_TAG = re.compile(r"<answer>(.*?)</answer>", re.DOTALL | re.IGNORECASE)


def extract_math_answer(text: str) -> str:
    tags = _TAG.findall(text or "")
    if tags:
        return tags[-1].strip()
    boxed = last_boxed(text or "")
    if boxed is not None:
        return boxed.strip()
    return extract_answer(text or "", "math")


def evaluate_math_completion(completion: str, ground_truth: Answers) -> Dict[str, Any]:
    pred = extract_math_answer(completion)
    correct = bool(pred) and _matches(pred, ground_truth)
    fmt = min(1.0, 0.35 * bool(pred) + 0.45 * ("\\boxed" in (completion or ""))
              + 0.20 * (len(completion or "") > len(pred) + 20))
    return {"reward": 1.0 if correct else 0.05 * fmt, "accuracy": float(correct), "prediction": pred,
            "format_score": fmt, "has_boxed": "\\boxed" in (completion or "")}


def math_validator_feedback(m: Dict[str, Any]) -> str:
    return ("### Math validator\n"
            f"status={'correct' if m['accuracy'] >= 1 else 'incorrect'} reward={m['reward']:.3f} "
            f"prediction={m['prediction'] or '<empty>'} format={m['format_score']:.2f}\n"
            "Check the reasoning and give the final answer once inside \\boxed{} at the end.")


def dapo_math_reward_fn(prompt: str = "", completion: str = "", ground_truth: Answers = "", answer: Answers = "",
                        **_) -> float:
    return float(evaluate_math_completion(completion, ground_truth or answer)["reward"])


def rlvr_math_reward_fn(prompt: str = "", completion: str = "", answer: Answers = "", ground_truth: Answers = "",
                        **_) -> float:
    """Binary verifiable reward: 1 when the extracted answer matches."""
    pred = extract_math_answer(completion)
    return 1.0 if pred and _matches(pred, answer or ground_truth) else 0.0


# ----------------------------------------------------------------------------- Search-R1
def _first(pattern: str, text: str) -> str:
    m = re.search(pattern, text or "", re.DOTALL)
    return m.group(1).strip() if m else ""


def extract_search_r1_answer(text: str) -> str:
    return _first(r"<answer>(.*?)</answer>", text)


def extract_search_r1_think(text: str) -> str:
    return _first(r"<think>(.*?)</think>", text) or _first(r"<thinking>(.*?)</thinking>", text)


def search_r1_reward_fn(prompt: str = "", completion: str = "", ground_truth: Answers = "", **_) -> float:
    ans = extract_search_r1_answer(completion)
    return 1.0 if ans and _matches(ans, ground_truth, drop_articles=True) else 0.0


def format_reward_fn(completion: str) -> float:
    r = 0.1 if ("<answer>" in completion and "</answer>" in completion) else 0.0
    r += 0.05 if ("<think>" in completion or "<thinking>" in completion) else 0.0
    return min(r, 0.15)


def combined_search_r1_reward_fn(prompt: str = "", completion: str = "", ground_truth: Answers = "",
                                 format_weight: float = 0.15, **kw) -> float:
    return search_r1_reward_fn(prompt, completion, ground_truth) + format_weight * format_reward_fn(completion)


# ----------------------------------------------------------------------------- R2E-Gym issue generation
_WORD = re.compile(r"[A-Za-z_][A-Za-z0-9_]{2,}")
_ISSUE = re.compile(r"\[ISSUE\](.*?)\[/ISSUE\]", re.DOTALL | re.IGNORECASE)
_COMMON = frozenset("the and for with that this from are but not when into should expected actual behavior "
                    "description issue test tests code output".split())


def _words(text: str) -> set:
    return {w.lower() for w in _WORD.findall(text or "") if w.lower() not in _COMMON}


def extract_issue_text(completion: str) -> str:
    found = _ISSUE.findall(completion or "")
    return found[-1].strip() if found else (completion or "")


def _json_dict(x) -> Dict[str, str]:
    if isinstance(x, dict):
        return {str(k): str(v) for k, v in x.items()}
    try:
        d = json.loads(x) if x else {}
    except (TypeError, ValueError):
        return {}
    return {str(k): str(v) for k, v in d.items()} if isinstance(d, dict) else {}


def _f1(a: set, b: set) -> float:
    if not a or not b:
        return 0.0
    hit = len(a & b)
    if hit == 0:
        return 0.0
    p, r = hit / len(a), hit / len(b)
    return 2 * p * r / (p + r)


def _parts(names: Iterable[str], split: str) -> set:
    return {p.lower() for n in names for p in re.split(split, str(n)) if len(p) >= 3}


def evaluate_issue(completion: str, target_issue: str, expected_output_json=None, modified_files=None) -> Dict[str, Any]:
    issue = extract_issue_text(completion)
    pred = _words(issue)
    f1 = _f1(pred, _words(target_issue))
    tests = _json_dict(expected_output_json)
    tnames = _parts(tests, r"[.:_\[\]\s]+")
    test_cov = len(tnames & pred) / len(tnames) if tnames else 0.0
    if isinstance(modified_files, str):
        try:
            modified_files = json.loads(modified_files)
        except ValueError:
            modified_files = [modified_files]
    fparts = _parts(modified_files or [], r"[/_.\-]+")
    file_cov = len(fparts & pred) / len(fparts) if fparts else 0.0
    checks = {"[ISSUE] tags": bool(_ISSUE.search(completion or "")),
              "title": bool(re.search(r"(title:|^#|\*\*title:\*\*)", issue, re.IGNORECASE | re.MULTILINE)),
              "expected behavior": "expected" in issue.lower(),
              "actual behavior/error": "actual" in issue.lower() or "error" in issue.lower()}
    fmt = sum(checks.values()) / 4.0
    reward = max(0.0, min(1.0, 0.55 * f1 + 0.20 * test_cov + 0.10 * file_cov + 0.15 * fmt))
    return {"reward": reward, "lexical_f1": f1, "test_coverage": test_cov, "file_coverage": file_cov,
            "format_score": fmt, "issue_length": len(issue), "n_expected_tests": len(tests),
            "missing_sections": [k for k, ok in checks.items() if not ok]}


def issue_validator_feedback(m: Dict[str, Any]) -> str:
    return ("### R2E-Gym issue validator\n"
            f"reward={m['reward']:.3f} lexical_f1={m['lexical_f1']:.3f} test_coverage={m['test_coverage']:.3f} "
            f"file_coverage={m['file_coverage']:.3f} format={m['format_score']:.3f}\n"
            f"missing={', '.join(m['missing_sections']) or 'none'}\n"
            "Revise the issue: concise, concrete and faithful to the failing behaviour.")


def r2e_gym_reward_fn(prompt: str = "", completion: str = "", target_issue: str = "", expected_output_json=None,
                      modified_files=None, **_) -> float:
    return float(evaluate_issue(completion, target_issue, expected_output_json, modified_files)["reward"])


# ----------------------------------------------------------------------------- code
def extract_code_block(text: str) -> Optional[str]:
    blocks = re.findall(r"```([A-Za-z0-9_+-]*)\n(.*?)```", text or "", re.DOTALL)
    if blocks:
        py = [b for lang, b in blocks if lang.lower() in ("python", "py", "python3")]
        return (py or [b for _, b in blocks])[-1].strip()
    return None


def code_reward_fn(prompt: str = "", completion: str = "", test_cases: Optional[Dict[str, Any]] = None,
                   executor=None, continuous: bool = True, format_weight: float = 0.0, **_) -> float:
    from libra_b200.env.code_executor import CodeExecutor, run_sync

    code = extract_code_block(completion)
    if not code:
        return format_weight
    ex = executor or CodeExecutor(mode="local", timeout=10)
    try:
        rate, _meta = run_sync(ex.execute(code, test_cases or {}))
    except Exception:  # noqa: BLE001 - an executor failure scores as no test passed
        rate = 0.0
    if continuous:
        return rate * (1.0 - format_weight) + format_weight
    full = 1.0 if rate >= 1.0 - 1e-6 else 0.0
    return full * (1.0 - format_weight) + format_weight if format_weight > 0 else full


def combined_code_reward_fn(prompt: str = "", completion: str = "", test_cases=None, executor=None,
                            format_weight: float = 0.1, compile_bonus: float = 0.0, **kw) -> float:
    r = code_reward_fn(prompt, completion, test_cases, executor, True, format_weight)
    if compile_bonus > 0:
        code = extract_code_block(completion)
        if code:
            try:
                ast.parse(code)
                r += compile_bonus
            except SyntaxError:
                pass
    return min(r, 1.0)


def make_code_reward_fn(executor=None, continuous: bool = True, format_weight: float = 0.1,
                        compile_bonus: float = 0.0):
    def fn(prompt: str = "", completion: str = "", **row) -> float:
        if not row.get("test_cases"):
            return 0.0
        return combined_code_reward_fn(prompt, completion, row["test_cases"], executor, format_weight, compile_bonus)

    return fn


REWARD_FUNCTIONS = {"dapo_math": dapo_math_reward_fn, "math": rlvr_math_reward_fn, "gsm8k": rlvr_math_reward_fn,
                    "search_r1": combined_search_r1_reward_fn, "r2e_gym": r2e_gym_reward_fn,
                    "code": make_code_reward_fn()}
