"""Convert benchmark datasets into workflow rows (JSONL).

Roles of the reference's ``data/prepare_r2e_gym.py``, ``prepare_search_r1.py``,
``preprocess_livecodebench.py`` and ``download_gsm8k.py``.  Inputs are local
files (JSONL, JSON list or Parquet) since this box has no network; the output
row schema is what the workflows consume:

* gsm8k / math / dapo_math: ``question``, ``answer`` / ``ground_truth``
* r2e_gym: ``prompt``, ``target_issue``, ``expected_output_json``, ``modified_files``, ``prompt_id``
* search_r1: ``question``, ``golden_answers``
* livecodebench / code: ``question``, ``starter_code``, ``test_cases`` ({inputs, outputs[, fn_name]})

    python -m libra_b200.data.prepare gsm8k --input train.jsonl --output data/gsm8k.jsonl
"""

from __future__ import annotations

import argparse
import base64
import json
import os
import pickle  # noqa: S403 - only for LiveCodeBench's own compressed test files, never network input
import re
import zlib
from typing import Any, Dict, Iterable, Iterator, List


def read_rows(path: str) -> List[Dict[str, Any]]:
    if path.endswith(".parquet"):
        import pyarrow.parquet as pq

        return pq.read_table(path).to_pylist()
    with open(path, encoding="utf-8") as f:
        text = f.read()
    if text.lstrip().startswith("["):
        return list(json.loads(text))
    return [json.loads(line) for line in text.splitlines() if line.strip()]


def write_rows(rows: Iterable[Dict[str, Any]], path: str) -> int:
    os.makedirs(os.path.dirname(os.path.abspath(path)), exist_ok=True)
    n = 0
    with open(path, "w", encoding="utf-8") as f:
        for r in rows:
            f.write(json.dumps(r, ensure_ascii=False) + "\n")
            n += 1
    return n


def gsm8k_rows(rows) -> Iterator[Dict[str, Any]]:
    for i, r in enumerate(rows):
        ans = str(r.get("answer", ""))
        final = ans.split("####")[-1].strip().replace(",", "") if "####" in ans else ans.strip()
        yield {"prompt_id": f"gsm8k-{i}", "question": r.get("question", ""), "answer": final, "solution": ans}


def math_rows(rows) -> Iterator[Dict[str, Any]]:
    from libra_b200.env.math_grader import last_boxed

    for i, r in enumerate(rows):
        gt = r.get("answer") or r.get("ground_truth")
        if gt is None and r.get("solution"):
            gt = last_boxed(str(r["solution"])) or ""
        rm = r.get("reward_model")
        if isinstance(rm, dict) and rm.get("ground_truth") is not None:
            gt = rm["ground_truth"]
        q = r.get("problem") or r.get("question") or r.get("prompt")
        if isinstance(q, list) and q and isinstance(q[-1], dict):
            q = q[-1].get("content", "")
        yield {"prompt_id": str(r.get("id", f"math-{i}")), "question": q, "ground_truth": gt, "answer": gt}


def r2e_gym_rows(rows) -> Iterator[Dict[str, Any]]:
    for i, r in enumerate(rows):
        files = r.get("modified_files") or r.get("modified_entity_summaries") or []
        if isinstance(files, str):
            try:
                files = json.loads(files)
            except ValueError:
                files = [files]
        files = [f.get("file_name", f) if isinstance(f, dict) else str(f) for f in files]
        tests = r.get("expected_output_json") or r.get("execution_result_content") or "{}"
        prompt = r.get("prompt") or "\n\n".join(str(x) for x in (r.get("commit_message", ""), r.get("diff", ""),
                                                                  r.get("parsed_commit_content", "")) if x)
        yield {"prompt_id": f"{r.get('repo_name', 'repo')}:{r.get('commit_hash', i)}", "prompt": prompt,
               "target_issue": r.get("problem_statement") or r.get("target_issue", ""),
               "expected_output_json": tests if isinstance(tests, str) else json.dumps(tests),
               "modified_files": files, "repo_name": r.get("repo_name", ""), "commit_hash": r.get("commit_hash", "")}


def search_r1_rows(rows) -> Iterator[Dict[str, Any]]:
    for i, r in enumerate(rows):
        gold = r.get("golden_answers") or r.get("answers") or r.get("answer") or []
        if isinstance(gold, str):
            gold = [gold]
        q = str(r.get("question", "")).strip()
        if q and not q.endswith("?"):
            q += "?"
        yield {"prompt_id": str(r.get("id", f"q-{i}")), "question": q, "golden_answers": list(gold),
               "data_source": r.get("data_source", "")}


def _lcb_tests(raw) -> List[Dict[str, Any]]:
    if isinstance(raw, list):
        return raw
    try:
        return json.loads(raw)
    except (TypeError, ValueError):
        # LiveCodeBench ships private tests as base64(zlib(pickle(json string)))
        return json.loads(pickle.loads(zlib.decompress(base64.b64decode(raw))))  # noqa: S301


def livecodebench_rows(rows) -> Iterator[Dict[str, Any]]:
    for i, r in enumerate(rows):
        tests = _lcb_tests(r.get("public_test_cases") or "[]") + _lcb_tests(r.get("private_test_cases") or "[]")
        meta = r.get("metadata") or {}
        if isinstance(meta, str):
            meta = json.loads(meta or "{}")
        tc = {"inputs": [t["input"] for t in tests], "outputs": [t["output"] for t in tests]}
        if meta.get("func_name"):
            tc["fn_name"] = meta["func_name"]
            tc["inputs"] = [[json.loads(x) for x in t.splitlines() if x.strip()] for t in tc["inputs"]]
            tc["outputs"] = [json.loads(o) for o in tc["outputs"]]
        yield {"prompt_id": str(r.get("question_id", i)), "question": r.get("question_content", ""),
               "starter_code": r.get("starter_code", ""), "test_cases": tc,
               "difficulty": r.get("difficulty", ""), "platform": r.get("platform", "")}


CONVERTERS = {"gsm8k": gsm8k_rows, "math": math_rows, "dapo_math": math_rows, "r2e_gym": r2e_gym_rows,
              "search_r1": search_r1_rows, "livecodebench": livecodebench_rows, "code": livecodebench_rows}


def main(argv=None) -> None:
    ap = argparse.ArgumentParser(description="convert a dataset file into workflow rows")
    ap.add_argument("kind", choices=sorted(CONVERTERS))
    ap.add_argument("--input", required=True)
    ap.add_argument("--output", required=True)
    ap.add_argument("--limit", type=int, default=0)
    a = ap.parse_args(argv)
    rows = read_rows(a.input)
    if a.limit:
        rows = rows[:a.limit]
    n = write_rows(CONVERTERS[a.kind](rows), a.output)
    print(json.dumps({"kind": a.kind, "rows": n, "output": a.output}))


if __name__ == "__main__":
    main()
