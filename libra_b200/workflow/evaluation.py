"""Dataset-level evaluation shared by every workflow.

Behaviour of the reference's ``workflow/dapo_math.py:241-288`` and
``workflow/r2e_gym.py:306`` (``evaluate(engine, dataset, max_samples,
concurrency, accuracy_threshold, max_new_tokens)``): pick the rows
(``first`` / ``spread`` / ``random``), run one greedy episode per row under a
concurrency bound, count a row as accurate when its reward reaches the
threshold, and return the ``eval_*`` summary plus up to ``record_limit``
sample records.  A row whose episode raises is a failure with reward 0.

The episode itself is the workflow's own ``run_episode`` on a shallow copy
whose sampling is switched to greedy (temperature 0, top-p 1) and whose
per-turn generation budget is ``max_new_tokens`` when given.
"""

from __future__ import annotations

import asyncio
import copy
import random
from typing import Any, Dict, List, Optional


def eval_indices(n_total: int, n_eval: int, strategy: str = "first", seed: int = 0) -> List[int]:
    """Row indices to evaluate: all rows, the first ``n_eval``, ``n_eval``
    evenly spread over the dataset, or a seeded random sample (sorted)."""
    if n_eval >= n_total:
        return list(range(n_total))
    if strategy == "first":
        return list(range(n_eval))
    if strategy == "random":
        return sorted(random.Random(seed).sample(range(n_total), n_eval))
    if strategy != "spread":
        raise ValueError(f"unknown evaluation strategy: {strategy!r}")
    return sorted({(i * n_total) // n_eval for i in range(n_eval)})


def greedy_copy(workflow, max_new_tokens: Optional[int]):
    wf = copy.copy(workflow)
    if hasattr(wf, "temperature"):
        wf.temperature = 0.0
    if hasattr(wf, "top_p"):
        wf.top_p = 1.0
    if max_new_tokens and max_new_tokens > 0 and hasattr(wf, "max_new_tokens"):
        wf.max_new_tokens = int(max_new_tokens)
    return wf


async def evaluate_workflow(workflow, engine, dataset, max_samples: Optional[int] = None, concurrency: int = 16,
                            accuracy_threshold: float = 1.0, max_new_tokens: Optional[int] = None,
                            strategy: str = "first", seed: int = 0, record_limit: int = 8) -> Dict[str, Any]:
    n_total = len(dataset)
    n_eval = n_total if max_samples is None or max_samples <= 0 else min(int(max_samples), n_total)
    rows = eval_indices(n_total, n_eval, strategy, seed)
    wf = greedy_copy(workflow, max_new_tokens)
    sem = asyncio.Semaphore(max(1, int(concurrency)))

    async def one(i: int) -> Dict[str, Any]:
        row = dataset[int(i)]
        async with sem:
            try:
                traj = await wf.run_episode(engine, row, version=0, rollout_index=0)
            except Exception as exc:  # noqa: BLE001 - counted as a failed row
                return {"index": int(i), "ok": False, "reward": 0.0, "error": f"{type(exc).__name__}: {exc}"}
        reward = float(traj["rewards"].reshape(-1)[0])
        return {"index": int(i), "ok": True, "reward": reward,
                "prompt_id": str(traj.get("prompt_id", "")), "output_len": int(traj.get("output_len", 0)),
                "num_turns": int(traj.get("num_turns", 1)), "completion": str(traj.get("completion", ""))[:4096]}

    results = await asyncio.gather(*(one(i) for i in rows))
    rewards = [r["reward"] for r in results]
    accurate = [1.0 if r["ok"] and r["reward"] >= accuracy_threshold else 0.0 for r in results]
    failures = [r for r in results if not r["ok"]]
    n = max(1, len(results))
    records = []
    for r, acc in zip(results[:max(0, int(record_limit))], accurate):
        records.append({**r, "accurate": bool(acc)})
    return {"eval_samples": len(results), "eval_total_rows": n_total, "eval_mode": f"greedy_{strategy}",
            "eval_accuracy_threshold": float(accuracy_threshold), "eval_accuracy": sum(accurate) / n,
            "eval_reward_mean": sum(rewards) / n, "eval_reward_min": min(rewards) if rewards else 0.0,
            "eval_reward_max": max(rewards) if rewards else 0.0, "eval_failures": len(failures),
            "eval_first_error": failures[0]["error"] if failures else "", "eval_records": records}
