"""Startup length profile for the planner (reference ``infra/cost_model/startup_profile.py``).

Samples dataset rows (``spread`` = evenly spaced, ``random`` = seeded,
``first``), turns each into ``{input_len, output_len, prompt_id, ...}``
history records, summarises percentiles, and decides whether an existing
profile on disk can be reused (same model, dataset, sampling parameters).
"""

from __future__ import annotations

import json
import math
import random
from pathlib import Path
from typing import Any, Callable, Dict, Iterable, List, Optional, Sequence

LengthFn = Callable[[Dict[str, Any]], int]
PROFILE_KEYS = ("model_path", "dataset", "sample_size", "strategy", "seed", "samples_per_prompt", "max_output_len")


def load_jsonl_rows(path, *, limit: int = 0) -> List[dict]:
    rows = []
    with open(path, "r", encoding="utf-8") as fh:
        for line in fh:
            line = line.strip()
            if not line:
                continue
            obj = json.loads(line)
            if isinstance(obj, dict):
                rows.append(obj)
            if limit and len(rows) >= limit:
                break
    return rows


def _as_record(d: dict) -> Optional[dict]:
    p = d.get("input_len", d.get("prompt_length", d.get("prompt_len")))
    g = d.get("output_len", d.get("gen_length", d.get("response_len")))
    try:
        p, g = int(p), int(g)
    except (TypeError, ValueError):
        return None
    if p <= 0 and g <= 0:
        return None
    rec = {"input_len": max(1, p), "output_len": max(1, g)}
    if d.get("prompt_id") is not None:
        rec["prompt_id"] = str(d["prompt_id"])
    return rec


def load_length_profile_records(path) -> List[dict]:
    """Accepts flat profile rows or history StepRecord rows (with ``raw_lengths``/``sequences``)."""
    out = []
    for row in load_jsonl_rows(path):
        rec = _as_record(row)
        if rec is not None:
            out.append(rec)
            continue
        for seq in row.get("sequences", []) or []:
            r = _as_record(seq) if isinstance(seq, dict) else None
            if r is not None:
                out.append(r)
        raw = row.get("raw_lengths") or {}
        for p, g in zip(raw.get("input_lens", []), raw.get("output_lens", [])):
            r = _as_record({"input_len": p, "output_len": g})
            if r is not None:
                out.append(r)
    return out


def profile_jsonl_has_records(path) -> bool:
    try:
        return bool(load_length_profile_records(path))
    except (OSError, ValueError):
        return False


def load_profile_summary(path) -> Optional[dict]:
    try:
        return json.loads(Path(path).read_text(encoding="utf-8"))
    except (OSError, ValueError):
        return None


def startup_profile_metadata(**kw) -> dict:
    return {k: kw.get(k) for k in PROFILE_KEYS}


def profile_metadata_matches(a: Optional[dict], b: Optional[dict]) -> bool:
    if not a or not b:
        return False
    return all(a.get(k) == b.get(k) for k in PROFILE_KEYS)


def profile_summary_matches(summary: Optional[dict], metadata: dict) -> bool:
    return bool(summary) and profile_metadata_matches(summary.get("metadata"), metadata)


def sample_indices(total: int, sample_size: int, *, strategy: str = "spread", seed: int = 0) -> List[int]:
    total, k = max(0, int(total)), max(0, int(sample_size))
    if not total or not k:
        return []
    if k >= total:
        return list(range(total))
    strategy = (strategy or "spread").lower()
    if strategy == "first":
        return list(range(k))
    if strategy == "random":
        return sorted(random.Random(int(seed)).sample(range(total), k))
    if strategy != "spread":
        raise ValueError("profile strategy must be one of: spread, random, first")
    if k == 1:
        return [0]
    return [min(total - 1, round(i * (total - 1) / (k - 1))) for i in range(k)]


def default_prompt_id(row: dict, index: int) -> str:
    for key in ("prompt_id", "id", "uid"):
        if row.get(key):
            return str(row[key])
    if row.get("repo_name") or row.get("commit_hash"):
        return f"{row.get('repo_name') or 'repo'}:{row.get('commit_hash') or index}"
    return str(index)


def build_length_profile(rows: Sequence[dict], *, prompt_length_fn: LengthFn, output_length_fn: LengthFn,
                         sample_size: int, strategy: str = "spread", seed: int = 0, samples_per_prompt: int = 1,
                         max_output_len: int = 0, prompt_id_fn=default_prompt_id) -> List[dict]:
    out = []
    for idx in sample_indices(len(rows), sample_size, strategy=strategy, seed=seed):
        row = rows[idx]
        p = max(1, int(prompt_length_fn(row)))
        g = max(1, int(output_length_fn(row)))
        if max_output_len > 0:
            g = min(g, int(max_output_len))
        pid = prompt_id_fn(row, idx)
        out.extend({"input_len": p, "output_len": g, "prompt_id": pid, "source_index": int(idx), "sample_index": s,
                    "profile_source": "startup_real_sample"} for s in range(max(1, int(samples_per_prompt))))
    return out


def _percentile(values: List[int], q: float) -> float:
    if not values:
        return 0.0
    s = sorted(values)
    pos = (len(s) - 1) * q / 100.0
    lo, hi = math.floor(pos), math.ceil(pos)
    return float(s[lo] + (s[hi] - s[lo]) * (pos - lo))


def _stats(values: Iterable[int]) -> Dict[str, float]:
    v = [int(x) for x in values]
    if not v:
        return {"count": 0, "mean": 0.0, "min": 0.0, "max": 0.0, "p25": 0.0, "p50": 0.0, "p75": 0.0, "p90": 0.0,
                "p95": 0.0, "p99": 0.0}
    out = {"count": len(v), "mean": sum(v) / len(v), "min": float(min(v)), "max": float(max(v))}
    out.update({f"p{q}": _percentile(v, q) for q in (25, 50, 75, 90, 95, 99)})
    return out


def summarize_length_profile(records: Sequence[dict]) -> Dict[str, Any]:
    recs = [r for r in (_as_record(x) for x in records if isinstance(x, dict)) if r is not None]
    return {"num_records": len(recs), "num_prompts": len({str(x.get("prompt_id")) for x in records
                                                            if isinstance(x, dict) and x.get("prompt_id")}),
            "input_len": _stats(r["input_len"] for r in recs), "output_len": _stats(r["output_len"] for r in recs),
            "total_len": _stats(r["input_len"] + r["output_len"] for r in recs)}


def write_profile_jsonl(records: Sequence[dict], path) -> None:
    p = Path(path)
    p.parent.mkdir(parents=True, exist_ok=True)
    p.write_text("".join(json.dumps(r) + "\n" for r in records), encoding="utf-8")


def write_profile_summary(summary: dict, path) -> None:
    p = Path(path)
    p.parent.mkdir(parents=True, exist_ok=True)
    p.write_text(json.dumps(summary, indent=2), encoding="utf-8")
