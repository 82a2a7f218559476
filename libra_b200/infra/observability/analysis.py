"""Run analysis with the reference's metric definitions
(``scripts/analyze_libra_experiment.py:99-429``):

* tokens/s (aggregate) = sum over steps and sequences of (input_len +
  output_len) / sum of step_total_time; per step likewise;
* trajectories/s = sum of trajectories / sum of step_total_time;
* mean / median step time and steps per hour;
* weight-sync time = mean of the non-zero weight_sync_time values.

    python -m libra_b200.infra.observability.analysis history.jsonl [...]
"""

from __future__ import annotations

import json
import statistics
import sys
from typing import Dict, Iterable, List


def load_records(paths: Iterable[str]) -> List[dict]:
    out = []
    for p in paths:
        with open(p, encoding="utf-8") as fh:
            out.extend(json.loads(line) for line in fh if line.strip())
    return out


def _tokens(rec: dict) -> int:
    seqs = rec.get("sequences") or []
    if seqs:
        return sum(int(s.get("input_len", 0)) + int(s.get("output_len", 0)) for s in seqs)
    st = rec.get("sequence_stats", {}).get("total", {})
    return int(round(st.get("mean", 0.0) * st.get("count", 0)))


def summarize(records: List[dict]) -> Dict[str, float]:
    steps = [float(r["timing"]["step_total_time"]) for r in records if r.get("timing", {}).get("step_total_time", 0) > 0]
    total_t = sum(steps)
    toks = [_tokens(r) for r in records]
    trajs = [int(r.get("training_metrics", {}).get("n_trajectories", 0)) or len(r.get("sequences") or [])
             for r in records]
    sync = [float(r["timing"].get("weight_sync_time", 0.0)) for r in records
            if float(r.get("timing", {}).get("weight_sync_time", 0.0)) > 0]
    per_step = [t / s for t, s in zip(toks, (float(r["timing"]["step_total_time"]) for r in records)) if s > 0]
    return {
        "steps": len(records),
        "tokens_per_second": sum(toks) / total_t if total_t else 0.0,
        "tokens_per_second_per_step_mean": statistics.fmean(per_step) if per_step else 0.0,
        "trajectories_per_second": sum(trajs) / total_t if total_t else 0.0,
        "step_time_mean": statistics.fmean(steps) if steps else 0.0,
        "step_time_median": statistics.median(steps) if steps else 0.0,
        "steps_per_hour": 3600.0 * len(steps) / total_t if total_t else 0.0,
        "weight_sync_time_mean": statistics.fmean(sync) if sync else 0.0,
    }


def main(argv=None) -> None:
    paths = (argv if argv is not None else sys.argv[1:])
    if not paths:
        raise SystemExit("usage: python -m libra_b200.infra.observability.analysis history.jsonl [...]")
    print(json.dumps(summarize(load_records(paths)), indent=2))


if __name__ == "__main__":
    main()
