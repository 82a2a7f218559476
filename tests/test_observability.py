import json

from libra_b200.infra.observability.analysis import load_records, summarize
from libra_b200.infra.observability.history_collector import HistoryDataCollector
from libra_b200.infra.observability.phase_tracer import PhaseTracer, to_chrome


def test_phase_tracer_schema_and_chrome(tmp_path):
    t = PhaseTracer(tmp_path / "r0.jsonl", rank=0, world_size=2)
    t.start(1, "grpo_update", {"n": 3})
    t.end(1, "grpo_update", {"loss": 0.5})
    t.device_span(1, "grpo_update", 12.5)
    t.start(2, "weight_sync", {})
    t.close()
    rows = [json.loads(x) for x in (tmp_path / "r0.jsonl").read_text().splitlines()]
    assert {r["event"] for r in rows} == {"phase_start", "phase_span", "device_span", "phase_unfinished"}
    span = next(r for r in rows if r["event"] == "phase_span")
    assert span["schema"] == "libra.phase_trace.v1" and span["details"] == {"n": 3, "loss": 0.5}
    ev = to_chrome([str(tmp_path / "r0.jsonl")])
    assert len(ev) == 3 and all(e["ph"] == "X" for e in ev)
    assert any(e["tid"] == "gpu:grpo_update" and abs(e["dur"] - 12500) < 1 for e in ev)


def test_history_and_analysis(tmp_path):
    h = HistoryDataCollector(str(tmp_path), length_profile_path=str(tmp_path / "prof.jsonl"), flush_interval=1)
    for step in range(3):
        h.record_step(step, sequence_pairs=[(100, 200), (50, 150)], rollout_time=1.0, train_time=2.0,
                      weight_sync_time=0.5 if step else 0.0, step_total_time=4.0,
                      training_stats={"loss": 0.1, "rewards": [0.0, 1.0]}, predicted_train_time=2.2)
    h.close()
    recs = load_records([h.jsonl_path])
    assert recs[0]["timing"]["overhead_time"] == 1.0 and recs[0]["sequence_stats"]["total"]["count"] == 2
    s = summarize(recs)
    assert s["tokens_per_second"] == 500 / 4.0 and s["weight_sync_time_mean"] == 0.5 and s["steps_per_hour"] == 900
    assert h.compute_cost_model_accuracy()["train_mape"] > 0
    prof = (tmp_path / "prof.jsonl").read_text().splitlines()
    assert len(prof) == 6
    assert json.load(open(h.summary_path))["total_steps"] == 3


def test_checkpoint_snapshot_breaks_cycles_and_limits_depth():
    """Trainer stats go into checkpoints as plain, acyclic, depth-limited data
    (reference tests/test_checkpoint_snapshot.py)."""
    import io

    import torch

    from libra_b200.utils.snapshot import RECURSIVE, TOO_DEEP, snapshot

    def depth(v):
        if isinstance(v, dict):
            return 1 + max((depth(x) for x in v.values()), default=0)
        if isinstance(v, list):
            return 1 + max((depth(x) for x in v), default=0)
        return 0

    rec = {"reward": 0.5}
    rec["self"] = rec
    nested = cur = {}
    for i in range(100):
        cur["next"] = {}
        cur = cur["next"]
        cur["index"] = i
    shared = [1, 2]
    snap = snapshot({"recursive": rec, "nested": nested, "a": shared, "b": shared,
                     "t": torch.ones(3), "big": torch.zeros(1000, 2), "nan": float("nan"), "obj": object()},
                    max_depth=32)
    assert snap["recursive"]["self"] == RECURSIVE and snap["recursive"]["reward"] == 0.5
    assert depth(snap) <= 33 and TOO_DEEP in str(snap["nested"])
    assert snap["a"] == snap["b"] == [1, 2]  # shared (not cyclic) values are copied, not marked
    assert snap["t"] == [1.0, 1.0, 1.0] and snap["big"].startswith("<tensor (1000, 2)")
    assert snap["nan"] == "nan" and snap["obj"].startswith("<object")
    buf = io.BytesIO()
    torch.save(snap, buf)
    assert buf.tell() > 0
