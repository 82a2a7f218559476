"""Cost model, optimizer, GRP and preflight behaviour (reference tests/test_preflight_planner.py,
test_global_resource_planner_simulators.py, test_memory_budget.py)."""

import json
import os
import sys

import pytest

from libra_b200.config import AsyncRLConfig
from libra_b200.infra.cost_model.calibrator import EpochRunData, ShadowCalibrator
from libra_b200.infra.cost_model.global_resource_planner import GlobalResourcePlanner, RuntimeResourceMetrics
from libra_b200.infra.cost_model.memory_budget import estimate_recompute_logprobs_memory
from libra_b200.infra.cost_model.model import CostModel, RequestInfo, RolloutClusterConfig, TrainParallelConfig
from libra_b200.infra.cost_model.optimizer import generate_rollout_configs, TwoLevelNestedOptimizer
from libra_b200.infra.cost_model.preflight_planner import PreflightPlanner, synthetic_history
from libra_b200.infra.cost_model.simulator_adapters import HybridSimulatorCostModel
from libra_b200.infra.cost_model.startup_profile import build_length_profile, sample_indices, summarize_length_profile

CFG = os.path.join(os.path.dirname(os.path.dirname(__file__)), "libra_b200", "configs", "qwen3_4b_grpo_8xb200.yaml")


def _cfg(tmp_path, **over):
    cfg = AsyncRLConfig.from_file(CFG)
    cfg.sync_path, cfg.log_dir = str(tmp_path / "s"), str(tmp_path / "l")
    cfg.global_resource_planner.simulator_cache_dir = str(tmp_path / "cache")
    for k, v in over.items():
        setattr(cfg.global_resource_planner, k, v)
    return cfg


def test_memory_budget_formula():
    est = estimate_recompute_logprobs_memory(batch_size=2, sequence_length=101, vocab_size=1000,
                                             tensor_parallel_size=4, logits_dtype_bytes=4, workspace_factor=1.5)
    assert est.local_vocab_size == 250 and est.logits_bytes == 2 * 100 * 250 * 4
    assert est.total_bytes == int(est.logits_bytes * 1.5)


def test_rollout_partitions():
    parts = {tuple(c.tp_list) for c in generate_rollout_configs(4, [1, 2, 4])}
    assert parts == {(4,), (2, 2), (2, 1, 1), (1, 1, 1, 1)}
    assert generate_rollout_configs(0) == []


def test_cost_model_monotonic(tmp_path):
    cfg = _cfg(tmp_path)
    cm = CostModel(cfg.hardware, cfg.model_arch, cfg.profiling)
    reqs = [RequestInfo(300, 1500)] * 64
    t1, _ = cm.evaluate_rollout(RolloutClusterConfig([1]), reqs)
    t4, _ = cm.evaluate_rollout(RolloutClusterConfig([1, 1, 1, 1]), reqs)
    assert t4 < t1
    tt1, _ = cm.evaluate_training(TrainParallelConfig(dp=1, b_micro=8), 64, 1800)
    tt4, _ = cm.evaluate_training(TrainParallelConfig(dp=4, b_micro=8), 64, 1800)
    assert tt4 < tt1
    big = TrainParallelConfig(dp=1, b_micro=64)
    assert cm.check_train_oom(big, 64, 16384)
    res = cm.evaluate(TrainParallelConfig(dp=2, b_micro=8), RolloutClusterConfig([2, 2]), reqs, 64)
    assert res.t_global == max(res.t_train, res.t_rollout) and not res.is_oom


def test_preflight_applies_grp_plan_on_single_box(tmp_path):
    cfg = _cfg(tmp_path)
    res = PreflightPlanner(cfg).run(synthetic_history(num_requests=64, input_len=300, output_len=1500))
    assert res.applied and res.planned_config.global_resource_planner.initial_allocation_applied
    plan = res.applied_plan
    assert plan.train_gpus + plan.rollout_gpus == 8 and plan.train_config.pp == 1
    gpus = [g for inst in res.planned_config.heterogeneous_rollout.instances for g in inst.gpus]
    assert sorted(gpus) == list(range(plan.train_gpus, 8))
    assert res.metadata["length_profile"]["num_records"] == 64


def test_triggers_and_gain_threshold(tmp_path):
    cfg = _cfg(tmp_path, plan_interval=10, warmup_steps=2, min_history_size=4, runtime_replan_cooldown_steps=3)
    grp = GlobalResourcePlanner.from_config(cfg)
    hist = synthetic_history(num_requests=16, input_len=300, output_len=1500)
    assert grp.plan_if_needed(1, cfg, batch=hist).reason == "warmup"
    assert grp.plan_if_needed(3, cfg).reason == "interval_skip"
    m = grp.observe_runtime(step=3, dispatcher_metrics={"pending_inputs": 90, "runner_max_queue": 50,
                                                        "staleness_pending_limit": 50, "staleness_running": 2,
                                                        "staleness_capacity": 8})
    assert m.queue_pressure == pytest.approx(0.9)
    d = grp.plan_if_needed(3, cfg, runtime_metrics=m)
    assert d.trigger == "queue_pressure" and d.candidate_plan is not None
    if d.should_reconfigure:
        assert grp.plan_if_needed(4, cfg, runtime_metrics=m).reason == "cooldown"
    m2 = RuntimeResourceMetrics(step=20, rollout_time_s=30.0, train_time_s=10.0)
    assert grp.trigger(21, m2) == "rollout_train_imbalance"


def test_forced_env_overrides(tmp_path, monkeypatch):
    cfg = _cfg(tmp_path, min_history_size=1)
    grp = GlobalResourcePlanner.from_config(cfg)
    monkeypatch.setenv("GRP_FORCE_ROLLOUT_TP_LIST", "2,2")
    d = grp.plan_if_needed(10, cfg, batch=synthetic_history(num_requests=8))
    assert d.candidate_plan.rollout_tp_list == [2, 2] and d.reason in ("forced_reconfigure", "same_plan")
    monkeypatch.setenv("GRP_FORCE_ROLLOUT_TP_LIST", "2,1")
    with pytest.raises(ValueError, match="must sum"):
        grp.plan_if_needed(20, cfg)


def test_elastic_hybrid_signal(tmp_path):
    cfg = _cfg(tmp_path, min_history_size=1, elastic_hybrid_planning_enabled=True)
    grp = GlobalResourcePlanner.from_config(cfg)
    hist = synthetic_history(num_requests=8)
    train_bound = RuntimeResourceMetrics(step=10, train_time_s=20.0, rollout_time_s=10.0)
    d = grp.plan_if_needed(10, cfg, batch=hist, runtime_metrics=train_bound)
    sig = d.elastic_hybrid_signal
    assert sig.replica_size_gpus == 2 and sig.max_workers == 2
    assert sig.action == "join" or sig.reason == "candidate_requests_more_training_capacity"
    busy = RuntimeResourceMetrics(step=20, train_time_s=20.0, rollout_time_s=10.0, queue_pressure=0.95)
    d2 = grp.plan_if_needed(20, cfg, runtime_metrics=busy)
    assert d2.elastic_hybrid_signal.reason == "protect_rollout_capacity"


def test_simulator_command_contract_and_fallback(tmp_path):
    script = tmp_path / "fake_sailor.py"
    script.write_text("import json,sys\nd=json.load(open(sys.argv[1]))\n"
                      "json.dump({'t_train': 1.0 + d['train_config']['dp']}, open(sys.argv[2],'w'))\n")
    (tmp_path / "sailor").mkdir()
    cfg = _cfg(tmp_path, train_backend="sailor", sailor_path=str(tmp_path / "sailor"),
               sailor_train_command=f"{{python}} {script} {{input_json}} {{output_json}}", sailor_python=sys.executable)
    ev = HybridSimulatorCostModel(cfg)
    t, d = ev.evaluate_training(TrainParallelConfig(dp=3), 64, 1000)
    assert t == 4.0 and d["backend"] == "sailor"
    cfg2 = _cfg(tmp_path, train_backend="sailor", sailor_path=str(tmp_path / "missing"), sailor_train_command="x")
    ev2 = HybridSimulatorCostModel(cfg2)
    t2, d2 = ev2.evaluate_training(TrainParallelConfig(dp=1), 64, 1000)
    assert d2["backend"] == "analytic" and ev2.fallback_events
    vid = tmp_path / "fake_vidur.py"
    vid.write_text("import sys\nprint('VIDUR_RESULT_JSON={\"makespan\": 7.5}')\n")
    (tmp_path / "vidur").mkdir()
    cfg3 = _cfg(tmp_path, rollout_backend="vidur", vidur_path=str(tmp_path / "vidur"),
                vidur_rollout_command=f"{{python}} {vid} {{trace_csv}} {{tp_list}}", vidur_python=sys.executable)
    t3, _ = HybridSimulatorCostModel(cfg3).evaluate_rollout(RolloutClusterConfig([1, 1]), [RequestInfo(10, 10)])
    assert t3 == 7.5


def test_startup_profile_sampling():
    assert sample_indices(10, 3) == [0, 4, 9] or sample_indices(10, 3) == [0, 5, 9]
    assert sample_indices(10, 3, strategy="first") == [0, 1, 2]
    assert sample_indices(3, 10) == [0, 1, 2]
    rows = [{"p": i + 1, "g": 10 * (i + 1), "id": f"r{i}"} for i in range(5)]
    recs = build_length_profile(rows, prompt_length_fn=lambda r: r["p"], output_length_fn=lambda r: r["g"],
                                sample_size=2, samples_per_prompt=2, max_output_len=25)
    assert len(recs) == 4 and all(r["output_len"] <= 25 for r in recs)
    s = summarize_length_profile(recs)
    assert s["num_records"] == 4 and s["num_prompts"] == 2


def test_calibrator_change_point():
    cal = ShadowCalibrator(min_epochs_for_calibration=2)
    for i in range(6):
        cal.update(EpochRunData(t_train_real=10.0, t_train_predicted=10.0 + 0.01 * i, gen_lengths=[500.0] * 4,
                                epoch_id=i))
    assert not cal.get_statistics()["is_change_point"]
    cal.update(EpochRunData(t_train_real=40.0, t_train_predicted=10.0, gen_lengths=[5000.0] * 4, epoch_id=7))
    st = cal.get_statistics()
    assert st["is_change_point"] and st["change_point_count"] == 1 and cal.params.eta_comp < 0.5


def test_b200_profile_predicts_measured_grpo_phases(tmp_path):
    """With the B200 profile of the presets, the cost model reproduces the
    phases of the 1-GPU Qwen3-4B GRPO step measured with ``python bench.py``
    (synthetic workload steps 3-7: rollout 17.97 s, train 5.85 s per step)."""
    from libra_b200.workflow.synthetic import WORKLOADS, rollout_requests

    cfg = _cfg(tmp_path)
    cm = CostModel(cfg.hardware, cfg.model_arch, cfg.profiling, max_seq_length=5136)
    train, roll = [], []
    for s in range(3, 8):
        reqs = [RequestInfo(len(r.prompt), r.response_len)
                for r in rollout_requests(WORKLOADS["qwen3-4b-grpo"], s, rank=0, prompts=8)]
        tok = sum(r.total_length for r in reqs)
        train.append(cm.evaluate_training(TrainParallelConfig(tp=1, pp=1, dp=1, b_micro=8), 64, tok // 64)[0])
        roll.append(cm.evaluate_rollout(RolloutClusterConfig([1]), reqs)[0])
    assert abs(sum(train) / 5 - 5.85) / 5.85 < 0.1
    assert abs(sum(roll) / 5 - 17.97) / 17.97 < 0.1


def test_fit_decode_profile_recovers_terms():
    from libra_b200.infra.cost_model.calibrator import fit_decode_profile, fit_train_mfu

    L, bw, a, r, u = 36, 6.5e12, 40e-6, 4e-7, 0.9
    samples = []
    for b, kv in ((4, 1e9), (16, 5e9), (64, 2e10), (64, 4e9), (32, 8e9)):
        ms = (L * (a + b * r) + (8e9 + kv) / (bw * u)) * 1e3
        samples.append({"batch": b, "weight_bytes": 8e9, "kv_bytes": kv, "ms": ms})
    fit = fit_decode_profile(samples, L, bw)
    assert abs(fit["decode_layer_overhead_s"] - a) / a < 1e-6
    assert abs(fit["decode_row_layer_s"] - r) / r < 1e-6
    assert abs(fit["decode_bw_util"] - u) < 1e-6 and fit["max_rel_error"] < 1e-9
    assert abs(fit_train_mfu(5.85, 6.05, 0.55) - 0.55 * 6.05 / 5.85) < 1e-12


def test_simulated_makespan_is_bounded_by_the_longest_generation(tmp_path):
    cfg = _cfg(tmp_path)
    cm = CostModel(cfg.hardware, cfg.model_arch, cfg.profiling, max_seq_length=5136)
    rm = cm.rollout_model
    reqs = [RequestInfo(300, 100) for _ in range(63)] + [RequestInfo(300, 4000)]
    t = rm.compute_instance_makespan(reqs, 1)
    per_step_floor = cfg.model_arch.n_layers * cfg.profiling.decode_layer_overhead_s
    assert t > 4000 * per_step_floor  # the long request's 4000 steps cannot overlap
    assert rm.compute_instance_makespan(reqs[:63], 1) < 0.1 * t
