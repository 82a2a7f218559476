"""RuntimeElasticExecutor strategies with a fake process launcher (CPU)."""

import json
import os
import threading
import time
from types import SimpleNamespace

import pytest

from libra_b200.config import AsyncRLConfig
from libra_b200.infra.cost_model.global_resource_planner import (ElasticHybridSignal, GlobalResourcePlan,
                                                                 GlobalResourcePlanner, PlannerDecision)
from libra_b200.infra.cost_model.model import RolloutClusterConfig, TrainParallelConfig
from libra_b200.infra.elastic.hybrid_pool import ElasticHybridPool, ReplicaRole
from libra_b200.infra.elastic.runtime_executor import (ManagedRolloutProcess, RuntimeElasticExecutor,
                                                       follow_reconfiguration_request)

CFG = os.path.join(os.path.dirname(os.path.dirname(__file__)), "libra_b200", "configs", "qwen3_4b_grpo_8xb200.yaml")


class FakeProc:
    def __init__(self, pid):
        self.pid, self.returncode = pid, None

    def poll(self):
        return self.returncode


class FakeLauncher:
    def __init__(self, events):
        self.events, self.next_pid = events, 1000

    def start(self, command, env, log_path=""):
        self.next_pid += 1
        self.events.append(("start", command, dict(env)))
        return FakeProc(self.next_pid)

    def stop(self, proc, timeout):
        proc.returncode = 0
        self.events.append(("stop", proc.pid))

    def stop_pid(self, pid, timeout):
        self.events.append(("stop_pid", pid))

    def run(self, command, timeout):
        self.events.append(("run", command))
        return 0

    def wait_ready(self, host, port, timeout):
        self.events.append(("ready", port))


class FakeDispatcher:
    def __init__(self, events):
        self.events = events

    def pause(self):
        self.events.append(("pause",))

    def wait_until_idle(self, timeout=0):
        self.events.append(("drain",))

    def resume(self):
        self.events.append(("resume",))


class FakeRollout:
    def __init__(self, events):
        self.events = events

    def reconfigure_from_plan(self, plan, config):
        self.events.append(("engine", tuple(plan.rollout_tp_list)))


def _cfg(tmp_path, **grp):
    cfg = AsyncRLConfig.from_file(CFG)
    cfg.log_dir = str(tmp_path / "logs")
    cfg.global_resource_planner.hybrid_worker_task_dir = str(tmp_path / "tasks")
    for k, v in grp.items():
        setattr(cfg.global_resource_planner, k, v)
    return cfg


def _plan(train=(2, 1, 2), tps=(1, 1, 2)):
    tp, pp, dp = train
    return GlobalResourcePlan(TrainParallelConfig(tp=tp, pp=pp, dp=dp), RolloutClusterConfig(list(tps)), 1.0, 1.0,
                              1.0, 8, 64)


def _decision(plan, signal=None, step=5):
    return PlannerDecision(step, True, "test", candidate_plan=plan, elastic_hybrid_signal=signal)


def _executor(cfg, events, **kw):
    planner = GlobalResourcePlanner.from_config(cfg)
    return RuntimeElasticExecutor(config=cfg, planner=planner, dispatcher=FakeDispatcher(events),
                                  rollout_engine=FakeRollout(events), launcher=FakeLauncher(events), **kw)


def _seed(ex, cfg, specs):
    base = cfg.heterogeneous_rollout.vllm_base_port
    for i, (iid, gpus, tp) in enumerate(specs):
        ex._meta[iid] = ManagedRolloutProcess(iid, "old", 500 + i, list(gpus), base + i, "127.0.0.1", tp, True)


def test_diff_starts_only_changed_instances_before_stopping(tmp_path):
    cfg = _cfg(tmp_path, runtime_manage_rollout_processes=True, runtime_rollout_reconfigure_strategy="diff")
    ev = []
    ex = _executor(cfg, ev)
    _seed(ex, cfg, [("grp_tp1_0", [4], 1), ("grp_tp1_1", [5], 1), ("grp_tp2_2", [6, 7], 2)])
    res = ex.execute(_decision(_plan(tps=(1, 1, 1, 1))))
    assert res.applied and "reconfigure_rollout_processes:diff" in res.actions
    kinds = [e[0] for e in ev]
    starts = [e for e in ev if e[0] == "start"]
    assert len(starts) == 2  # grp_tp1_2, grp_tp1_3 (the first two are unchanged)
    assert all("CUDA_VISIBLE_DEVICES=6" in s[1] or "CUDA_VISIBLE_DEVICES=7" in s[1] for s in starts)
    assert max(i for i, k in enumerate(kinds) if k == "start") < kinds.index("stop_pid")
    assert kinds.index("pause") < kinds.index("engine") < kinds.index("resume")
    assert ("stop_pid", 502) in ev and ("stop_pid", 500) not in ev
    manifest = json.loads(open(os.path.join(cfg.log_dir, "runtime_rollout_manifest.json")).read())
    assert manifest["phase"] == "applied"
    for _, _, env in starts:
        assert "RANK" not in env and env["PLANNED_CUDA_VISIBLE_DEVICES"] in ("6", "7")


def test_restart_all_stops_before_starting(tmp_path):
    cfg = _cfg(tmp_path, runtime_manage_rollout_processes=True, runtime_rollout_reconfigure_strategy="restart_all")
    ev = []
    ex = _executor(cfg, ev)
    _seed(ex, cfg, [("a", [4], 1), ("b", [5, 6, 7], 3)])
    ex.execute(_decision(_plan(tps=(2, 2))))
    kinds = [e[0] for e in ev]
    assert kinds.count("stop_pid") == 2 and kinds.count("start") == 2
    assert max(i for i, k in enumerate(kinds) if k == "stop_pid") < kinds.index("start")


def test_prewarm_starts_before_pause_and_falls_back_without_spares(tmp_path):
    cfg = _cfg(tmp_path, runtime_manage_rollout_processes=True, runtime_rollout_reconfigure_strategy="prewarm")
    cfg.heterogeneous_rollout.available_gpus = [4, 5, 6, 7]
    ev = []
    ex = _executor(cfg, ev)
    _seed(ex, cfg, [("grp_tp1_0", [4], 1), ("grp_tp1_1", [5], 1)])
    res = ex.execute(_decision(_plan(tps=(1, 1, 2))))
    kinds = [e[0] for e in ev]
    assert "prewarm_rollout_processes" in res.actions and kinds.index("start") < kinds.index("pause")
    assert "stop_pid" not in kinds  # grp_tp1_0/1 unchanged; nothing replaced
    cfg2 = _cfg(tmp_path, runtime_manage_rollout_processes=True, runtime_rollout_reconfigure_strategy="prewarm")
    cfg2.heterogeneous_rollout.available_gpus = [4, 5, 6, 7]
    ev2 = []
    ex2 = _executor(cfg2, ev2)
    _seed(ex2, cfg2, [("x0", [4], 1), ("x1", [5], 1), ("x2", [6], 1), ("x3", [7], 1)])
    res2 = ex2.execute(_decision(_plan(tps=(2, 2))))
    assert any(a.startswith("prewarm_unavailable:no_spare_gpu_capacity") for a in res2.actions)
    assert "reconfigure_rollout_processes:restart_all" in res2.actions


def test_blue_green_moves_a_changed_instance_to_a_spare_port(tmp_path):
    cfg = _cfg(tmp_path, runtime_manage_rollout_processes=True, runtime_rollout_reconfigure_strategy="blue_green")
    ev = []
    ex = _executor(cfg, ev)
    base = cfg.heterogeneous_rollout.vllm_base_port
    _seed(ex, cfg, [("grp_tp2_0", [4, 5], 2), ("grp_tp2_1", [6, 7], 2)])
    res = ex.execute(_decision(_plan(tps=(1, 1, 2))))
    started = {m.instance_id: m.port for m in res.started_processes}
    assert started["grp_tp1_0"] not in (base, base + 1)  # old instances still own those ports
    kinds = [e[0] for e in ev]
    assert kinds.index("engine") < kinds.index("stop_pid")


def test_external_config_preserved_and_disable_switch(tmp_path):
    cfg = _cfg(tmp_path, apply_to_runtime=False)
    before = [i.instance_id for i in cfg.heterogeneous_rollout.instances]
    res = _executor(cfg, []).execute(_decision(_plan(tps=(4,))))
    assert "preserve_external_rollout_config" in res.actions
    assert [i.instance_id for i in cfg.heterogeneous_rollout.instances] == before
    cfg2 = _cfg(tmp_path, runtime_dynamic_reconfiguration_enabled=False)
    assert _executor(cfg2, []).execute(_decision(_plan())).reason == "runtime_dynamic_reconfiguration_disabled"


def test_training_pool_plan_only(tmp_path):
    cfg = _cfg(tmp_path, runtime_reconfigure_training=True, runtime_training_pool_target_gpus=6)
    res = _executor(cfg, []).execute(_decision(_plan()))
    assert res.training_actions[0] == "training_pool_plan_only"
    assert res.training_actions[1].startswith("plan_join_replica:ehp_replica_rollout0[rollout0,rollout1]->dp0")
    assert cfg.train_gpus == 4  # fixed training topology survives the plan


def _pool(fetch=None):
    return ElasticHybridPool(core_train_workers=["dp0", "dp1"],
                             core_rollout_workers=["rollout0", "rollout1", "rollout2", "rollout3"],
                             snapshot_fetcher=fetch or (lambda *_: 7), zero_sync_steps=0)


def test_signal_joins_then_release_cancels_pending(tmp_path):
    cfg = _cfg(tmp_path, runtime_reconfigure_training=True, runtime_training_pool_plan_only=False,
               elastic_hybrid_require_planner_signal=True)
    release = threading.Event()
    pool = _pool(lambda *_: (release.wait(5), 7)[1])
    ex = _executor(cfg, [], elastic_pool=pool)
    sig = ElasticHybridSignal(step=5, desired_workers=1, current_workers=0, max_workers=2, action="borrow",
                              reason="train_bound", train_rollout_ratio=1.4, rollout_pressure=0.2, ttl_steps=10,
                              replica_size_gpus=2)
    res = ex.execute(_decision(_plan(), sig))
    assert any(a.startswith("join_replica_submitted:ehp_replica_rollout0[rollout0,rollout1]->dp0")
               for a in res.training_actions)
    assert ex.hybrid_runtime_state()["pending_hybrid_replica_joins"] == 1
    stop = ElasticHybridSignal(step=6, desired_workers=0, current_workers=1, max_workers=2, action="release",
                               reason="rollout_bound", train_rollout_ratio=0.8, rollout_pressure=0.9, ttl_steps=10)
    res2 = ex.execute(PlannerDecision(6, False, "signal", elastic_hybrid_signal=stop))
    assert any(a.startswith("join_replica_cancelled:ehp_replica_rollout0") for a in res2.training_actions)
    release.set()
    time.sleep(0.2)
    snap = pool.snapshot()
    assert snap["rollout0"].role == ReplicaRole.HYBRID_ROLLOUT and pool.gradient_domain.active_hybrid_ids() == ()
    pool.close()


def test_join_completes_and_is_reported(tmp_path):
    cfg = _cfg(tmp_path, runtime_reconfigure_training=True, runtime_training_pool_plan_only=False,
               runtime_training_pool_target_gpus=6, hybrid_worker_task_dir=str(tmp_path / "tasks"))
    pool = _pool()
    ex = _executor(cfg, [], elastic_pool=pool)
    ex.execute(_decision(_plan()))
    deadline = time.time() + 3
    while pool.gradient_domain.active_hybrid_ids() == () and time.time() < deadline:
        time.sleep(0.02)
    st = ex.hybrid_runtime_state()
    assert st["active_hybrid_replicas"] == 1 and st["replica_size_gpus"] == 2
    member = json.loads((tmp_path / "tasks" / "membership" / "ehp_replica_rollout0.json").read_text())
    assert member["role"] == "hybrid_training" and member["members"] == ["rollout0", "rollout1"]
    res = ex.execute(_decision(_plan()))  # target reached: no second join
    assert any(a.startswith("training_gpus_unchanged") for a in res.training_actions)
    pool.close()


def test_cluster_swap_hands_rollout_gpus_to_training(tmp_path):
    cfg = _cfg(tmp_path, runtime_manage_rollout_processes=True, runtime_reconfigure_training=True,
               runtime_training_pool_plan_only=False, runtime_cluster_swap_enabled=True,
               runtime_training_pool_target_gpus=6)
    ev = []
    pool = _pool()
    ex = _executor(cfg, ev, elastic_pool=pool)
    _seed(ex, cfg, [("r0", [4], 1), ("r1", [5], 1), ("r2", [6, 7], 2)])
    plan = _plan(tps=(2,))
    res = ex.execute(_decision(plan))
    assert res.applied and "reconfigure_rollout_processes:cluster_swap" in res.actions
    slots = [a for a in res.training_actions if a.startswith("cluster_swap_training_slots:")]
    # the new TP-2 instance lands on GPUs 4,5; the stopped instances' GPUs 6,7 go to training
    assert slots == ["cluster_swap_training_slots:rollout0@127.0.0.1:[6],rollout1@127.0.0.1:[7]"]
    assert ("stop_pid", 500) in ev and ("stop_pid", 501) in ev and ("stop_pid", 502) in ev
    assert any(a.startswith("join_replica_submitted") for a in res.training_actions)
    pool.close()


def test_peer_ranks_drain_through_coordination_files(tmp_path, monkeypatch):
    cfg = _cfg(tmp_path, runtime_manage_rollout_processes=True, runtime_drain_timeout_s=5.0)
    monkeypatch.setenv("WORLD_SIZE", "4")
    monkeypatch.setenv("RANK", "0")
    cfg.train_tp_size = 2
    ex = _executor(cfg, [])
    _seed(ex, cfg, [("a", [4], 1)])
    assert ex._expected_ready_ranks() == [2]
    coord = os.path.join(cfg.log_dir, "runtime_reconfiguration")
    drained = []

    def follower():
        deadline = time.time() + 5
        while time.time() < deadline:
            if follow_reconfiguration_request(coord, 2, drain=lambda: drained.append(1)):
                return
            time.sleep(0.05)

    t = threading.Thread(target=follower)
    t.start()
    res = ex.execute(_decision(_plan(tps=(4,))))
    t.join(5)
    assert drained and "peer_reconfig_drain:2" in res.actions
    assert json.loads(open(os.path.join(coord, "applied.json")).read())["phase"] == "applied"
    cfg.global_resource_planner.runtime_drain_timeout_s = 0.3
    with pytest.raises(TimeoutError):
        ex.execute(_decision(_plan(tps=(2, 2))))
    assert json.loads(open(os.path.join(coord, "aborted.json")).read())["phase"] == "aborted"
