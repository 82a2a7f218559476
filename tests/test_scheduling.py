"""Scheduler behaviour (reference tests/test_cmlfq_scheduler.py, test_hetero_cmlfq_integration.py)."""

import json
import os
from types import SimpleNamespace

import pytest
import torch

from libra_b200.config import HeterogeneousRolloutConfig, SchedulingConfig
from libra_b200.infra.scheduling import SchedulerFactory
from libra_b200.infra.scheduling.baselines import (LAMLFQScheduler, LengthAwareScheduler, LoadBalanceScheduler,
                                                   ScoutStatus)
from libra_b200.infra.scheduling.cmlfq_migration import (CMLFQMigrationCoordinator, KVCacheManager,
                                                         MigrationCostProfiler, reshard_heads)
from libra_b200.infra.scheduling.cmlfq_offline_profile import CMLFQOfflineProfiler, CMLFQTreeUpdater
from libra_b200.infra.scheduling.cmlfq_prefix_tree import CausalPrefixTree, PrefixTreeNode, Trajectory
from libra_b200.infra.scheduling.cmlfq_scheduler import CMLFQScheduler, rank_file
from libra_b200.infra.scheduling.cmlfq_shared_state import SharedCMLFQLoadState
from libra_b200.infra.scheduling.cmlfq_tool_state import (DefaultToolStateExtractor, ExecutionStatus,
                                                          PayloadSizeClass, ToolReturnState)

S = lambda t="code", size=PayloadSizeClass.SizeSmall, st=ExecutionStatus.ToolSuccess: ToolReturnState(t, size, st)  # noqa: E731

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _register(s, tps=(1, 1, 2, 4, 8)):
    for i, tp in enumerate(tps):
        s.register_instance(i, f"inst{i}_tp{tp}", tp)
    return s


def test_tool_state_extraction():
    ex = DefaultToolStateExtractor()
    assert ex.extract("ok").to_key() == "text:small:success"
    assert ex.extract("x" * 600 + " Error").to_key() == "text:medium:failure"
    assert ex.extract({"tool_type": "search", "output": "x" * 6000}).to_key() == "search:large:success"
    assert ex.extract({"tool": "py", "status": "timeout"}).execution_status == ExecutionStatus.ToolTimeout
    assert ex.extract({"tool": "py", "traceback": "..."}).execution_status == ExecutionStatus.ToolFailure
    assert ex.extract({"tool": "py", "payload_tokens": 10, "payload_size_class": "large"}).payload_size_class == \
        PayloadSizeClass.SizeLarge
    assert ToolReturnState.from_key("a:medium:timeout") == S("a", PayloadSizeClass.SizeMedium, ExecutionStatus.ToolTimeout)
    with pytest.raises(ValueError):
        DefaultToolStateExtractor(10, 5)


def test_prefix_tree_insert_lookup_fallback_bucket():
    tree = CausalPrefixTree()
    a, b = S("a"), S("b")
    tree.insert(Trajectory("p1", [a, b], [3000.0, 1000.0], total_length=4000))
    tree.insert(Trajectory("p1", [a], [9000.0], total_length=9500))
    node = tree.lookup("p1", [a])
    assert node.visit_count == 2 and node.mean_remaining_length == pytest.approx(6000.0)
    assert tree.lookup("p1", [a, S("zzz")]) is None
    assert tree.lookup_with_fallback("p1", [a, S("zzz")]) is node  # deepest matching prefix
    g = tree.lookup_with_fallback("unseen", [a])  # global root fallback
    assert g is not None and g.visit_count == 2
    th = {"short": 5000, "long": 50000}
    deep = tree.lookup("p1", [a, b])
    assert tree.get_bucket_for_node(deep, th) == "short"
    assert tree.get_bucket_for_node(node, th) == "long"  # mean 6000 and p90 8400 both above 5000
    assert tree.get_bucket_for_node(node, {"short": 7000, "long": 50000}) is None  # mean short, p90 long
    st = tree.get_stats()
    assert st["n_prompts"] == 1 and st["total_insertions"] == 2 and st["max_depth"] == 2


def test_bucket_requires_mean_p90_agreement():
    tree = CausalPrefixTree()
    for r in [100.0] * 8 + [20000.0, 20000.0]:
        tree.insert(Trajectory("p", [S()], [r]))
    node = tree.lookup("p", [S()])
    th = {"short": 5000, "long": 50000}
    mean_b = tree._length_to_bucket(node.mean_remaining_length, th)
    p90_b = tree._length_to_bucket(node.p90_remaining_length, th)
    assert (tree.get_bucket_for_node(node, th) is None) == (mean_b != p90_b)
    assert p90_b == "long"


def test_tree_rebuild_merge_save_load(tmp_path):
    t1, t2 = CausalPrefixTree(), CausalPrefixTree()
    t1.insert(Trajectory("p", [S("a")], [100.0]))
    t2.insert(Trajectory("p", [S("a")], [300.0]))
    t2.insert(Trajectory("q", [S("b")], [50.0]))
    t1.merge(t2)
    n = t1.lookup("p", [S("a")])
    assert n.visit_count == 2 and n.mean_remaining_length == pytest.approx(200.0)
    assert t1.get_stats()["n_prompts"] == 2
    path = tmp_path / "tree.json"
    t1.save(str(path))
    data = json.loads(path.read_text())
    assert data["version"] == 2 and "global_root" in data and set(data["roots"]) == {"p", "q"}
    t3 = CausalPrefixTree()
    t3.load(str(path))
    assert t3.lookup("q", [S("b")]).visit_count == 1
    # version-1 file (no global root) upgrades on load
    data.pop("global_root")
    data["version"] = 1
    path.write_text(json.dumps(data))
    t4 = CausalPrefixTree()
    t4.load(str(path))
    assert t4.lookup_with_fallback("new", [S("a")]).visit_count == 2
    t4.rebuild([Trajectory("z", [S("c")], [1.0])])
    assert t4.get_stats()["n_prompts"] == 1


def test_cmlfq_initial_placement_and_migration():
    s = _register(CMLFQScheduler())
    r = s.schedule(input_tokens=100, prompt_id="p")
    assert r.category == "short" and r.tp_degree in (1, 2) and r.request_id
    d = s.on_tool_return(r.request_id, {"tool_type": "code", "output": "x"}, generated_tokens=200)
    assert not d.should_migrate and d.reason == "tree_node_not_found"
    s.finish_request(r.request_id, 20000)  # teaches the tree: after code:small:success, ~19800 remain
    r2 = s.schedule(input_tokens=100, prompt_id="p")
    d2 = s.on_tool_return(r2.request_id, {"tool_type": "code", "output": "y"}, generated_tokens=100)
    assert d2.should_migrate and d2.target_bucket == "long"
    m = s.execute_migration(r2.request_id, d2)
    assert m.tp_degree in (4, 8) and s.get_request_route(r2.request_id).category == "long"
    assert s.get_stats().migrated_routes == 1
    s.cancel_request(r2.request_id)
    assert not s.has_request(r2.request_id)
    assert all(h.active_requests == 0 for h in s._instances)


def test_cmlfq_no_migration_when_already_in_bucket_and_fallbacks():
    s = _register(CMLFQScheduler(), tps=(4,))  # only a long-bucket instance
    r = s.schedule(10, "p")
    assert r.is_fallback and r.tp_degree == 4
    empty = CMLFQScheduler()
    assert empty.schedule(10, "p").instance_index == -1


def test_cmlfq_from_config_and_persistence(tmp_path, monkeypatch):
    monkeypatch.setenv("RANK", "3")
    tree_path = tmp_path / "t.json"
    cfg = HeterogeneousRolloutConfig(scheduling=SchedulingConfig(scheduler_type="cmlfq", cmlfq_tree_path=str(tree_path),
                                                                 cmlfq_shared_load_dir=str(tmp_path / "load")))
    s = SchedulerFactory.create("cmlfq", cfg)
    _register(s)
    r = s.schedule(5, "p")
    s.on_tool_return(r.request_id, "ok", 10)
    s.finish_request(r.request_id, 50)
    assert (tmp_path / "t.rank_3.json").exists()
    s.on_epoch_end(2)
    assert (tmp_path / "t.rank_3.step_2.json").exists()
    assert rank_file(str(tree_path), 0, 7).endswith("t.rank_0.step_7.json")
    s2 = SchedulerFactory.create("cmlfq", cfg)
    assert s2.prefix_tree.get_stats()["total_insertions"] == 1


def test_shared_load_live_rows(tmp_path):
    import struct
    import subprocess
    import sys
    import time

    a = SharedCMLFQLoadState(str(tmp_path), ttl_s=60, heartbeat_interval_s=10, writer_id="rank_0")
    b = SharedCMLFQLoadState(str(tmp_path), ttl_s=60, heartbeat_interval_s=10, writer_id="rank_1")
    a.increment("i0")
    b.increment("i0")
    b.increment("i1")
    assert a.aggregate() == {"i0": 2, "i1": 1}
    b.decrement("i1")
    assert a.aggregate() == {"i0": 2}
    # a row whose heartbeat is older than the TTL stops counting
    struct.pack_into("<qd", b._mm, b._base, b._pid, time.time() - 1000)
    assert a.aggregate() == {"i0": 1}
    b.close()
    # another process shares the table; once it dies its counts vanish at once
    code = (
        "import os, sys, time, pathlib\n"
        f"sys.path.insert(0, {str(ROOT)!r})\n"
        "from libra_b200.infra.scheduling.cmlfq_shared_state import SharedCMLFQLoadState\n"
        f"s = SharedCMLFQLoadState({str(tmp_path)!r}, writer_id='child')\n"
        "s.increment('i2'); s.increment('i2')\n"
        f"pathlib.Path({str(tmp_path / 'ready')!r}).write_text('1')\n"
        "t0 = time.time()\n"
        f"while not os.path.exists({str(tmp_path / 'go')!r}) and time.time() - t0 < 60: time.sleep(0.01)\n"
        "os._exit(0)\n")
    child = subprocess.Popen([sys.executable, "-c", code])
    t0 = time.time()
    while not (tmp_path / "ready").exists() and time.time() - t0 < 60:
        time.sleep(0.01)
    assert a.aggregate() == {"i0": 1, "i2": 2}
    (tmp_path / "go").write_text("1")
    assert child.wait(timeout=60) == 0
    assert a.aggregate() == {"i0": 1}
    c = SharedCMLFQLoadState(str(tmp_path), writer_id="rank_2")  # the dead writer's row is reusable
    c.increment("i1")
    assert a.aggregate() == {"i0": 1, "i1": 1}
    c.close()
    a.close()


def test_load_balance_rotates_ties_and_weighted():
    s = _register(LoadBalanceScheduler(), tps=(1, 1, 2))
    picks = []
    for _ in range(3):
        r = s.schedule(10)
        picks.append(r.instance_index)
        s.on_request_done(r.instance_index)
    assert sorted(picks) == [0, 1, 2]
    w = _register(LoadBalanceScheduler("weighted", weights={2: 4.0}), tps=(1, 2))
    w._instances[1].active_requests = 3
    assert w.schedule(1).instance_index == 0  # loads 0/1 vs 3/4
    w._instances[0].active_requests = 1
    assert w.schedule(1).instance_index == 1  # 2/1 vs 3/4
    rr = _register(LoadBalanceScheduler("round_robin"), tps=(1, 1))
    assert [rr.schedule(1).instance_index for _ in range(4)] == [0, 1, 0, 1]


def test_length_aware_categories_and_fallback():
    s = _register(LengthAwareScheduler(), tps=(1, 8))
    assert s.categorize(100) == "short" and s.categorize(12000) == "long" and s.categorize(99999) == "extra_long"
    r = s.schedule(7000)  # medium prefers [2, 4] -> fallback [1, 8]
    assert r.is_fallback and r.tp_degree == 1
    assert s.schedule(20000).tp_degree == 8


def test_la_mlfq_scout_pending_and_release():
    s = _register(LAMLFQScheduler(), tps=(1, 4))
    scout = s.schedule(100, "p", n_samples=4)
    assert scout.category == "short" and s.scout_manager.get_scout_status("p") == ScoutStatus.RUNNING
    wait = s.schedule(100, "p", n_samples=4)
    assert wait.pending and wait.reason == "waiting_for_scout"
    d = s.check_and_migrate("p_scout", generated_tokens=6000)
    assert d.should_migrate and d.target_bucket == "long"
    follow = s.schedule(100, "p", n_samples=4)
    assert follow.category == "long" and follow.tp_degree == 4
    s.on_request_done(scout.instance_index, "p", final_bucket="long")
    assert s.history_table.lookup("p") == "long"
    s.on_epoch_end(0)
    assert s.scout_manager.active_scouts == 0


def test_kv_reshard_roundtrip():
    kv = torch.arange(2 * 8 * 4, dtype=torch.float32).view(2, 8, 4)  # [tokens, heads, dim]
    for src, dst in [(2, 4), (4, 2), (2, 2), (1, 8), (8, 1)]:
        shards = list(torch.chunk(kv, src, dim=1))
        out = reshard_heads(shards, dst, dim=1)
        assert len(out) == dst and torch.equal(torch.cat(out, dim=1), kv)
    with pytest.raises(ValueError):
        reshard_heads(list(torch.chunk(kv, 2, dim=1)), 3, dim=1)
    coord = CMLFQMigrationCoordinator()
    cache = {0: (kv, kv + 1)}
    out = coord.execute_full_migration("r", 0, 1, 1, 2, cache, seq_len=2, target_rank=1, target_device="cpu")
    assert torch.equal(out[0][0], kv[:, 4:])


def test_migration_cost_profiler(tmp_path):
    p = MigrationCostProfiler()
    assert p.decide_migration_path(1, 4, 1000)[0] == "recompute"
    assert p.decide_migration_path(1, 4, 10000)[0] == "migrate"
    p.record_measurement(1, 4, 2048, 1, 1, 5, 1, recompute_prefill_ms=4.0)
    assert p.decide_migration_path(1, 4, 2000) == ("migrate", 3)  # on-box: offload+reshard+reload
    assert p.decide_migration_path(1, 4, 2000, is_cross_node=True)[0] == "recompute"  # + 5 ms network
    p.save_profile(str(tmp_path / "prof.json"))
    assert MigrationCostProfiler(str(tmp_path / "prof.json"))._lookup(1, 4, 9999) is not None
    nv = MigrationCostProfiler(kv_bytes_per_token=147456, prefill_tokens_per_s=50000)
    assert nv.decide_migration_path(1, 2, 8192)[0] == "migrate"


def test_offline_profile_and_updater():
    raw = [{"prompt_id": "p", "total_output_tokens": 1000,
            "tool_returns": [{"tool_type": "code", "output": "x", "token_position": 200},
                             {"tool_type": "code", "output": "err error", "remaining_length": 100}]}]
    prof = CMLFQOfflineProfiler()
    tree = prof.profile_from_raw_trajectories(raw)
    n = tree.lookup("p", [S("code")])
    assert n.mean_remaining_length == 800
    rec = SimpleNamespace(step=3, sequences=[{"index": 0, "output_len": 50, "tool_returns": [{"tool": "t", "token_position": 10}]}])
    prof.profile_from_step_records([rec])
    assert tree.get_stats()["n_prompts"] == 2
    up = CMLFQTreeUpdater(CausalPrefixTree(), rebuild_interval=2, max_recent_trajectories=1)
    up.update_from_step(1, [Trajectory("a", [S()], [1.0])])
    up.update_from_step(2, [Trajectory("b", [S()], [1.0])])
    assert up.prefix_tree.get_stats()["n_prompts"] == 1  # rebuilt from the 1-trajectory window


def test_factory_unknown():
    with pytest.raises(ValueError, match="Available types"):
        SchedulerFactory.create("nope", HeterogeneousRolloutConfig())
