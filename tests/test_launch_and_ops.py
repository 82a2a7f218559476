"""Launcher planning, data preparation, preflight CLIs, supervisor, tracker, CoT env (CPU)."""

import json
import os
import sys
import time

import pytest

from libra_b200.launcher.cluster import (auto_plan_cluster, build_rollout_launch_commands, build_torchrun_command,
                                         compute_gpu_allocation)


def test_cluster_plan_and_commands():
    plan = auto_plan_cluster(4, 4, nodes=["box0"], tp_list=[1, 1, 2])
    assert plan["endpoints"] == ["box0:8000", "box0:8001", "box0:8002"]
    a = compute_gpu_allocation(["box0"], 8, 4, 4)
    cmds = build_rollout_launch_commands(a, "qwen3-4b", tp_list=[1, 1, 2])
    assert [c["gpu_ids"] for c in cmds] == [[4], [5], [6, 7]]
    assert "CUDA_VISIBLE_DEVICES=6,7" in cmds[2]["command"] and "--nproc-per-node 2" in cmds[2]["command"]
    tr = build_torchrun_command(a, "examples/train.py")
    assert "--local-addr 127.0.0.1" in tr["command"] and tr["nproc_per_node"] == 4
    with pytest.raises(ValueError):
        compute_gpu_allocation(["box0"], 8, 6, 4)


def test_box_launcher_dry_run(capsys):
    from libra_b200.config import AsyncRLConfig
    from libra_b200.launcher.box_launcher import BoxLauncher

    cfg = AsyncRLConfig.from_file(os.path.join("libra_b200", "configs", "qwen3_4b_grpo_8xb200.yaml"))
    cfg.rollout_backend = "http"
    assert BoxLauncher(cfg, "cfg.yaml").launch(dry_run=True) == 0
    out = capsys.readouterr().out.strip().splitlines()
    assert len(out) == 1 + len(cfg.heterogeneous_rollout.instances)
    assert "torch.distributed.run" in out[-1] and "--nproc-per-node 4" in out[-1]


def test_data_prepare_converters(tmp_path):
    from libra_b200.data.prepare import main, read_rows

    src = tmp_path / "gsm.jsonl"
    src.write_text(json.dumps({"question": "1+1?", "answer": "so 2\n#### 2"}) + "\n")
    main(["gsm8k", "--input", str(src), "--output", str(tmp_path / "o.jsonl")])
    (row,) = read_rows(str(tmp_path / "o.jsonl"))
    assert row["answer"] == "2" and row["question"] == "1+1?"
    src2 = tmp_path / "lcb.json"
    src2.write_text(json.dumps([{"question_id": "x", "question_content": "add", "public_test_cases":
                                 json.dumps([{"input": "1 2", "output": "3"}]), "private_test_cases": "[]",
                                 "metadata": "{}"}]))
    main(["livecodebench", "--input", str(src2), "--output", str(tmp_path / "c.jsonl")])
    (c,) = read_rows(str(tmp_path / "c.jsonl"))
    assert c["test_cases"] == {"inputs": ["1 2"], "outputs": ["3"]}
    src3 = tmp_path / "nq.jsonl"
    src3.write_text(json.dumps({"question": "who wrote hamlet", "golden_answers": ["Shakespeare"]}) + "\n")
    main(["search_r1", "--input", str(src3), "--output", str(tmp_path / "s.jsonl")])
    assert read_rows(str(tmp_path / "s.jsonl"))[0]["question"].endswith("?")


def test_preflight_validate_and_merge(tmp_path, capsys):
    from libra_b200.config import AsyncRLConfig
    from libra_b200.infra.preflight.__main__ import main, validate_ehp
    from libra_b200.infra.scheduling.cmlfq_prefix_tree import CausalPrefixTree

    cfg = AsyncRLConfig.from_file(os.path.join("libra_b200", "configs", "qwen3_4b_grpo_8xb200.yaml"))
    assert validate_ehp(cfg) == []
    cfg.global_resource_planner.elastic_hybrid_replica_size_gpus = 3
    assert any("replica" in p for p in validate_ehp(cfg))
    paths = []
    for i in range(2):
        t = CausalPrefixTree()
        p = tmp_path / f"t{i}.json"
        t.save(str(p))
        paths.append(str(p))
    assert main(["merge-trees", *paths, "--output", str(tmp_path / "m.json")]) == 0
    assert (tmp_path / "m.json").exists()


def test_supervisor_restarts_and_reloads(tmp_path):
    from libra_b200.engine.supervisor import Supervisor

    sentinel = str(tmp_path / "reload.json")
    sup = Supervisor([sys.executable, "-c", "import time; time.sleep(0.2)"], sentinel=sentinel, max_restarts=2,
                     backoff_s=0.01)
    sup.start()
    time.sleep(0.6)
    assert sup.poll_once() == "restarted" and sup.restarts == 1
    with open(sentinel, "w") as f:
        json.dump({"checkpoint_path": "/ckpt/v3", "version": 3}, f)
    assert sup.poll_once() == "reloaded" and "--checkpoint /ckpt/v3" in sup._cmd()
    assert json.load(open(sentinel + ".ack"))["version"] == 3
    sup.stop()


def test_jsonl_tracker(tmp_path):
    from types import SimpleNamespace

    from libra_b200.utils.tracking import JsonlTracker, Tracker

    t = Tracker.create(SimpleNamespace(log_dir=str(tmp_path)), rank=0)
    assert isinstance(t, JsonlTracker)
    t.log({"loss": 0.5, "note": "x", "skip": [1]}, step=3)
    t.finish()
    recs = [json.loads(line) for line in open(tmp_path / "metrics.jsonl")]
    assert recs[-1]["step"] == 3 and recs[-1]["loss"] == 0.5 and "skip" not in recs[-1]


def test_cot_env():
    from libra_b200.env.base_env import CoTEnv, NoLegalActionException

    env = CoTEnv([{"question": "2+3?", "answer": "5"}], max_steps=2)
    q = env.reset(0)
    assert "2+3?" in q
    _, r, done, _ = env.step("Add them.")
    assert not done and r == 0.0
    _, r, done, _ = env.step("The answer is \\boxed{5}")
    assert done and r == 1.0
    with pytest.raises(NoLegalActionException):
        env.step("more")


def test_preflight_nvlink_classification(capsys):
    import torch

    from libra_b200.infra.preflight.__main__ import classify_links, main

    pairs = [{"src": 0, "dst": 1, "gbs": 760.0}, {"src": 1, "dst": 0, "gbs": 742.0}]
    res = classify_links(pairs, expect_gbs=770.0, min_fraction=0.6)
    assert res["ok"] and res["min_gbs"] == 742.0 and res["max_gbs"] == 760.0 and not res["slow"]
    res = classify_links(pairs + [{"src": 0, "dst": 2, "gbs": 120.0}], expect_gbs=770.0, min_fraction=0.6)
    assert not res["ok"] and [p["dst"] for p in res["slow"]] == [2]
    assert not classify_links([], 770.0, 0.6)["ok"]
    if torch.cuda.device_count() < 2:
        assert main(["nvlink"]) == 1
        assert "needs two or more" in capsys.readouterr().out


@pytest.mark.gpu
@pytest.mark.multigpu
def test_preflight_nvlink_probe_two_gpus(capsys):
    from libra_b200.infra.preflight.__main__ import main

    rc = main(["nvlink", "--gpus", "2", "--mbytes", "64", "--iters", "4", "--min-fraction", "0.3"])
    out = json.loads(capsys.readouterr().out)
    assert out["pairs"] == 2 and out["min_gbs"] > 0
    assert rc == 0, out
