"""End-to-end async GRPO plumbing: torchrun, 2 gloo ranks on CPU, tiny model."""

import glob
import json
import os
import socket
import subprocess
import sys

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _free_port() -> int:
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


def _run(tmp_path, task, *extra, steps=3, **env_extra):
    env = dict(os.environ, DIST_BACKEND="gloo", CUDA_VISIBLE_DEVICES="", OMP_NUM_THREADS="2", **env_extra)
    out = tmp_path / "stats.json"
    cmd = [sys.executable, "-m", "torch.distributed.run", "--nproc-per-node", "2", "--master-addr", "127.0.0.1",
           "--master-port", str(_free_port()), os.path.join(ROOT, "examples", "synthetic_grpo.py"),
           "--config", os.path.join(ROOT, "libra_b200", "configs", "tiny_cpu_gloo.yaml"), "--total-steps", str(steps),
           "--log-dir", str(tmp_path), "--stats-out", str(out), "--task", task, *extra]
    proc = subprocess.run(cmd, env=env, capture_output=True, text=True, timeout=600)
    assert proc.returncode == 0, proc.stderr[-3000:]
    return json.loads(out.read_text())


def test_two_rank_async_grpo_plumbing(tmp_path):
    """The CPU/gloo plumbing configuration: 2 ranks, 10 steps, staleness bound 1."""
    stats = _run(tmp_path, "target_token", steps=10)
    assert stats["n_trajectories"] == 16 and stats["version"] == 10
    hist = glob.glob(str(tmp_path / "history" / "*history_*.jsonl"))
    assert hist and len(open(hist[0]).read().splitlines()) == 10
    traces = glob.glob(str(tmp_path / "phase_trace" / "phase_trace_rank*.jsonl"))
    assert len(traces) == 2
    phases = {json.loads(l)["phase"] for l in open(sorted(traces)[0]) if '"phase_span"' in l}
    assert {"collect_batch", "grpo_update", "weight_sync", "recompute_logprobs"} <= phases


def test_two_rank_agentic_multiturn(tmp_path):
    stats = _run(tmp_path, "agentic")
    assert stats["n_trajectories"] == 16


def test_periodic_evaluation_rank0_with_sentinel(tmp_path):
    """Rank 0 evaluates at step 2; rank 1 waits on the done file, not a collective."""
    stats = _run(tmp_path, "target_token", "--eval-interval", "2", EVAL_MAX_SAMPLES="6", EVAL_WAIT_POLL_S="0.1",
                 EVAL_ACCURACY_THRESHOLD="1.0")
    assert stats["version"] == 3
    assert (tmp_path / "eval" / "eval_step_2.done").read_text().strip() == "ok"
    assert not (tmp_path / "eval" / "eval_step_2.error").exists()
    rows = [json.loads(l) for l in (tmp_path / "eval" / "eval_metrics.jsonl").read_text().splitlines()]
    assert len(rows) == 1 and rows[0]["step"] == 2 and rows[0]["eval_samples"] == 6
    assert 0.0 <= rows[0]["eval_accuracy"] <= 1.0 and rows[0]["eval_failures"] == 0
    samples = (tmp_path / "eval" / "eval_samples_step_2.jsonl").read_text().splitlines()
    assert 1 <= len(samples) <= 6


def test_online_replanning_applies_forced_decisions(tmp_path):
    """Planner on, forced reconfiguration every step: rank 0 applies each decision through the
    RuntimeElasticExecutor while rank 1 answers the drain request between steps."""
    stats = _run(tmp_path, "target_token", "--replan-every", "1", steps=4, GRP_FORCE_RUNTIME_RECONFIGURE="1",
                 GRP_FORCE_ROLLOUT_TP_LIST="1")
    assert stats["version"] == 4
    recs = [json.loads(l) for l in (tmp_path / "runtime_reconfigurations.jsonl").read_text().splitlines()]
    assert [r["step"] for r in recs] == [1, 2, 3]
    assert all(r["applied"] and "peer_reconfig_drain:1" in r["actions"] for r in recs)
    assert (tmp_path / "runtime_reconfiguration" / "ready" / "rank_1.json").exists()
    hist = glob.glob(str(tmp_path / "history" / "*history_*.jsonl"))
    rows = [json.loads(l) for l in open(hist[0]).read().splitlines()]
    assert rows[-1]["resource_config"]["rollout_gpus"] == 1


def test_two_rank_pipeline_parallel_training(tmp_path):
    """Two pipeline stages of one data-parallel replica: rank 0 generates the
    batch, both stages receive the same trajectories, the update runs 1F1B."""
    stats = _run(tmp_path, "target_token", "--train-pp", "2", steps=3)
    assert stats["version"] == 3 and stats["n_trajectories"] == 32


def test_two_rank_tensor_parallel_training(tmp_path):
    """Two tensor-parallel ranks (sequence parallel) of one replica train on the same batch."""
    stats = _run(tmp_path, "target_token", "--train-tp", "2", steps=2)
    assert stats["version"] == 2 and stats["n_trajectories"] == 32


def test_two_rank_expert_parallel_training(tmp_path):
    """A mixture-of-experts model with its experts split over two data-parallel
    ranks (EP=2): each rank trains its own batch, the in-process rollout engine
    gets every expert."""
    stats = _run(tmp_path, "target_token", "--model", "tiny-moe", "--train-ep", "2", steps=2)
    assert stats["version"] == 2 and stats["n_trajectories"] == 16


def test_resume_from_checkpoint_continues_the_run(tmp_path):
    """A 2-rank run saves checkpoints every 2 steps; a second run with
    RL_TRAIN_START_STEP=2 loads version 2 (weights + sharded optimizer state)
    and finishes the remaining steps to the same final version."""
    first = _run(tmp_path, "target_token", "--save-interval", "2", steps=4)
    assert first["version"] == 4
    assert os.path.isdir(tmp_path / "checkpoints" / "v2" / "megatron_dist")
    again = _run(tmp_path, "target_token", "--save-interval", "0", steps=4, RL_TRAIN_START_STEP="2")
    assert again["resumed_from"] == 2 and again["version"] == 4
