"""AsyncRLTrainer with the colocated rollout backend (CPU, one rank): every
step generates through the rank's own engine, trains, and syncs the weights
into the engine with one flat copy."""

import torch

from libra_b200.config import AsyncRLConfig
from libra_b200.trainer.async_rl_trainer import AsyncRLTrainer
from libra_b200.workflow.synthetic import GRPOWorkload, LengthDist, rollout_requests
from libra_b200.workflow.synthetic_workflows import GRPOLengthWorkflow, grpo_length_dataset


def test_colocated_trainer_steps_and_syncs(tmp_path):
    wl = GRPOWorkload("t", vocab_size=1024, prompts_per_step=2, group_size=4, prompt=LengthDist(20, 0.3, 8, 32),
                      response=LengthDist(10, 0.5, 1, 16))
    reqs = []
    for s in range(4):
        reqs += rollout_requests(wl, s, prompts=2)
    cfg = AsyncRLConfig.from_dict({
        "model_path": "tiny", "rollout_backend": "colocated", "train_gpus": 1, "rollout_gpus": 0,
        "batch_size": 8, "n_samples": 4, "micro_batch_size": 4, "max_concurrent_rollouts": 16,
        "max_head_offpolicyness": 1, "total_steps": 3, "sync_interval": 1, "max_seq_length": 64,
        "learning_rate": 1e-3, "enable_history_collection": False, "log_dir": str(tmp_path / "l"),
        "sync_path": str(tmp_path / "s"), "save_interval": 0, "global_resource_planner": {"enabled": False},
        "heterogeneous_rollout": {"enabled": False}})
    tr = AsyncRLTrainer(cfg)
    seen = []
    tr.step_callback = lambda step, stats, batch: seen.append((step, len(batch), stats["version"]))
    tr.train(GRPOLengthWorkflow(), grpo_length_dataset(reqs))
    assert [s for s, _, _ in seen] == [0, 1, 2]
    assert all(n == 8 for _, n, _ in seen) and seen[-1][2] == 3
    llm = tr._local_engines[0]
    assert llm.version == 3 and torch.equal(llm.flat, tr.train_engine.flat_param)


def test_hetero_pool_runs_tp2_bucket_as_server_processes(tmp_path):
    """A heterogeneous pool with a TP-1 in-process instance and a TP-2 bucket:
    the TP-2 bucket runs as two server processes (gloo on CPU), receives the
    trainer's weights at start and after every step (checkpoint reload on CPU;
    peer-memory reshard on GPUs), and serves rollouts to the C-MLFQ pool."""
    import json
    import urllib.request

    wl = GRPOWorkload("t", vocab_size=1024, prompts_per_step=2, group_size=4, prompt=LengthDist(20, 0.3, 8, 32),
                      response=LengthDist(6, 0.5, 1, 8))
    reqs = []
    for s in range(3):
        reqs += rollout_requests(wl, s, prompts=2)
    cfg = AsyncRLConfig.from_dict({
        "model_path": "tiny", "rollout_backend": "native", "train_gpus": 1, "rollout_gpus": 3,
        "batch_size": 8, "n_samples": 4, "micro_batch_size": 4, "max_concurrent_rollouts": 16,
        "max_head_offpolicyness": 1, "total_steps": 2, "sync_interval": 1, "max_seq_length": 64,
        "learning_rate": 1e-3, "enable_history_collection": False, "log_dir": str(tmp_path / "l"),
        "sync_path": str(tmp_path / "s"), "save_interval": 0, "global_resource_planner": {"enabled": False},
        "heterogeneous_rollout": {"enabled": True, "startup_timeout": 240,
                                  "instances": [{"tp": 1, "gpus": [0]}, {"tp": 2, "gpus": [1, 2]}],
                                  "scheduling": {"scheduler_type": "cmlfq"}}})
    tr = AsyncRLTrainer(cfg)
    seen, groups = [], []

    def on_step(step, stats, batch):
        groups[:] = list(tr._tp_groups)
        with urllib.request.urlopen(groups[0].base_url + "/health", timeout=10) as r:
            seen.append((step, stats["version"], json.loads(r.read())["version"]))

    tr.step_callback = on_step
    try:
        tr.train(GRPOLengthWorkflow(), grpo_length_dataset(reqs))
    finally:
        tr.shutdown()
    assert [s for s, _, _ in seen] == [0, 1]
    assert len(groups) == 1 and groups[0].tp == 2
    # the server group holds the weights of the version the trainer just produced
    assert all(v_trainer == v_server for _, v_trainer, v_server in seen), seen
    assert not tr._tp_groups and groups[0].proc.poll() is not None  # stopped with the trainer
