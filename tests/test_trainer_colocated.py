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
