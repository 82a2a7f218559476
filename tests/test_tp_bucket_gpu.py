"""A TP-2 rollout bucket as two server processes on two GPUs, fed by the
trainer over peer memory: every step the trainer publishes its flat bf16
buffer (CUDA IPC handle as JSON) and each server rank reshards its own TP slice
into its served weights with the weight_reshard kernel."""

import json
import urllib.request

import pytest

pytestmark = [pytest.mark.gpu, pytest.mark.multigpu]


def test_trainer_syncs_tp2_bucket_over_peer_memory(tmp_path):
    from libra_b200.config import AsyncRLConfig
    from libra_b200.trainer.async_rl_trainer import AsyncRLTrainer
    from libra_b200.workflow.synthetic import GRPOWorkload, LengthDist, rollout_requests
    from libra_b200.workflow.synthetic_workflows import GRPOLengthWorkflow, grpo_length_dataset

    wl = GRPOWorkload("t", vocab_size=2048, prompts_per_step=2, group_size=4, prompt=LengthDist(40, 0.3, 8, 64),
                      response=LengthDist(12, 0.5, 1, 24))
    reqs = []
    for s in range(3):
        reqs += rollout_requests(wl, s, prompts=2)
    cfg = AsyncRLConfig.from_dict({
        "model_path": "tiny-gpu", "rollout_backend": "native", "train_gpus": 1, "rollout_gpus": 2,
        "batch_size": 8, "n_samples": 4, "micro_batch_size": 4, "max_concurrent_rollouts": 16,
        "max_head_offpolicyness": 1, "total_steps": 2, "sync_interval": 1, "max_seq_length": 128,
        "learning_rate": 1e-4, "enable_history_collection": False, "log_dir": str(tmp_path / "l"),
        "sync_path": str(tmp_path / "s"), "save_interval": 0, "global_resource_planner": {"enabled": False},
        "heterogeneous_rollout": {"enabled": True, "startup_timeout": 300, "gpu_memory_utilization": 0.2,
                                  "instances": [{"tp": 2, "gpus": [0, 1]}],
                                  "scheduling": {"scheduler_type": "cmlfq"}}})
    tr = AsyncRLTrainer(cfg)
    seen = []

    def on_step(step, stats, batch):
        g = tr._tp_groups[0]
        with urllib.request.urlopen(g.base_url + "/health", timeout=10) as r:
            seen.append((step, stats["version"], json.loads(r.read())["version"]))

    tr.step_callback = on_step
    try:
        tr.train(GRPOLengthWorkflow(), grpo_length_dataset(reqs))
    finally:
        tr.shutdown()
    assert [s for s, _, _ in seen] == [0, 1]
    assert all(a == b for _, a, b in seen), seen
