"""Asynchronous GRPO on synthetic data (no datasets or checkpoints needed).

Single-turn target-token task (reward 1 if the response contains the prompt's
seeded target token) or the multi-turn agentic task with simulated tool
returns.  Runs on CPU (gloo) or GPUs (NCCL):

    torchrun --nproc-per-node 2 --master-addr 127.0.0.1 examples/synthetic_grpo.py \\
        --config libra_b200/configs/tiny_cpu_gloo.yaml
"""

import argparse
import json
import os
import sys

sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))

from libra_b200.config import load_config  # noqa: E402
from libra_b200.trainer.async_rl_trainer import AsyncRLTrainer  # noqa: E402
from libra_b200.workflow.synthetic_workflows import (AgenticSpec, SyntheticAgenticWorkflow,  # noqa: E402
                                                     TargetTokenWorkflow, target_token_dataset)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--config", required=True)
    ap.add_argument("--task", choices=["target_token", "agentic"], default="target_token")
    ap.add_argument("--num-prompts", type=int, default=64)
    ap.add_argument("--total-steps", type=int, default=0)
    ap.add_argument("--log-dir", default="")
    ap.add_argument("--stats-out", default="")
    ap.add_argument("--eval-interval", type=int, default=-1, help="override eval_interval (-1 = keep the config's)")
    ap.add_argument("--train-tp", type=int, default=0, help="override train_tp_size")
    ap.add_argument("--train-pp", type=int, default=0, help="override train_pp_size")
    ap.add_argument("--train-ep", type=int, default=0, help="override train_ep_size")
    ap.add_argument("--model", default="", help="override model_path (a preset name) and its architecture summary")
    ap.add_argument("--save-interval", type=int, default=-1, help="override save_interval (-1 = keep the config's)")
    ap.add_argument("--replan-every", type=int, default=0,
                    help="turn on the Global Resource Planner with online replanning every N steps")
    a = ap.parse_args()
    cfg = load_config(a.config)
    if a.train_tp or a.train_pp or a.train_ep or a.model:
        from libra_b200.config import AsyncRLConfig, read_config_file

        d = cfg.to_dict()
        d.update(train_dp_size=0, tp_size=0)
        if a.train_ep:
            d["train_ep_size"] = a.train_ep
        if a.model:
            d["model_path"] = a.model
            arch = os.path.join(os.path.dirname(os.path.abspath(a.config)), "model_arch_config", f"{a.model}.yaml")
            if os.path.exists(arch):
                d["model_arch"] = read_config_file(arch)
        if a.train_tp:
            d["train_tp_size"] = a.train_tp
        if a.train_pp:
            d["train_pp_size"] = a.train_pp
        cfg = AsyncRLConfig.from_dict(d)  # validated and derived again (data-parallel size)
    if a.replan_every > 0:
        p = cfg.global_resource_planner
        p.enabled, p.initial_allocation_strategy = True, "configured"
        p.plan_interval, p.warmup_steps, p.min_history_size = a.replan_every, 1, 1
        p.runtime_async_planning, p.runtime_dynamic_reconfiguration_enabled = False, True
    if a.total_steps:
        cfg.total_steps = a.total_steps
    if a.eval_interval >= 0:
        cfg.eval_interval = a.eval_interval
    if a.save_interval >= 0:
        cfg.save_interval = a.save_interval
    if a.log_dir:
        cfg.log_dir = a.log_dir
        cfg.sync_path = os.path.join(a.log_dir, "weights")
        cfg.history_output_dir = os.path.join(a.log_dir, "history")
    vocab = int(cfg.model_arch.vocab_size)
    data = target_token_dataset(a.num_prompts, vocab=vocab, seed=cfg.seed)
    if a.task == "target_token":
        wf = TargetTokenWorkflow(max_new_tokens=cfg.max_new_tokens, temperature=cfg.temperature)
    else:
        wf = SyntheticAgenticWorkflow(AgenticSpec(turn_max_tokens=cfg.max_new_tokens, context_cap=cfg.max_seq_length,
                                                  vocab=vocab, tool_len_median=16, tool_len_max=32,
                                                  tool_latency_median_s=0.01), latency_scale=1.0)
    trainer = AsyncRLTrainer(cfg)
    stats = trainer.train(wf, data)
    if trainer.is_main_process and a.stats_out:
        with open(a.stats_out, "w") as fh:
            json.dump({k: v for k, v in stats.items() if isinstance(v, (int, float, str))}, fh, indent=2)
    if trainer.world_size > 1:
        import torch.distributed as dist

        dist.destroy_process_group()


if __name__ == "__main__":
    main()
