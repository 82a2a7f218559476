"""Train with a real workflow and dataset (the entry point the launchers run).

    torchrun --standalone --nproc-per-node 4 examples/train.py --config cfg.yaml \\
        --task r2e_gym --data data/r2e_gym.jsonl

Tasks: rlvr, dapo_math, r2e_gym, search_r1, code_agent, target_token (synthetic).
Rows come from ``python -m libra_b200.data.prepare``.
"""

import argparse
import json
import os
import sys

sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))

from libra_b200.config import load_config  # noqa: E402
from libra_b200.data.prepare import read_rows  # noqa: E402
from libra_b200.engine.tokenizer import load_tokenizer  # noqa: E402
from libra_b200.trainer.async_rl_trainer import AsyncRLTrainer  # noqa: E402


def build_workflow(task: str, cfg, tokenizer):
    kw = dict(tokenizer=tokenizer, max_new_tokens=cfg.max_new_tokens, max_seq_length=cfg.max_seq_length,
              temperature=cfg.temperature, top_p=cfg.top_p)
    if task == "rlvr":
        from libra_b200.workflow.rlvr import RLVRWorkflow

        return RLVRWorkflow(**kw)
    if task == "dapo_math":
        from libra_b200.workflow.dapo_math import DAPOMathWorkflow

        return DAPOMathWorkflow(**kw)
    if task == "r2e_gym":
        from libra_b200.workflow.r2e_gym import R2EGymWorkflow

        return R2EGymWorkflow(max_turns=cfg.r2e_max_turns, stop_reward=cfg.r2e_stop_reward,
                              max_prompt_tokens=cfg.r2e_max_prompt_tokens or None, **kw)
    if task == "search_r1":
        from libra_b200.workflow.search_r1 import SearchR1Workflow

        return SearchR1Workflow(**kw)
    if task == "code_agent":
        from libra_b200.workflow.code_agent import CodeAgentWorkflow

        return CodeAgentWorkflow(**kw)
    if task == "target_token":
        from libra_b200.workflow.synthetic_workflows import TargetTokenWorkflow

        return TargetTokenWorkflow(max_new_tokens=cfg.max_new_tokens, temperature=cfg.temperature)
    raise ValueError(f"unknown task {task}")


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--config", required=True)
    ap.add_argument("--task", default="rlvr")
    ap.add_argument("--data", default="")
    ap.add_argument("--limit", type=int, default=0)
    ap.add_argument("--stats-out", default="")
    a = ap.parse_args()
    cfg = load_config(a.config)
    tok = load_tokenizer(cfg.tokenizer_path or cfg.model_path, int(cfg.model_arch.vocab_size))
    if a.task == "target_token":
        from libra_b200.workflow.synthetic_workflows import target_token_dataset

        rows = target_token_dataset(a.limit or 64, vocab=int(cfg.model_arch.vocab_size), seed=cfg.seed)
    else:
        rows = read_rows(a.data)[: a.limit or None]
    trainer = AsyncRLTrainer(cfg)
    stats = trainer.train(build_workflow(a.task, cfg, tok), rows)
    if trainer.is_main_process and a.stats_out:
        with open(a.stats_out, "w") as fh:
            json.dump({k: v for k, v in stats.items() if isinstance(v, (int, float, str))}, fh, indent=2)
    if trainer.world_size > 1:
        import torch.distributed as dist

        dist.destroy_process_group()


if __name__ == "__main__":
    main()
