"""Tensor-parallel rollout engine (driver + follower replay) against one rank, gloo on CPU."""

import os
import socket

import torch
import torch.distributed as dist
import torch.multiprocessing as mp


def _port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _worker(rank, world, port, out_dir):
    import datetime

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=120))
    from libra_b200.engine.rollout.llm_engine import LLMEngine
    from libra_b200.engine.rollout.sampler import SamplingParams
    from libra_b200.models.qwen3 import ParamLayout, get_config, init_params, param_shapes
    from libra_b200.parallel.tensor_parallel import shard_full_params

    cfg = get_config("tiny")
    layout = ParamLayout(param_shapes(cfg))
    full = layout.views(torch.zeros(layout.numel))
    init_params(cfg, full, seed=3)
    full = {k: (v * 4 if v.dim() > 1 else v).clone() for k, v in full.items()}  # sharper logits
    prompts = [[5, 9, 13, 17, 21], [7, 7, 7], [100, 200, 300, 400, 500, 600, 700]]
    greedy = SamplingParams(max_tokens=6, temperature=0.0)
    ref = LLMEngine(cfg, full, kv_blocks=64, block_size=4).generate_sync(prompts, greedy)
    local = shard_full_params(full, cfg, world, rank)
    eng = LLMEngine(cfg, local, kv_blocks=64, block_size=4, tp_group=dist.group.WORLD, tp_size=world,
                    tp_channel=dist.group.WORLD)
    if rank == 0:
        out = eng.generate_sync(prompts, greedy)
        again = eng.generate_sync(prompts[:1], greedy)  # prefix-cache hit path replayed by the follower
        eng.shutdown()
        assert [r.output_tokens for r in out] == [r.output_tokens for r in ref]
        assert again[0].output_tokens == ref[0].output_tokens
    else:
        eng.follower_loop()
    open(os.path.join(out_dir, f"ok_{rank}"), "w").close()
    dist.destroy_process_group()


def test_tp_rollout_matches_single_rank(tmp_path):
    mp.start_processes(_worker, args=(2, _port(), str(tmp_path)), nprocs=2, join=True, start_method="spawn")
    assert {p.name for p in tmp_path.iterdir()} == {"ok_0", "ok_1"}
