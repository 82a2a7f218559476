"""Sequence parallelism on two GPUs (NCCL): the fused GEMM + reduce-scatter and
all-gather + GEMM kernels (peer memory) inside the TP model, against the same
model without sequence parallelism."""

import os
import socket

import pytest
import torch

pytestmark = [pytest.mark.gpu, pytest.mark.multigpu]


def _port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _run(model, batch):
    lp = model.action_logprobs(batch)
    w = torch.linspace(0.5, 1.5, lp.numel(), device=lp.device)
    (lp.float() * w).sum().backward()
    return lp.detach().float()


def _worker(rank, world, port, out_dir):
    import datetime

    import torch.distributed as dist

    from libra_b200 import ops
    from libra_b200.models.qwen3 import ParamLayout, Qwen3Model, get_config, init_params, pack_sequences, param_shapes
    from libra_b200.parallel.sequence_parallel import (disable_fused_sequence_parallel,
                                                       enable_fused_sequence_parallel, sp_multiple)
    from libra_b200.parallel.tensor_parallel import shard_full_params, tp_partial_grad_params

    torch.cuda.set_device(rank)
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=120),
                            device_id=torch.device("cuda", rank))
    dev = torch.device("cuda", rank)
    grp = dist.group.WORLD
    cfg = get_config("tiny-gpu")
    layout = ParamLayout(param_shapes(cfg))
    flat = torch.zeros(layout.numel, dtype=torch.bfloat16, device=dev)
    init_params(cfg, layout.views(flat), seed=5)
    local = shard_full_params(layout.views(flat), cfg, world, rank)
    g = torch.Generator().manual_seed(0)
    seqs = [torch.randint(4, cfg.vocab_size, (n,), generator=g) for n in (700, 137, 290)]
    m = sp_multiple(world, dev)
    batch = pack_sequences(seqs, pad_multiple=m).to(dev)
    assert batch.num_tokens % m == 0
    # fused kernels: GEMM + reduce-scatter for width H; all-gather + GEMM for the qkv input shard
    enable_fused_sequence_parallel(grp, batch.num_tokens, [cfg.hidden_size],
                                   [(batch.num_tokens // world, cfg.hidden_size)], dev)
    results = {}
    for sp in (False, True):
        ps = {k: torch.nn.Parameter(v.clone()) for k, v in local.items()}
        model = Qwen3Model(cfg, ps, tp_group=grp, tp_size=world, tp_rank=rank, sequence_parallel=sp)
        lp = _run(model, batch)
        grads = {k: p.grad.float() for k, p in ps.items()}
        for n in tp_partial_grad_params(list(grads), sequence_parallel=sp):
            dist.all_reduce(grads[n], group=grp)
        results[sp] = (lp, grads)
    torch.cuda.synchronize()
    ops.check_kernel_errors()
    lp0, g0 = results[False]
    lp1, g1 = results[True]
    assert (lp1 - lp0).abs().max().item() < 0.05, (lp1 - lp0).abs().max().item()
    for n in g0:
        rel = ((g1[n] - g0[n]).norm() / g0[n].norm().clamp_min(1e-12)).item()
        assert rel < 0.05, (n, rel)
    disable_fused_sequence_parallel()
    dist.barrier()
    open(os.path.join(out_dir, f"ok_{rank}"), "w").close()
    dist.destroy_process_group()


def test_tp2_sequence_parallel_fused(tmp_path):
    import torch.multiprocessing as mp

    mp.start_processes(_worker, args=(2, _port(), str(tmp_path)), nprocs=2, join=True, start_method="spawn")
    assert {p.name for p in tmp_path.iterdir()} == {"ok_0", "ok_1"}
