"""Distributed-optimizer AdamW fused with the parameter all-gather (peer memory) against
AdamW + NCCL all_gather_into_tensor."""

import os
import socket

import pytest
import torch

HP = dict(lr=1e-3, beta1=0.9, beta2=0.95, eps=1e-8, weight_decay=0.1, max_grad_norm=1.0)


def _state(n, seed):
    g = torch.Generator(device="cuda").manual_seed(seed)
    master = torch.randn(n, device="cuda", generator=g)
    return master, torch.zeros_like(master), torch.zeros_like(master)


@pytest.mark.gpu
def test_single_rank_fused_adamw_matches_adamw():
    from libra_b200 import ops
    from libra_b200.parallel.peer_param_gather import PeerParamGather

    n = 1_000_003  # exercises the scalar tail
    flat = torch.zeros(n, dtype=torch.bfloat16, device="cuda")
    ref_flat = torch.zeros_like(flat)
    m1, a1, b1 = _state(n, 0)
    m2, a2, b2 = (t.clone() for t in (m1, a1, b1))
    pg = PeerParamGather(None, flat, 0, n)
    for step in range(1, 4):
        grad = torch.randn(n, device="cuda", generator=torch.Generator(device="cuda").manual_seed(step))
        sq = grad.pow(2).sum().reshape(1)
        pg.step(m1, grad, a1, b1, step=step, sq_norm=sq, **HP)
        ops.adamw_step(m2, grad, a2, b2, ref_flat, step=step, sq_norm=sq, **HP)
    torch.cuda.synchronize()
    ops.check_kernel_errors()
    assert torch.equal(m1, m2) and torch.equal(a1, a2) and torch.equal(b1, b2)
    assert torch.equal(flat, ref_flat)
    pg.close()


def _port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _worker(rank, world, port, out_dir):
    import datetime

    import torch.distributed as dist

    from libra_b200 import ops
    from libra_b200.parallel.peer_param_gather import PeerParamGather

    torch.cuda.set_device(rank)
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60),
                            device_id=torch.device("cuda", rank))
    grp = dist.group.WORLD
    shard = 1 << 20
    flat = torch.zeros(world * shard, dtype=torch.bfloat16, device="cuda")
    ref_flat = torch.zeros_like(flat)
    m1, a1, b1 = _state(shard, 100 + rank)
    m2, a2, b2 = (t.clone() for t in (m1, a1, b1))
    pg = PeerParamGather(grp, flat, rank * shard, shard)
    for step in range(1, 4):
        grad = torch.randn(shard, device="cuda", generator=torch.Generator(device="cuda").manual_seed(10 * step + rank))
        sq = grad.pow(2).sum().reshape(1)
        dist.all_reduce(sq, group=grp)
        pg.step(m1, grad, a1, b1, step=step, sq_norm=sq, **HP)
        mine = ref_flat[rank * shard:(rank + 1) * shard]
        ops.adamw_step(m2, grad, a2, b2, mine, step=step, sq_norm=sq, **HP)
        dist.all_gather_into_tensor(ref_flat, mine.clone(), group=grp)
        torch.cuda.synchronize()
        ops.check_kernel_errors()
        assert torch.equal(flat, ref_flat), f"step {step}"
    assert torch.equal(m1, m2)
    pg.close()
    dist.barrier()
    open(os.path.join(out_dir, f"ok_{rank}"), "w").close()
    dist.destroy_process_group()


@pytest.mark.gpu
@pytest.mark.multigpu
def test_two_rank_fused_adamw_allgather(tmp_path):
    import torch.multiprocessing as mp

    mp.start_processes(_worker, args=(2, _port(), str(tmp_path)), nprocs=2, join=True, start_method="spawn")
    assert {p.name for p in tmp_path.iterdir()} == {"ok_0", "ok_1"}
