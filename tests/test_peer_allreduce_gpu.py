"""Peer-memory TP all-reduce + residual + RMSNorm kernel against torch."""

import os
import socket

import pytest
import torch


def _ref(partials, residual, w, eps):
    x = (residual.float() + sum(p.float() for p in partials)).bfloat16()
    h = (x.float() * torch.rsqrt(x.float().pow(2).mean(-1, keepdim=True) + eps) * w.float()).bfloat16()
    return x, h


@pytest.mark.gpu
def test_single_rank_kernel_matches_reference():
    from libra_b200 import ops
    from libra_b200.parallel.peer_allreduce import PeerAllReduce

    par = PeerAllReduce(None, max_rows=64, hidden=2560, device="cuda")
    for rows in (1, 37, 64):
        y = torch.randn(rows, 2560, device="cuda").bfloat16()
        res = torch.randn(rows, 2560, device="cuda").bfloat16()
        w = torch.rand(2560, device="cuda").bfloat16()
        par.partial(rows).copy_(y)
        x, h = par.reduce_add_rmsnorm(res, w, 1e-6)
        torch.cuda.synchronize()
        ops.check_kernel_errors()
        rx, rh = _ref([y], res, w, 1e-6)
        torch.testing.assert_close(x.float(), rx.float(), rtol=1e-2, atol=1e-2)
        torch.testing.assert_close(h.float(), rh.float(), rtol=2e-2, atol=2e-2)


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
    from libra_b200.parallel.peer_allreduce import PeerAllReduce

    torch.cuda.set_device(rank)
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60),
                            device_id=torch.device("cuda", rank))
    par = PeerAllReduce(dist.group.WORLD, max_rows=128, hidden=2560, device="cuda")
    g = torch.Generator(device="cuda").manual_seed(0)
    for it, rows in enumerate((128, 7, 96, 128)):
        ys = [torch.randn(rows, 2560, device="cuda", generator=g).bfloat16() for _ in range(world)]
        res = torch.randn(rows, 2560, device="cuda", generator=g).bfloat16()
        w = torch.rand(2560, device="cuda", generator=g).bfloat16()
        par.partial(rows).copy_(ys[rank])
        x, h = par.reduce_add_rmsnorm(res, w, 1e-6)
        torch.cuda.synchronize()
        ops.check_kernel_errors()
        rx, rh = _ref(ys, res, w, 1e-6)
        torch.testing.assert_close(x.float(), rx.float(), rtol=1e-2, atol=2e-2)
        torch.testing.assert_close(h.float(), rh.float(), rtol=2e-2, atol=3e-2)
    dist.barrier()
    open(os.path.join(out_dir, f"ok_{rank}"), "w").close()
    dist.destroy_process_group()


@pytest.mark.gpu
@pytest.mark.multigpu
def test_two_rank_peer_allreduce(tmp_path):
    import torch.multiprocessing as mp

    mp.start_processes(_worker, args=(2, _port(), str(tmp_path)), nprocs=2, join=True, start_method="spawn")
    assert {p.name for p in tmp_path.iterdir()} == {"ok_0", "ok_1"}
