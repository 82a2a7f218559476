"""Vocab-parallel log-softmax statistics exchanged over peer memory (one kernel)
against the two-all-reduce combine, on one rank and on two."""

import os
import socket

import pytest
import torch

pytestmark = pytest.mark.gpu


def _stats(R, seed, dev):
    g = torch.Generator(device=dev).manual_seed(seed)
    m = torch.randn(R, device=dev, generator=g) * 3
    s = torch.rand(R, device=dev, generator=g) * 50 + 1
    zt = torch.randn(R, device=dev, generator=g)
    return m, s, zt


def test_single_rank_exchange_matches_combine():
    from libra_b200 import ops
    from libra_b200.parallel import tensor_parallel as tp

    dev = torch.device("cuda", 0)
    x = tp.PeerLogprobExchange(None, 5000, dev)
    for call, R in enumerate([4097, 1, 5000]):  # alternating parity slots, odd sizes
        m, s, zt = _stats(R, call, dev)
        lse, z = x(m, s, zt)
        torch.cuda.synchronize()
        ops.check_kernel_errors()
        torch.testing.assert_close(lse, m + torch.log(s), rtol=1e-6, atol=1e-5)
        torch.testing.assert_close(z, zt, rtol=0, atol=0)
    x.close()


def _port():
    sck = socket.socket()
    sck.bind(("127.0.0.1", 0))
    p = sck.getsockname()[1]
    sck.close()
    return p


def _worker(rank, world, port, out_dir):
    import datetime

    import torch.distributed as dist

    from libra_b200 import ops
    from libra_b200.parallel import tensor_parallel as tp

    torch.cuda.set_device(rank)
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60),
                            device_id=torch.device("cuda", rank))
    dev = torch.device("cuda", rank)
    grp = dist.group.WORLD
    for call, R in enumerate([3000, 17, 8192]):
        m, s, zt = _stats(R, 10 * call + rank, dev)
        zt = zt * (torch.arange(R, device=dev) % world == rank)  # each target lives in one shard
        ref_lse, ref_z = tp._combine(m, s, zt, grp)  # NCCL path (nothing registered yet in call 0)
        tp.enable_peer_logprob_exchange(grp, 8192, dev)
        lse, z = tp._combine(m, s, zt, grp)
        tp.disable_peer_logprob_exchange()
        torch.cuda.synchronize()
        ops.check_kernel_errors()
        torch.testing.assert_close(lse, ref_lse, rtol=1e-6, atol=1e-5)
        torch.testing.assert_close(z, ref_z, rtol=1e-6, atol=1e-6)
    dist.barrier()
    open(os.path.join(out_dir, f"ok_{rank}"), "w").close()
    dist.destroy_process_group()


@pytest.mark.multigpu
def test_two_rank_exchange_matches_nccl(tmp_path):
    import torch.multiprocessing as mp

    mp.start_processes(_worker, args=(2, _port(), str(tmp_path)), nprocs=2, join=True, start_method="spawn")
    assert {p.name for p in tmp_path.iterdir()} == {"ok_0", "ok_1"}
