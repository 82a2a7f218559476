"""Fused tensor-parallel GEMM + peer-memory all-reduce against torch."""

import os
import socket

import pytest
import torch


def _inputs(rank, M, K, N, b_mn, seed):
    g = torch.Generator(device="cuda").manual_seed(seed * 100 + rank)
    a = (torch.randn(M, K, device="cuda", generator=g) * 0.5).bfloat16()
    w = (torch.randn(N, K, device="cuda", generator=g) / K ** 0.5).bfloat16()
    return a, (w.t().contiguous() if b_mn else w), w


@pytest.mark.gpu
def test_single_rank_fused_gemm_allreduce():
    from libra_b200 import ops
    from libra_b200.parallel.peer_gemm import PeerGemmAllReduce

    f = PeerGemmAllReduce(None, max_rows=4096, n_cols=2560, device="cuda")
    for it, (M, b_mn) in enumerate([(4096, False), (37, False), (1000, True), (4096, True)]):
        a, wop, w = _inputs(0, M, 512, 2560, b_mn, it)
        res = torch.randn(M, 2560, device="cuda").bfloat16() if it % 2 == 0 else None
        y = f(a, wop, res, b_mn=b_mn)
        torch.cuda.synchronize()
        ops.check_kernel_errors()
        ref = a.float() @ w.float().t() + (res.float() if res is not None else 0)
        torch.testing.assert_close(y.float(), ref, rtol=2e-2, atol=2e-2)
    # reduce-scatter with one rank: the whole sum
    a, wop, w = _inputs(0, 1024, 512, 2560, False, 9)
    y = f.reduce_scatter(a, wop)
    torch.testing.assert_close(y.float(), a.float() @ w.float().t(), rtol=2e-2, atol=2e-2)


@pytest.mark.gpu
def test_single_rank_fused_allgather_gemm():
    from libra_b200 import ops
    from libra_b200.parallel.peer_gemm import PeerAllGatherGemm

    f = PeerAllGatherGemm(None, shard_rows=1024, k_cols=512, device="cuda")
    for it, b_mn in enumerate([False, True, False]):
        a, wop, w = _inputs(0, 1024, 512, 3072, b_mn, 20 + it)
        y = f(a, wop, b_mn=b_mn)
        torch.cuda.synchronize()
        ops.check_kernel_errors()
        torch.testing.assert_close(y.float(), a.float() @ w.float().t(), rtol=2e-2, atol=2e-2)


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
    from libra_b200.parallel import peer_gemm
    from libra_b200.parallel.tensor_parallel import row_parallel_linear

    torch.cuda.set_device(rank)
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60),
                            device_id=torch.device("cuda", rank))
    grp = dist.group.WORLD
    f = peer_gemm.PeerGemmAllReduce(grp, max_rows=4096, n_cols=2560, device="cuda")
    K = 1024
    for it, (M, b_mn) in enumerate([(4096, False), (300, False), (2048, True), (4096, False), (1, True)]):
        parts = [_inputs(r, M, K, 2560, b_mn, it) for r in range(world)]
        res = torch.randn(M, 2560, device="cuda", generator=torch.Generator(device="cuda").manual_seed(it)).bfloat16()
        a, wop, _ = parts[rank]
        y = f(a, wop, res, b_mn=b_mn)
        torch.cuda.synchronize()
        ops.check_kernel_errors()
        ref = sum(p[0].float() @ p[2].float().t() for p in parts) + res.float()
        torch.testing.assert_close(y.float(), ref, rtol=2e-2, atol=3e-2)
    # reduce-scatter: this rank's row shard of the sum
    for it, b_mn in enumerate([False, True]):
        M = 2048
        parts = [_inputs(r, M, K, 2560, b_mn, 40 + it) for r in range(world)]
        ref = sum(p[0].float() @ p[2].float().t() for p in parts)
        y = f.reduce_scatter(parts[rank][0], parts[rank][1], b_mn=b_mn)
        torch.cuda.synchronize()
        ops.check_kernel_errors()
        rows = M // world
        torch.testing.assert_close(y.float(), ref[rank * rows:(rank + 1) * rows], rtol=2e-2, atol=3e-2)
    # all-gather of row shards fused into the GEMM
    ag = peer_gemm.PeerAllGatherGemm(grp, shard_rows=1024, k_cols=K, device="cuda")
    for it in range(3):
        shards = [_inputs(r, 1024, K, 8, False, 60 + it)[0] for r in range(world)]
        _, wop, w = _inputs(0, 8, K, 3072, it == 1, 70 + it)  # the same local weight on every rank
        y = ag(shards[rank], wop, b_mn=(it == 1))
        torch.cuda.synchronize()
        ops.check_kernel_errors()
        torch.testing.assert_close(y.float(), torch.cat(shards).float() @ w.float().t(), rtol=2e-2, atol=2e-2)
    ag.close()
    # autograd through row_parallel_linear: fused path against the NCCL path
    peer_gemm.enable_fused_row_parallel(grp, 4096, [2560], "cuda")
    a, _, w = _inputs(rank, 1536, K, 2560, False, 7)
    res = torch.randn(1536, 2560, device="cuda").bfloat16()
    outs = []
    for fused_on in (True, False):
        if not fused_on:
            peer_gemm.disable_fused_row_parallel()
        a1 = a.clone().requires_grad_(True)
        w1 = w.clone().requires_grad_(True)
        r1 = res.clone().requires_grad_(True)
        y = row_parallel_linear(a1, w1, r1, grp)
        y.float().pow(2).mean().backward()
        outs.append((y.detach(), a1.grad, w1.grad, r1.grad))
    torch.cuda.synchronize()
    ops.check_kernel_errors()
    for x1, x2 in zip(*outs):
        torch.testing.assert_close(x1.float(), x2.float(), rtol=2e-2, atol=2e-2)
    f.close()
    dist.barrier()
    open(os.path.join(out_dir, f"ok_{rank}"), "w").close()
    dist.destroy_process_group()


@pytest.mark.gpu
@pytest.mark.multigpu
def test_two_rank_fused_gemm_allreduce(tmp_path):
    import torch.multiprocessing as mp

    mp.start_processes(_worker, args=(2, _port(), str(tmp_path)), nprocs=2, join=True, start_method="spawn")
    assert {p.name for p in tmp_path.iterdir()} == {"ok_0", "ok_1"}
