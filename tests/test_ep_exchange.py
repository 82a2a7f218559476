"""Expert-parallel dispatch / combine: routing-plan layout (CPU) and the
peer-memory kernels against the plain MoE block and the NCCL all-to-all path (GPU)."""

import os
import socket

import pytest
import torch


def _ranks_inputs(n, T, E, k, seed=0):
    g = torch.Generator().manual_seed(seed)
    return [torch.stack([torch.randperm(E, generator=g)[:k] for _ in range(T)]) for _ in range(n)]


def test_route_plan_layout_is_grouped_permutation():
    from libra_b200.parallel.expert_parallel import route_plan

    n, T, E, k = 4, 37, 16, 3
    El = E // n
    experts = _ranks_inputs(n, T, E, k)
    counts = torch.stack([torch.bincount(e.reshape(-1), minlength=E) for e in experts]).to(torch.int32)
    plans = [route_plan(experts[s], counts, s) for s in range(n)]
    for d in range(n):
        rows, tags = [], []
        for s in range(n):
            sel = plans[s].dst_rank == d
            rows.append(plans[s].dst_row[sel].long())
            flat = experts[s].reshape(-1)[sel]
            tags += [(int(e) % El, s, j) for e, j in zip(flat, sel.nonzero().flatten().tolist())]
        rows = torch.cat(rows)
        ordered = [t for _, t in sorted(zip(rows.tolist(), tags))]
        assert ordered == sorted(ordered)  # (local expert, source rank, source order)
        # each local expert's rows fill the start of a group that begins on a 128-row boundary
        offs = plans[d].offs.tolist()
        real = [int(counts[:, d * El + e].sum()) for e in range(El)]
        want = [offs[e] + i for e in range(El) for i in range(real[e])]
        assert sorted(rows.tolist()) == want
        assert all(o % 128 == 0 for o in offs) and offs[-1] == plans[d].recv_total
        assert plans[d].valid.sum().item() == sum(real)


def test_route_plan_emulated_exchange_matches_moe_block():
    """Move rows exactly as the kernels do (pure torch) and compare with the unsharded MoE block."""
    from libra_b200.models.moe import moe_mlp, route
    from libra_b200.models.qwen3 import get_config
    from libra_b200.parallel.expert_parallel import route_plan

    cfg = get_config("tiny-moe")
    n, T = 2, 24
    E, H, F, k = cfg.num_experts, cfg.hidden_size, cfg.moe_intermediate_size, cfg.num_experts_per_tok
    El = E // n
    g = torch.Generator().manual_seed(3)
    hs = [torch.randn(T, H, generator=g) * 0.5 for _ in range(n)]
    res = [torch.randn(T, H, generator=g) for _ in range(n)]
    router = torch.randn(E, H, generator=g) * 0.05
    w1 = torch.randn(E, 2 * F, H, generator=g) * 0.05
    w2 = torch.randn(E, H, F, generator=g) * 0.05
    routed = [route(h, router, k, cfg.norm_topk_prob) for h in hs]
    counts = torch.stack([torch.bincount(r[1].reshape(-1), minlength=E) for r in routed]).to(torch.int32)
    plans = [route_plan(routed[s][1], counts, s) for s in range(n)]
    recv = [torch.zeros(plans[d].recv_total, H) for d in range(n)]
    for s in range(n):
        for j in range(T * k):
            recv[int(plans[s].dst_rank[j])][int(plans[s].dst_row[j])] = hs[s][j // k]
    from libra_b200 import ops

    ys = []
    for d in range(n):
        a = ops.grouped_swiglu(recv[d], w1[d * El:(d + 1) * El], plans[d].offs)
        ys.append(ops.grouped_linear(a, w2[d * El:(d + 1) * El], plans[d].offs))
    for s in range(n):
        w = routed[s][0].reshape(-1)
        got = res[s].clone()
        for j in range(T * k):
            got[j // k] += w[j] * ys[int(plans[s].dst_rank[j])][int(plans[s].dst_row[j])]
        ref = moe_mlp(hs[s], res[s], router, w1, w2, cfg)
        torch.testing.assert_close(got, ref, rtol=1e-4, atol=1e-4)


def test_grouped_linear_writes_into_caller_slot_and_keeps_grads():
    """The expert GEMM can write into a bf16 slot carved from a byte buffer (the send slot)
    without cutting the autograd history."""
    from libra_b200.models.moe import GroupedLinear

    buf = torch.zeros(256 + 6 * 8 * 2, dtype=torch.uint8)
    slot = buf[256:].view(torch.bfloat16).view(6, 8)
    x = torch.randn(6, 4).bfloat16().requires_grad_(True)
    w = torch.randn(2, 8, 4).bfloat16().requires_grad_(True)
    y = GroupedLinear.apply(x, w, [2, 4], (slot,))
    assert y.data_ptr() == slot.data_ptr()
    ref = torch.cat([x[:2].float() @ w[0].float().t(), x[2:].float() @ w[1].float().t()])
    torch.testing.assert_close(slot.float(), ref, rtol=2e-2, atol=2e-2)
    y.float().sum().backward()
    assert x.grad is not None and w.grad is not None
    torch.testing.assert_close(x.grad.float(), torch.cat([w[0].float().sum(0).expand(2, 4),
                                                          w[1].float().sum(0).expand(4, 4)]), rtol=2e-2, atol=2e-2)


def _moe_inputs(cfg, T, seed, device="cuda"):
    g = torch.Generator().manual_seed(seed)
    E, H, F = cfg.num_experts, cfg.hidden_size, cfg.moe_intermediate_size
    h = (torch.randn(T, H, generator=g) * 0.5).bfloat16().to(device)
    res = torch.randn(T, H, generator=g).bfloat16().to(device)
    router = (torch.randn(E, H, generator=g) * 0.05).to(device)
    w1 = (torch.randn(E, 2 * F, H, generator=g) * 0.05).bfloat16().to(device)
    w2 = (torch.randn(E, H, F, generator=g) * 0.05).bfloat16().to(device)
    return h, res, router, w1, w2


def _grads(fn, h, res, router, w1, w2):
    leaves = [t.clone().requires_grad_(True) for t in (h, res, router, w1, w2)]
    out = fn(*leaves)
    out.float().pow(2).mean().backward()
    return [out.detach()] + [t.grad for t in leaves]


@pytest.mark.gpu
def test_single_rank_peer_moe_matches_moe_block():
    from libra_b200 import ops
    from libra_b200.models.moe import moe_mlp
    from libra_b200.models.qwen3 import get_config
    from libra_b200.parallel.expert_parallel import PeerExpertExchange, ep_moe_mlp

    cfg = get_config("tiny-moe")
    xchg = PeerExpertExchange(None, max_rows=4096, hidden=cfg.hidden_size, device="cuda")
    for it, T in enumerate([300, 1, 1024]):
        args = _moe_inputs(cfg, T, it)
        peer = _grads(lambda h, r, ro, a, b: ep_moe_mlp(h, r, ro, a, b, cfg, None, exchange=xchg), *args)
        ref = _grads(lambda h, r, ro, a, b: moe_mlp(h, r, ro, a, b, cfg), *args)
        torch.cuda.synchronize()
        ops.check_kernel_errors()
        for name, x, y in zip(["out", "dh", "dres", "drouter", "dw1", "dw2"], peer, ref):
            torch.testing.assert_close(x.float(), y.float(), rtol=3e-2, atol=3e-2, msg=name)
    xchg.close()


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
    from libra_b200.models.qwen3 import get_config
    from libra_b200.parallel.expert_parallel import PeerExpertExchange, ep_moe_mlp

    torch.cuda.set_device(rank)
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60),
                            device_id=torch.device("cuda", rank))
    grp = dist.group.WORLD
    cfg = get_config("tiny-moe")
    El = cfg.num_experts // world
    xchg = PeerExpertExchange(grp, max_rows=8192, hidden=cfg.hidden_size, device="cuda")
    for it, T in enumerate([512, 3, 2048]):
        h, res, router, w1, w2 = _moe_inputs(cfg, T, 10 * it + rank)
        _, _, router, w1, w2 = _moe_inputs(cfg, T, 99 + it)  # weights shared by all ranks
        w1l, w2l = w1[rank * El:(rank + 1) * El].contiguous(), w2[rank * El:(rank + 1) * El].contiguous()
        outs = []
        for ex in (xchg, None):
            outs.append(_grads(lambda a, b, c, d, e: ep_moe_mlp(a, b, c, d, e, cfg, grp, exchange=ex),
                               h, res, router, w1l, w2l))
        torch.cuda.synchronize()
        ops.check_kernel_errors()
        for name, x, y in zip(["out", "dh", "dres", "drouter", "dw1", "dw2"], *outs):
            torch.testing.assert_close(x.float(), y.float(), rtol=3e-2, atol=3e-2, msg=f"{name} T={T}")
    xchg.close()
    dist.barrier()
    open(os.path.join(out_dir, f"ok_{rank}"), "w").close()
    dist.destroy_process_group()


@pytest.mark.gpu
@pytest.mark.multigpu
def test_two_rank_peer_moe_matches_nccl_path(tmp_path):
    import torch.multiprocessing as mp

    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    mp.start_processes(_worker, args=(2, _port(), str(tmp_path)), nprocs=2, join=True, start_method="spawn")
    assert {p.name for p in tmp_path.iterdir()} == {"ok_0", "ok_1"}
