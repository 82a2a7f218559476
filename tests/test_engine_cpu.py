"""CPU (reference-op) path of the training engine and GRPO math."""

import torch

from libra_b200.engine.train_engine import B200TrainEngine
from libra_b200.ops import reference as ref
from libra_b200.workflow.synthetic import WORKLOADS, group_normalize


def _trajs(n=8, seed=0):
    return WORKLOADS["tiny-cpu"].trajectories(seed)[:n]


def test_grpo_loss_matches_reference_formula():
    torch.manual_seed(0)
    logp, old = torch.randn(50) * 0.1 - 2, torch.randn(50) * 0.1 - 2
    adv = torch.randn(50)
    eng = B200TrainEngine("tiny", device="cpu")
    loss, pg, kl = eng.loss(logp, old, adv)
    rl, rpg, rkl = ref.grpo_loss(logp, old, torch.ones(50), adv, 0.2, 0.001)
    assert torch.allclose(loss, rl) and torch.allclose(kl, rkl) and kl >= 0


def test_group_normalize_rules():
    ts = [{"rewards": torch.tensor([r]), "grpo_group_id": g} for g, r in
          [("a", 1.0), ("a", 0.0), ("b", 1.0), ("b", 1.0), ("c", 0.7)]]
    group_normalize(ts)
    assert ts[0]["advantages"].item() > 0 > ts[1]["advantages"].item()
    assert ts[2]["advantages"].item() == 0.0 and ts[3]["advantages"].item() == 0.0
    assert abs(ts[4]["advantages"].item() - 0.7) < 1e-6


def test_recompute_then_update_is_on_policy():
    eng = B200TrainEngine("tiny", device="cpu", micro_batch_size=4, learning_rate=1e-3, seed=0)
    eng.initialize()
    trajs = _trajs()
    eng.recompute_logprobs(trajs)
    stats = eng.grpo_update(trajs)
    # logprobs equal old logprobs on the first update -> ratio 1 -> kl 0
    assert abs(stats["kl"]) < 1e-6
    assert stats["n_samples"] == 8.0
    stats2 = eng.grpo_update(trajs)
    assert stats2["kl"] > 0


def test_packing_skips_prompt_rows():
    eng = B200TrainEngine("tiny", device="cpu")
    trajs = _trajs(2)
    packed = eng.pack(trajs)
    b = packed["batch"]
    n_actions = sum(int(t["loss_mask"][:, 1:].sum()) for t in trajs)
    assert b.action_rows.numel() == n_actions == packed["old_logp"].numel()
    assert torch.equal(b.tokens[b.action_rows + 1], b.action_targets)


def test_loss_weights_make_gradient_chunking_invariant():
    trajs = _trajs(8, seed=3)
    grads = []
    for budget in (10 ** 6, 60):
        eng = B200TrainEngine("tiny", device="cpu", micro_batch_size=4, seed=5, max_tokens_per_micro_batch=budget)
        eng.initialize()
        eng.recompute_logprobs(trajs)
        chunks = eng.prepare_update(trajs)
        if budget == 60:
            assert len(chunks) > 2
        eng.flat_grad.zero_()
        for c in chunks:
            lp = eng.model.action_logprobs(c["batch"])
            loss, _, _ = eng.loss(lp, c["old_logp"], c["adv"], c["w"])
            loss.backward()
        grads.append(eng.flat_grad.clone())
    # identical maths; only bf16 rounding of differently blocked CPU matmuls differs
    assert ((grads[0] - grads[1]).norm() / grads[0].norm()).item() < 2e-2


def test_loss_weights_match_reference_group_mean():
    trajs = _trajs(8, seed=4)
    eng = B200TrainEngine("tiny", device="cpu", micro_batch_size=4)
    w = eng.loss_weights(trajs)
    counts = [int(t["loss_mask"][:, 1:].sum()) for t in trajs]
    g0 = sum(counts[:4])
    assert abs(w[0] - 1.0 / (g0 * 2)) < 1e-12
    total = sum(wi * c for wi, c in zip(w, counts))
    assert abs(total - 1.0) < 1e-9  # mean of two group means -> weights sum to 1


def test_fused_param_gather_declines_without_sharded_nccl_optimizer():
    """The peer-memory AdamW + parameter all-gather only applies to a sharded optimizer on NCCL ranks;
    elsewhere the switch leaves the plain optimizer step in place."""
    import pytest

    eng = B200TrainEngine("tiny", device="cpu")
    with pytest.raises(RuntimeError):
        eng.enable_fused_param_gather()  # before initialize()
    eng.initialize()
    assert eng.enable_fused_param_gather() is False
    assert getattr(eng, "_peer_param_gather", None) is None


def test_grouped_moe_matches_looped_reference():
    """Padded grouped MoE (device-side layout, one grouped GEMM per projection) equals the per-expert loop."""
    import torch

    from libra_b200.models.moe import expert_layout, moe_mlp, moe_mlp_looped
    from libra_b200.models.qwen3 import get_config

    cfg = get_config("tiny-moe")
    g = torch.Generator().manual_seed(0)
    T, H, E, F = 37, cfg.hidden_size, cfg.num_experts, cfg.moe_intermediate_size
    h = torch.randn(T, H, generator=g)
    res = torch.randn(T, H, generator=g)
    router = torch.randn(E, H, generator=g) * 0.1
    w1 = torch.randn(E, 2 * F, H, generator=g) * 0.05
    w2 = torch.randn(E, H, F, generator=g) * 0.05
    ref = moe_mlp_looped(h, res, router, w1, w2, cfg)
    got = moe_mlp(h, res, router, w1, w2, cfg)
    assert torch.allclose(got.float(), ref.float(), atol=1e-4, rtol=1e-4)
    offs, rows = expert_layout(torch.tensor([[3, 1], [1, 1], [7, 3]]), 8)
    assert offs.tolist() == [0, 0, 128, 128, 256, 256, 256, 256, 384]
    assert rows.tolist() == [128, 0, 1, 2, 256, 129]


def test_optimizer_offload_and_precision_aware_state(tmp_path):
    """Optimizer CPU offload (a fraction of the shard stepped on the host) gives
    the same parameters as the all-device step; bf16 moments (precision-aware
    optimizer) track the fp32 ones closely; the split state round-trips through
    the distributed checkpoint."""
    from libra_b200.engine.checkpointing import DistributedCheckpointManager

    trajs = _trajs()
    engines = {}
    for name, kw in {"plain": {}, "offload": dict(optimizer_cpu_offload=True, optimizer_offload_fraction=0.4),
                     "bf16": dict(precision_aware_optimizer=True)}.items():
        eng = B200TrainEngine("tiny", device="cpu", micro_batch_size=4, learning_rate=1e-3, seed=0, **kw)
        eng.initialize()
        for _ in range(3):
            eng.recompute_logprobs(trajs)
            eng.grpo_update(trajs)
        engines[name] = eng
    plain, off, bf = engines["plain"], engines["offload"], engines["bf16"]
    assert off._offload_k > 0 and off.master.numel() + off._offload_k == plain.master.numel()
    assert bf.exp_avg.dtype == torch.bfloat16 and plain.exp_avg.dtype == torch.float32
    torch.testing.assert_close(off.flat_param.float(), plain.flat_param.float(), rtol=0, atol=0)
    full = off.optimizer_state_tensors()
    for n in ("master", "exp_avg", "exp_avg_sq"):
        torch.testing.assert_close(full[n], getattr(plain, n), rtol=1e-6, atol=1e-7)
    torch.testing.assert_close(bf.flat_param.float(), plain.flat_param.float(), rtol=2e-2, atol=2e-3)
    rel = ((bf.exp_avg.float() - plain.exp_avg).norm() / plain.exp_avg.norm()).item()
    assert rel < 2e-2, rel
    # checkpoint round trip of the split state
    mgr = DistributedCheckpointManager(str(tmp_path / "ck"))
    mgr.save(off, 3, include_optimizer=True)
    fresh = B200TrainEngine("tiny", device="cpu", micro_batch_size=4, learning_rate=1e-3, seed=1,
                            optimizer_cpu_offload=True, optimizer_offload_fraction=0.4)
    fresh.initialize()
    mgr.load(fresh, 3)
    back = fresh.optimizer_state_tensors()
    for n in ("master", "exp_avg", "exp_avg_sq"):
        torch.testing.assert_close(back[n], full[n], rtol=0, atol=0)
