"""Train-engine elastic hooks: payload merge before the DP reduction, snapshots,
hybrid-side gradient payloads (CPU, tiny model)."""

import pytest
import torch

from libra_b200.engine.train_engine import B200TrainEngine
from libra_b200.infra.elastic.hybrid_pool import GradientPayload
from libra_b200.workflow.synthetic import GRPOWorkload, LengthDist


@pytest.fixture()
def engine():
    e = B200TrainEngine("tiny", device="cpu", use_distributed_optimizer=False)
    e.initialize()
    return e


def test_active_payload_merges_into_flat_grad(engine):
    d = engine.configure_elastic_training()
    assert d.core_replica_ids == ("dp0",) and d.decoupled_communication_domains
    d.request_join("h0", "dp0")
    engine.flat_grad.fill_(1.0)
    engine.enqueue_hybrid_gradient_payload(
        GradientPayload("h0", "dp0", (torch.full_like(engine.flat_grad, 2.0),), step=engine.step_count + 1,
                        membership_epoch=d.membership_epoch("h0")))
    assert engine._apply_elastic_inter_replica_gradients() == 0  # still joining: counts as zero
    assert torch.all(engine.flat_grad == 1.0)
    d.mark_active("h0")
    ep = d.membership_epoch("h0")
    for step in (engine.step_count + 1, engine.step_count + 5):  # the second is stale and dropped
        engine.enqueue_hybrid_gradient_payload(
            GradientPayload("h0", "dp0", (torch.full_like(engine.flat_grad, 2.0),), step=step, membership_epoch=ep))
    assert engine._apply_elastic_inter_replica_gradients() == 1
    assert torch.all(engine.flat_grad == 3.0)
    assert engine._pending_hybrid_gradients == []


def test_no_domain_or_no_payload_is_a_noop(engine):
    engine.flat_grad.fill_(1.0)
    engine.enqueue_hybrid_gradient_payload(GradientPayload("h0", "dp0", (torch.ones_like(engine.flat_grad),)))
    assert engine._apply_elastic_inter_replica_gradients() == 0 and torch.all(engine.flat_grad == 1.0)


def test_snapshot_roundtrip(engine, tmp_path, monkeypatch):
    monkeypatch.setenv("ELASTIC_TRAINING_STATE_DIR", str(tmp_path))
    engine.set_version(4)
    before = engine.flat_param.clone()
    v = engine.capture_elastic_state_snapshot("r0", "dp0")
    assert v == 4 and (tmp_path / "v4" / "rank_0.pt").exists()
    engine.flat_param.add_(1.0)
    engine.set_version(9)
    assert engine.load_elastic_state_snapshot(str(tmp_path / "v4" / "rank_0.pt")) == 4
    assert torch.equal(engine.flat_param, before)


def test_hybrid_gradient_then_lockstep_update_matches_core(engine):
    trajs = GRPOWorkload("t", vocab_size=engine.cfg.vocab_size, prompts_per_step=2, group_size=4,
                         prompt=LengthDist(12, 0.3, 4, 24), response=LengthDist(16, 0.3, 2, 32)).trajectories(0)
    engine.recompute_logprobs(trajs)
    hybrid = B200TrainEngine("tiny", device="cpu", use_distributed_optimizer=False)
    hybrid.initialize()
    hybrid.flat_param.copy_(engine.flat_param)
    hybrid.master.copy_(engine.master)
    p = hybrid.compute_gradient_payload(trajs, replica_id="h", target_core_id="dp0", step=1, membership_epoch=2)
    assert p.tensors[0] is hybrid.flat_grad and float(p.tensors[0].abs().sum()) > 0
    engine.grpo_update(trajs)
    hybrid.apply_gradient_update(engine.flat_grad.clone())
    torch.testing.assert_close(hybrid.flat_param.float(), engine.flat_param.float(), rtol=0, atol=0)
