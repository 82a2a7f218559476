"""Elastic Hybrid Pool state machine and inter-replica gradient domain (CPU)."""

import threading
import time

import pytest
import torch

from libra_b200.infra.elastic import hybrid_pool as hp
from libra_b200.infra.elastic.hybrid_pool import (ElasticHybridPool, GradientCommunicationDomains, GradientPayload,
                                                  InterReplicaGradientDomain, JoinCancelledError, JoinState,
                                                  PeerMemoryTransport, ReplicaJoinHandle, ReplicaRole,
                                                  TorchDistributedTransport)


def _payload(rid, core, vals, **kw):
    return GradientPayload(rid, core, (torch.tensor(vals),), **kw)


def test_joining_replica_counts_as_zero():
    d = InterReplicaGradientDomain(core_replica_ids=["c0", "c1"])
    d.request_join("h0", "c0")
    out = d.reduce_core_gradients(core_gradients={"c0": (torch.tensor([2.0, 4.0]),), "c1": (torch.tensor([4.0, 8.0]),)},
                                  hybrid_payloads=[_payload("h0", "c0", [50.0, 50.0])])
    assert torch.equal(out["c0"][0], torch.tensor([3.0, 6.0])) and torch.equal(out["c1"][0], out["c0"][0])


def test_active_replica_added_to_target_before_reduce():
    d = InterReplicaGradientDomain(core_replica_ids=["c0", "c1"])
    d.request_join("h0", "c1")
    d.mark_active("h0")
    out = d.reduce_core_gradients(core_gradients={"c0": (torch.tensor([2.0]),), "c1": (torch.tensor([4.0]),)},
                                  hybrid_payloads=[_payload("h0", "c1", [6.0])])
    assert torch.equal(out["c0"][0], torch.tensor([6.0]))


def test_payload_filters_lane_epoch_step_version():
    d = InterReplicaGradientDomain(core_replica_ids=["c0"], local_replica_rank=1, replica_world_size=2)
    d.request_join("h0", "c0")
    d.mark_active("h0")
    ep = d.membership_epoch("h0")
    ps = [_payload("h0", "c0", [100.0], replica_rank=0, replica_world_size=2, membership_epoch=ep, step=3),
          _payload("h0", "c0", [1.0], replica_rank=1, replica_world_size=2, membership_epoch=ep, step=3),
          _payload("h0", "c0", [1000.0], replica_rank=1, replica_world_size=2, membership_epoch=ep - 1, step=3),
          _payload("h0", "c0", [1000.0], replica_rank=1, replica_world_size=2, membership_epoch=ep, step=2),
          _payload("h0", "c0", [1000.0], replica_rank=1, replica_world_size=2, membership_epoch=ep, step=3,
                   zero_placeholder=True)]
    out = d.accumulate_local_gradients(core_replica_id="c0", core_gradients=(torch.tensor([2.0]),),
                                       hybrid_payloads=ps, step=3)
    assert torch.equal(out[0], torch.tensor([3.0]))
    with pytest.raises(ValueError, match="world size"):
        d.accumulate_local_gradients(core_replica_id="c0", core_gradients=(torch.tensor([2.0]),),
                                     hybrid_payloads=[_payload("h0", "c0", [1.0], replica_world_size=4,
                                                               membership_epoch=ep)])


def test_membership_epochs_and_isolation():
    doms = GradientCommunicationDomains(core_process_group="core", hybrid_process_group="elastic", decoupled=True)
    d = InterReplicaGradientDomain(core_replica_ids=["c0", "c1"], communication_domains=doms)
    d.request_join("h", "c1")
    e1 = d.membership_state()["membership_epoch"]
    d.mark_active("h")
    e2 = d.membership_state()["membership_epoch"]
    d.detach("h")
    st = d.membership_state()
    assert (e1, e2, st["membership_epoch"]) == (1, 2, 3) and st["active_replica_ids"] == ()
    assert doms.core_process_group == "core" and doms.hybrid_process_group == "elastic"
    with pytest.raises(ValueError, match="core process group"):
        d.bind_hybrid_process_group("core")


class _FakeDist:
    @staticmethod
    def is_available():
        return True

    @staticmethod
    def is_initialized():
        return True

    @staticmethod
    def get_world_size(group=None):
        return 1


class _Recorder:
    def __init__(self):
        self.calls = []

    def exchange(self, local, *, group, average):
        self.calls.append((group, average))
        return local.clone()


def test_decoupled_domain_never_reduces_on_core_group(monkeypatch):
    monkeypatch.setattr(hp, "dist", _FakeDist)
    rec = _Recorder()
    d = InterReplicaGradientDomain(core_replica_ids=["c0"], transport=rec, communication_domains=
                                   GradientCommunicationDomains(core_process_group="core", decoupled=True))
    d.request_join("h", "c0")
    d.mark_active("h")
    out = d.reduce_core_gradients(core_gradients={"c0": (torch.tensor([1.0]),)},
                                  hybrid_payloads=[_payload("h", "c0", [2.0])])
    assert torch.equal(out["c0"][0], torch.tensor([3.0])) and rec.calls == []
    assert d.communication_state()["uses_core_group_for_elastic_reduce"] is False
    d2 = InterReplicaGradientDomain(core_replica_ids=["c0"], transport=rec, process_group="core",
                                    decouple_communication_domains=False)
    d2.reduce_core_gradients(core_gradients={"c0": (torch.tensor([1.0]),)})
    assert rec.calls == [("core", True)]
    d3 = InterReplicaGradientDomain(core_replica_ids=["c0"], require_isolated_process_group=True,
                                    communication_domains=GradientCommunicationDomains(core_process_group="core"))
    with pytest.raises(RuntimeError, match="isolated elastic"):
        d3.reduce_core_gradients(core_gradients={"c0": (torch.tensor([1.0]),)})


def test_transports_without_process_group():
    t = torch.arange(10, dtype=torch.float32)
    out = TorchDistributedTransport(chunk_bytes=8).exchange(t, group=None, average=True)
    assert torch.equal(out, t) and out.data_ptr() != t.data_ptr()
    lane = PeerMemoryTransport()
    lane.publish("a", t)
    lane.publish("b", t * 3)
    assert torch.equal(lane.exchange(t, average=True), t * 2)


def test_nonblocking_join_and_activation_barrier():
    release = threading.Event()

    def barrier(worker, target, version):
        assert (worker, target, version) == ("r0", "c0", 11)
        assert release.wait(2.0)

    pool = ElasticHybridPool(core_train_workers=["c0"], core_rollout_workers=["r0"],
                             snapshot_fetcher=lambda *_: (time.sleep(0.05), 11)[1])
    t0 = time.perf_counter()
    h = pool.join_training("r0", "c0", activation_barrier=barrier, timeout_s=5.0)
    assert time.perf_counter() - t0 < 0.05 and not h.done()
    assert pool.snapshot()["r0"].role == ReplicaRole.HYBRID_JOINING
    deadline = time.time() + 2
    while pool.snapshot()["r0"].join_state != JoinState.ACTIVATING and time.time() < deadline:
        time.sleep(0.01)
    assert pool.snapshot()["r0"].join_state == JoinState.ACTIVATING and not h.done()
    release.set()
    w = h.result(2.0)
    assert w.role == ReplicaRole.HYBRID_TRAINING and w.state_version == 11
    assert pool.gradient_domain.active_hybrid_ids() == ("r0",)
    pool.close()


def test_replica_join_is_atomic_and_rolls_back_on_member_failure():
    pool = ElasticHybridPool(core_train_workers=["c0", "c1"], core_rollout_workers=["r0", "r1", "r2", "r3"],
                             snapshot_fetcher=lambda *_: 5)
    h = pool.join_replica("dp0", ["r0", "r1"], "c1")
    assert isinstance(h, ReplicaJoinHandle)
    ws = h.result(2.0)
    assert {w.role for w in ws} == {ReplicaRole.HYBRID_TRAINING} and {w.state_version for w in ws} == {5}

    def bad(worker, _t):
        if worker == "r3":
            raise RuntimeError("snapshot broke")
        return 5

    pool.snapshot_fetcher = bad
    h2 = pool.join_replica("dp1", ["r2", "r3"], "c0")
    with pytest.raises(RuntimeError, match="snapshot broke"):
        h2.result(2.0)
    snap = pool.snapshot()
    assert {snap[w].join_state for w in ("r2", "r3")} == {JoinState.FAILED}
    assert {snap[w].role for w in ("r2", "r3")} == {ReplicaRole.HYBRID_ROLLOUT}
    assert set(pool.replica_snapshot()) == {"dp0"}
    pool.release_replica_to_rollout("dp0")
    pool.snapshot_fetcher = lambda *_: 6
    h3 = pool.join_replica("dp0", ["r0", "r1"], "c1")
    assert h3.generation > h.generation and h3.result(2.0)[0].state_version == 6
    pool.close()


def test_inconsistent_replica_versions_fail():
    pool = ElasticHybridPool(core_train_workers=["c0"], core_rollout_workers=["r0", "r1"],
                             snapshot_fetcher=lambda w, _t: 1 if w == "r0" else 2)
    with pytest.raises(RuntimeError, match="inconsistent"):
        pool.join_replica("dp", ["r0", "r1"], "c0").result(2.0)
    pool.close()


def test_cancel_during_fetch_never_activates():
    release = threading.Event()
    pool = ElasticHybridPool(core_train_workers=["c0"], core_rollout_workers=["r0"],
                             snapshot_fetcher=lambda *_: (release.wait(2.0), 3)[1])
    h = pool.join_training("r0", "c0", timeout_s=5.0)
    h.cancel()
    release.set()
    with pytest.raises(JoinCancelledError):
        h.result(2.0)
    w = pool.snapshot()["r0"]
    assert w.role == ReplicaRole.HYBRID_ROLLOUT and w.join_state == JoinState.CANCELLED
    assert pool.gradient_domain.active_hybrid_ids() == () and pool.replica_snapshot() == {}
    pool.close()


def test_join_timeout_rolls_back():
    pool = ElasticHybridPool(core_train_workers=["c0"], core_rollout_workers=["r0"],
                             snapshot_fetcher=lambda *_: (time.sleep(0.2), 1)[1])
    with pytest.raises(TimeoutError):
        pool.join_training("r0", "c0", timeout_s=0.05).result(2.0)
    assert pool.snapshot()["r0"].join_state == JoinState.FAILED
    pool.close()
