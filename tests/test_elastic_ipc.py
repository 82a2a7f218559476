"""Gradient IPC framing, authentication and lockstep updates (CPU, loopback TCP)."""

import threading

import pytest
import torch

from libra_b200.infra.elastic.gradient_ipc import (ElasticGradientClient, ElasticGradientServer, GradientEndpoint,
                                                   GradientUpdate)
from libra_b200.infra.elastic.hybrid_pool import GradientPayload


def _payload(step=0, epoch=1):
    return GradientPayload("h0", "c0", (torch.randn(3, 5), torch.randn(7).bfloat16(), torch.empty(0)),
                           replica_rank=1, replica_world_size=2, step=step, state_version=4, membership_epoch=epoch)


def test_roundtrip_preserves_tensors_and_metadata():
    got = []
    srv = ElasticGradientServer(authkey="k", on_payload=got.append)
    ep = srv.start()
    try:
        p = _payload()
        assert ElasticGradientClient(ep, timeout=5).send(p) is None
        (q,) = got
        assert (q.replica_id, q.target_core_id, q.replica_rank, q.replica_world_size, q.step, q.state_version,
                q.membership_epoch) == ("h0", "c0", 1, 2, 0, 4, 1)
        for a, b in zip(p.tensors, q.tensors):
            assert a.dtype == b.dtype and torch.equal(a, b)
        assert srv.received_count == 1
    finally:
        srv.close()


def test_wrong_authkey_is_rejected():
    got = []
    srv = ElasticGradientServer(authkey="right", on_payload=got.append)
    ep = srv.start()
    try:
        with pytest.raises(ConnectionError):
            ElasticGradientClient(GradientEndpoint(ep.host, ep.port, "wrong"), timeout=5).send(_payload())
        assert got == [] and srv.rejected_count == 1
    finally:
        srv.close()


def test_lockstep_update_returns_published_reduction():
    srv = ElasticGradientServer(authkey="k", on_payload=lambda p: None, update_timeout=5)
    ep = srv.start()
    out = {}
    try:
        t = threading.Thread(target=lambda: out.setdefault(
            "u", ElasticGradientClient(ep, timeout=10).send(_payload(step=7, epoch=3), expect_update=True)))
        t.start()
        srv.publish_update(GradientUpdate("h0", (torch.ones(4),), 7, 4, 3))
        t.join(10)
        u = out["u"]
        assert (u.replica_id, u.step, u.membership_epoch) == ("h0", 7, 3) and torch.equal(u.tensors[0], torch.ones(4))
    finally:
        srv.close()


def test_lockstep_times_out_without_update():
    srv = ElasticGradientServer(authkey="k", on_payload=lambda p: None, update_timeout=0.3)
    ep = srv.start()
    try:
        with pytest.raises(ConnectionError):
            ElasticGradientClient(ep, timeout=5).send(_payload(), expect_update=True)
    finally:
        srv.close()
