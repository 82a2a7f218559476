"""Native peer_xfer service: host shared-memory path on CPU, device path on GPU."""

import os
import subprocess
import sys

import pytest
import torch

from libra_b200.infra.elastic import native_peer as npx
from libra_b200.infra.elastic.hybrid_pool import GradientPayload

pytestmark = pytest.mark.skipif(not npx.available(), reason="libpeer_xfer.so not built")


def test_host_copy_add_and_errors():
    srv = npx.PeerXferServer(token="tok")
    dst = torch.zeros(1024)
    srv.register("grad", dst)
    hb = npx.HostBuffer(1024 * 4)
    try:
        src = hb.tensor(torch.float32)
        src.copy_(torch.arange(1024, dtype=torch.float32))
        npx.push("127.0.0.1", srv.port, "tok", "grad", hb.handle)
        assert torch.equal(dst, torch.arange(1024, dtype=torch.float32))
        npx.push("127.0.0.1", srv.port, "tok", "grad", hb.handle, op=npx.OP_ADD)
        assert torch.equal(dst, 2 * torch.arange(1024, dtype=torch.float32))
        npx.push("127.0.0.1", srv.port, "tok", "grad", hb.handle, nbytes=16, dst_offset=4096 - 16)
        assert dst[-4:].tolist() == [0.0, 1.0, 2.0, 3.0]
        with pytest.raises(npx.PeerXferError) as e:
            npx.push("127.0.0.1", srv.port, "bad", "grad", hb.handle)
        assert e.value.code == 2
        with pytest.raises(npx.PeerXferError) as e:
            npx.push("127.0.0.1", srv.port, "tok", "nope", hb.handle)
        assert e.value.code == 3
        with pytest.raises(npx.PeerXferError) as e:
            npx.push("127.0.0.1", srv.port, "tok", "grad", hb.handle, dst_offset=8)
        assert e.value.code == 4
        assert srv.stats() == {"served": 3, "failed": 3}
    finally:
        hb.close()
        srv.close()
    with pytest.raises(npx.PeerXferError) as e:
        npx.push("127.0.0.1", srv.port, "tok", "grad", hb.handle, timeout_s=1.0)
    assert e.value.code == 1


def test_gradient_lane_accumulates_host_payloads():
    srv = npx.PeerXferServer()
    lane = npx.NativePeerGradientLane(srv)
    core = (torch.ones(8), torch.ones(3, 2))
    lane.register_replica("h0", core)
    try:
        p = GradientPayload("h0", "c0", (torch.full((8,), 2.0), torch.full((3, 2), 3.0)))
        npx.NativePeerGradientLane.send(lane.endpoint, p)
        npx.NativePeerGradientLane.send(lane.endpoint, p)
        npx.NativePeerGradientLane.send(lane.endpoint, GradientPayload.zeros_like(replica_id="h0", target_core_id="c0",
                                                                                  reference=core))
        g = [t.clone() for t in core]
        lane.drain_into("h0", g)
        assert torch.equal(g[0], torch.full((8,), 5.0)) and torch.equal(g[1], torch.full((3, 2), 7.0))
        assert torch.count_nonzero(lane.buffers["h0/0"]) == 0
    finally:
        srv.close()


_CHILD = r"""
import sys, torch
from libra_b200.infra.elastic import native_peer as npx
port, token = int(sys.argv[1]), sys.argv[2]
x = torch.arange(4096, dtype=torch.float32, device="cuda")[1024:]
npx.push("127.0.0.1", port, token, "dst", npx.export_tensor(x), op=npx.OP_ADD, timeout_s=20)
torch.cuda.synchronize()
"""


@pytest.mark.gpu
def test_device_same_process_and_cross_process():
    srv = npx.PeerXferServer(token="t")
    dst = torch.ones(3072, device="cuda")
    srv.register("dst", dst)
    try:
        big = torch.randn(8192, device="cuda")
        src = big[100:100 + 3072]
        npx.push("127.0.0.1", srv.port, "t", "dst", npx.export_tensor(src), op=npx.OP_COPY)
        torch.cuda.synchronize()
        assert torch.equal(dst, src)
        dst.fill_(1.0)
        torch.cuda.synchronize()
        env = dict(os.environ, PYTHONPATH=os.pathsep.join([os.getcwd(), os.environ.get("PYTHONPATH", "")]))
        subprocess.run([sys.executable, "-c", _CHILD, str(srv.port), "t"], check=True, timeout=120, env=env)
        expect = 1.0 + torch.arange(1024, 4096, dtype=torch.float32, device="cuda")
        assert torch.equal(dst, expect)
    finally:
        srv.close()
