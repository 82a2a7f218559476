"""Distributed-optimizer gradient reduce-scatter over NVLink peer memory.

The reference's Megatron distributed optimizer reduce-scatters the fp32 main
gradients with NCCL, divides by the data-parallel size and all-reduces the
squared norm for clipping (engine/megatron_core_train_engine.py:209-222 and
531-533).  ``PeerGradReduce`` does all three in one kernel
(``grad_reduce_scatter_peer`` in ``ops/csrc/grad_reduce.cu``): every rank pulls
its own shard of every rank's flat fp32 gradient over NVLink, sums in rank
order, scales by ``1/dp``, writes the fp32 shard and leaves the global sum of
squares in ``sq_norm``.  The kernel ends only after every rank finished reading
this rank's gradient, so the next step may zero it at once.

Every rank of the group maps every rank's gradient buffer and a small counter
area (CUDA IPC, same box).  ``reduce`` is collective: each rank calls it once
per optimizer step, in the same order.
"""

from __future__ import annotations

from typing import List, Optional

import torch
import torch.distributed as dist

from libra_b200 import ops


def agree_grid(group, device, n: int, per_sm: int = 4) -> int:
    """Same CTA count on every rank (counters compare against calls x grid):
    the smallest ``per_sm x SMs`` of the group."""
    sms = torch.cuda.get_device_properties(device).multi_processor_count
    grid = torch.tensor([sms * per_sm], dtype=torch.int64, device=device)
    if n > 1:
        dist.all_reduce(grid, op=dist.ReduceOp.MIN, group=group)
    return int(grid.item())


def map_peer_tensors(group, tensors: List[torch.Tensor], n: int, me: int):
    """Exchange CUDA IPC handles of ``tensors`` over ``group`` and map every
    peer's copies into this process.  Returns (bases, opened): ``bases[i][r]``
    is the address of tensor i of rank r as seen here; ``opened`` lists the
    mappings to close."""
    if n == 1:
        return [[int(t.data_ptr())] for t in tensors], []
    C = ops.ext()
    mine = [C.ipc_export(t) for t in tensors]
    handles = [None] * n
    dist.all_gather_object(handles, mine, group=group)
    bases: List[List[int]] = [[0] * n for _ in tensors]
    opened = []
    with torch.cuda.device(tensors[0].device):
        for r, theirs in enumerate(handles):
            for i, (h, off) in enumerate(theirs):
                if r == me:
                    bases[i][r] = int(tensors[i].data_ptr())
                    continue
                b = C.ipc_open(h)
                opened.append(b)
                bases[i][r] = b + int(off)
    return bases, opened


class PeerGradReduce:
    """Reduce-scatter of one flat fp32 gradient (identical layout on every rank)."""

    def __init__(self, group, flat_grad: torch.Tensor, shard_start: int, shard_numel: int):
        from libra_b200.parallel.peer_gemm import MAX_RANKS

        if flat_grad.dtype != torch.float32 or not flat_grad.is_cuda or not flat_grad.is_contiguous():
            raise ValueError("flat_grad must be a contiguous fp32 CUDA tensor")
        if group is None and dist.is_initialized():
            group = dist.group.WORLD  # torch.distributed's meaning of "no group"
        self.group = group
        self.n = dist.get_world_size(group) if group is not None else 1
        self.me = dist.get_rank(group) if group is not None else 0
        if self.n > MAX_RANKS:
            raise ValueError(f"at most {MAX_RANKS} ranks")
        if shard_start % 4 or shard_numel % 4:
            raise ValueError("shard start and size must be multiples of 4 elements (16-byte peer loads)")
        if shard_start + shard_numel > flat_grad.numel():
            raise ValueError("shard outside the gradient buffer")
        self.flags = torch.zeros(64, dtype=torch.int32, device=flat_grad.device)
        (grad_bases, flag_bases), self._opened = map_peer_tensors(group, [flat_grad, self.flags], self.n, self.me)
        # this rank's shard sits at the same offset in every rank's buffer
        self.src_peers = [b + 4 * int(shard_start) for b in grad_bases]
        self.flag_peers = flag_bases
        self.shard_numel = int(shard_numel)
        self.grid = agree_grid(group, flat_grad.device, self.n)
        self.calls = 0
        if self.n > 1:
            torch.cuda.synchronize(flat_grad.device)
            dist.barrier(group=self.group)

    def close(self) -> None:
        for base in self._opened:
            ops.ext().ipc_close(base)
        self._opened = []

    def reduce(self, out: torch.Tensor, scale: Optional[float] = None, sq_norm: Optional[torch.Tensor] = None) -> None:
        """out[:] = scale * sum over ranks of their gradient's shard ``me``
        (default scale 1/n); ``sq_norm[0]`` = global sum of squares of the result."""
        if out.numel() != self.shard_numel:
            raise ValueError(f"shard has {self.shard_numel} elements, got {out.numel()}")
        s = 1.0 / self.n if scale is None else float(scale)
        ops.ext().grad_reduce_scatter_peer(out, s, sq_norm, self.src_peers, self.flag_peers, self.me, self.calls + 1,
                                           ops.error_flag(out.device), self.grid)
        self.calls += 1  # only after the launch went through, so a rejected call leaves the epochs aligned


def _bench(argv=None) -> None:
    """Bucket sweep: fused peer reduce-scatter (+ scale + global norm) against
    NCCL reduce_scatter_tensor + div_ + squared norm + all_reduce of the norm.

    torchrun --nproc-per-node N --master-addr 127.0.0.1 -m libra_b200.parallel.peer_grad_reduce
    Prints one JSON line per bucket size (rank 0): max over ranks of the mean
    device time per call, bus bandwidth, and the fraction of the NVLink bound
    ((n-1)/n x bucket bytes into each rank at the measured 770 GB/s per direction).
    """
    import argparse
    import datetime
    import json
    import os

    p = argparse.ArgumentParser()
    p.add_argument("--sizes-mb", default="1,4,16,64,256,1024")
    p.add_argument("--iters", type=int, default=20)
    p.add_argument("--link-gbs", type=float, default=770.0)
    a = p.parse_args(argv)
    rank, world = int(os.environ.get("RANK", 0)), int(os.environ.get("WORLD_SIZE", 1))
    torch.cuda.set_device(int(os.environ.get("LOCAL_RANK", 0)))
    dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                            device_id=torch.device("cuda", torch.cuda.current_device()))
    grp = dist.group.WORLD
    for mb in [int(x) for x in a.sizes_mb.split(",")]:
        numel = (mb << 20) // 4 // (4 * world) * (4 * world)
        shard = numel // world
        g = torch.randn(numel, device="cuda")
        out = torch.empty(shard, device="cuda")
        sq = torch.zeros(1, device="cuda")
        red = PeerGradReduce(grp, g, rank * shard, shard)

        def fused():
            red.reduce(out, sq_norm=sq)

        def nccl():
            dist.reduce_scatter_tensor(out, g, op=dist.ReduceOp.SUM, group=grp)
            out.div_(world)
            sq.zero_()
            ops.grad_sq_norm(out, sq)
            dist.all_reduce(sq, group=grp)

        res = {"bucket_mb": mb, "ranks": world}
        fused()
        torch.cuda.synchronize()
        ref = g.view(world, shard)[rank].clone()
        got = out.clone()
        nccl()
        torch.cuda.synchronize()
        res["max_abs_diff"] = float((got - out).abs().max()) if shard else 0.0
        del ref
        for name, fn in (("fused", fused), ("nccl", nccl)):
            for _ in range(3):
                fn()
            dist.barrier()
            torch.cuda.synchronize()
            t0, t1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            t0.record()
            for _ in range(a.iters):
                fn()
            t1.record()
            torch.cuda.synchronize()
            ms = torch.tensor([t0.elapsed_time(t1) / a.iters], device="cuda")
            dist.all_reduce(ms, op=dist.ReduceOp.MAX, group=grp)
            res[name + "_ms"] = round(float(ms), 4)
        nbytes = numel * 4
        bound_ms = (world - 1) / world * nbytes / (a.link_gbs * 1e9) * 1e3
        res["nvlink_bound_ms"] = round(bound_ms, 4)
        res["fused_of_bound"] = round(bound_ms / res["fused_ms"], 3) if world > 1 else None
        res["nccl_of_bound"] = round(bound_ms / res["nccl_ms"], 3) if world > 1 else None
        res["fused_busbw_gbs"] = round((world - 1) / world * nbytes / (res["fused_ms"] / 1e3) / 1e9, 1)
        res["nccl_busbw_gbs"] = round((world - 1) / world * nbytes / (res["nccl_ms"] / 1e3) / 1e9, 1)
        ops.check_kernel_errors()
        if rank == 0:
            print(json.dumps(res), flush=True)
        red.close()
        dist.barrier()
        del g, out
        torch.cuda.empty_cache()
    dist.destroy_process_group()


if __name__ == "__main__":
    _bench()
