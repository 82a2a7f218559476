"""ZeRO-1 optimizer step fused with the parameter all-gather over NVLink peer memory.

With the distributed optimizer each data-parallel rank owns a contiguous shard
of the flat fp32 master weights and Adam moments; after the step the updated
bf16 shards are all-gathered so every rank holds the full bf16 parameters
(the reference's Megatron distributed optimizer, engine/megatron_core_train_
engine.py:360-380, does the gather with NCCL after the Adam kernel).  Here the
AdamW kernel itself (``adamw_step_allgather`` in ``ops/csrc/elementwise.cu``)
stores each updated bf16 value into the same shard of every rank's parameter
buffer, so the gather overlaps the update and costs no extra pass over memory;
an arrival barrier at the end of the kernel makes the full vector visible
before the next forward.

``PeerParamGather`` maps every rank's flat parameter buffer and a counter area
into this process (CUDA IPC).  ``step`` is collective: every rank of the group
calls it once per optimizer step, in the same order.
"""

from __future__ import annotations

from typing import Optional

import torch
import torch.distributed as dist

from libra_b200 import ops


class PeerParamGather:
    def __init__(self, group, flat_param: torch.Tensor, shard_start: int, shard_numel: int):
        from libra_b200.parallel.peer_gemm import MAX_RANKS

        if flat_param.dtype != torch.bfloat16 or not flat_param.is_cuda or not flat_param.is_contiguous():
            raise ValueError("flat_param must be a contiguous bf16 CUDA tensor")
        if group is None and dist.is_initialized():
            group = dist.group.WORLD  # torch.distributed's meaning of "no group"
        self.group = group
        self.n = dist.get_world_size(group) if group is not None else 1
        self.me = dist.get_rank(group) if group is not None else 0
        if self.n > MAX_RANKS:
            raise ValueError(f"at most {MAX_RANKS} ranks")
        if (shard_start * 2) % 8:
            raise ValueError("shard start must be a multiple of 4 elements")
        self.flags = torch.zeros(64, dtype=torch.int32, device=flat_param.device)
        param_bases, flag_bases = [int(flat_param.data_ptr())], [int(self.flags.data_ptr())]
        self._opened = []
        if self.n > 1:
            C = ops.ext()
            mine = (C.ipc_export(flat_param), C.ipc_export(self.flags))
            handles = [None] * self.n
            dist.all_gather_object(handles, mine, group=self.group)
            param_bases, flag_bases = [], []
            with torch.cuda.device(flat_param.device):
                for r, ((hp, op), (hf, of)) in enumerate(handles):
                    if r == self.me:
                        param_bases.append(int(flat_param.data_ptr()))
                        flag_bases.append(int(self.flags.data_ptr()))
                        continue
                    bp = C.ipc_open(hp)
                    bf = C.ipc_open(hf)
                    self._opened += [bp, bf]
                    param_bases.append(bp + int(op))
                    flag_bases.append(bf + int(of))
        # every rank's flat parameter layout is identical: this rank's shard sits at the same offset
        self.param_peers = [b + 2 * int(shard_start) for b in param_bases]
        self.flag_peers = flag_bases
        self.shard_numel = int(shard_numel)
        self.calls = 0
        # the kernel's arrival target is calls x grid, so all ranks launch the same grid: the smallest
        # "4 CTAs per SM" of the group (ranks may sit on GPUs with different SM counts)
        sms = torch.cuda.get_device_properties(flat_param.device).multi_processor_count
        grid = torch.tensor([sms * 4], dtype=torch.int64, device=flat_param.device)
        if self.n > 1:
            dist.all_reduce(grid, op=dist.ReduceOp.MIN, group=self.group)
        self.grid = int(grid.item())
        if self.n > 1:
            torch.cuda.synchronize(flat_param.device)
            dist.barrier(group=self.group)

    def close(self) -> None:
        for base in self._opened:
            ops.ext().ipc_close(base)
        self._opened = []

    def step(self, master, grad, exp_avg, exp_avg_sq, *, lr, beta1, beta2, eps, weight_decay, step,
             max_grad_norm: float = 0.0, sq_norm: Optional[torch.Tensor] = None, grad_scale: float = 1.0) -> None:
        """AdamW on this rank's shard; afterwards every rank holds the full updated bf16 parameters."""
        if master.numel() != self.shard_numel:
            raise ValueError(f"shard has {self.shard_numel} elements, got {master.numel()}")
        # the epoch advances only once the launch went through, so a rejected call on one rank does not
        # leave its counters a step ahead of its peers'
        ops.ext().adamw_step_allgather(master, grad, exp_avg, exp_avg_sq, lr, beta1, beta2, eps, weight_decay, step,
                                       sq_norm, max_grad_norm, grad_scale, self.param_peers, self.flag_peers,
                                       self.me, self.calls + 1, ops.error_flag(master.device), self.grid)
        self.calls += 1


def _bench(argv=None) -> None:
    """Device time of one distributed-optimizer step: fused AdamW + peer all-gather against AdamW followed
    by NCCL all_gather_into_tensor.

    torchrun --nproc-per-node 2 --master-addr 127.0.0.1 -m libra_b200.parallel.peer_param_gather
    Prints one JSON line (rank 0), max over ranks of the mean per step.
    """
    import argparse
    import datetime
    import json
    import os

    p = argparse.ArgumentParser()
    p.add_argument("--params", type=float, default=1.0e9, help="total parameters over the group")
    p.add_argument("--iters", type=int, default=10)
    a = p.parse_args(argv)
    rank, world = int(os.environ.get("RANK", 0)), int(os.environ.get("WORLD_SIZE", 1))
    torch.cuda.set_device(int(os.environ.get("LOCAL_RANK", 0)))
    dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                            device_id=torch.device("cuda", torch.cuda.current_device()))
    grp = dist.group.WORLD
    shard = int(a.params) // world // 4 * 4
    flat = torch.zeros(world * shard, dtype=torch.bfloat16, device="cuda")
    master = torch.randn(shard, device="cuda")
    grad = torch.randn(shard, device="cuda")
    m, v = torch.zeros_like(master), torch.zeros_like(master)
    sq = grad.pow(2).sum().reshape(1)
    hp = dict(lr=1e-5, beta1=0.9, beta2=0.95, eps=1e-8, weight_decay=0.0, max_grad_norm=1.0, sq_norm=sq)
    pg = PeerParamGather(grp, flat, rank * shard, shard)
    mine = flat[rank * shard:(rank + 1) * shard]
    step = [0]

    def fused():
        step[0] += 1
        pg.step(master, grad, m, v, step=step[0], **hp)

    def nccl():
        step[0] += 1
        ops.adamw_step(master, grad, m, v, mine, step=step[0], **hp)
        dist.all_gather_into_tensor(flat, mine.clone(), group=grp)

    out = {}
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
        out[name + "_ms"] = round(float(ms), 3)
    ops.check_kernel_errors()
    out.update(params=world * shard, ranks=world, shard=shard)
    if rank == 0:
        print(json.dumps(out))
    pg.close()
    dist.barrier()
    dist.destroy_process_group()


if __name__ == "__main__":
    _bench()
