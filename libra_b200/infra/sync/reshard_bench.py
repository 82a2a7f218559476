"""Trainer -> rollout weight-sync microbenchmark (one box, one process per GPU).

    python -m torch.distributed.run --nproc-per-node 8 --master-addr 127.0.0.1 \\
        -m libra_b200.infra.sync.reshard_bench --model qwen3-14b --src-tp 4 --dst-tp 1 2 4 8

The trainer's TP shards (random weights, bf16) live on ranks 0..src_tp-1; a
rollout bucket of TP degree m lives on the last m ranks.  Two ways to refresh
the bucket are timed, each as the max over ranks of CUDA-event time after a
barrier:

* ``peer``: every bucket rank maps the trainer shards (CUDA IPC) and runs the
  ``weight_reshard`` kernel: its slice is read straight from the owning
  trainer GPUs over NVLink and written into its flat weight buffer;
* ``nccl``: the reference's path (infra/sync/nccl_weight_sync.py:126-197 after
  Megatron Bridge's export): the TP shards are all-gathered, trainer rank 0
  assembles full tensors and broadcasts them in 256 MB chunks to the bucket,
  which copies out its slice.

Rank 0 prints one JSON line per bucket degree: ms, bytes each bucket rank
receives, GB/s per receiving GPU, and the NVLink bound for the peer path
(bytes that must cross into the busiest receiving GPU at the measured 770 GB/s
per direction).
"""

from __future__ import annotations

import argparse
import datetime
import json
import os

import torch
import torch.distributed as dist

from libra_b200.infra.sync.reshard import (DeviceReshard, apply_plan, build_plan, export_buffer, open_buffer,
                                           plan_bytes)
from libra_b200.models.qwen3 import ParamLayout, get_config, param_shapes

NVLINK_GBS = 770.0  # measured peer copy, GB/s per direction per GPU


def _fill(flat: torch.Tensor, seed: int) -> None:
    g = torch.Generator(device=flat.device).manual_seed(seed)
    flat.normal_(0.0, 0.02, generator=g)


def _time(fn, dev, iters: int) -> float:
    fn()
    torch.cuda.synchronize(dev)
    dist.barrier()
    t0, t1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    t0.record()
    for _ in range(iters):
        fn()
    t1.record()
    torch.cuda.synchronize(dev)
    ms = torch.tensor([t0.elapsed_time(t1) / iters], device=dev)
    dist.all_reduce(ms, op=dist.ReduceOp.MAX)
    return float(ms)


def main(argv=None) -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--model", default="qwen3-14b")
    ap.add_argument("--src-tp", type=int, default=4)
    ap.add_argument("--dst-tp", type=int, nargs="+", default=[1, 2, 4, 8])
    ap.add_argument("--iters", type=int, default=3)
    ap.add_argument("--chunk-mb", type=int, default=256)
    ap.add_argument("--skip-nccl", action="store_true")
    a = ap.parse_args(argv)
    rank, world = int(os.environ.get("RANK", 0)), int(os.environ.get("WORLD_SIZE", 1))
    local = int(os.environ.get("LOCAL_RANK", 0))
    dev = torch.device("cuda", local)
    torch.cuda.set_device(dev)
    dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300), device_id=dev)
    cfg = get_config(a.model)
    k = a.src_tp
    if k > world:
        raise SystemExit(f"--src-tp {k} needs at least {k} ranks")
    src_flat = None
    if rank < k:
        src_flat = torch.empty(ParamLayout(param_shapes(cfg, k, rank)).numel, dtype=torch.bfloat16, device=dev)
        _fill(src_flat, 1000 + rank)
    descs = [None] * world
    dist.all_gather_object(descs, export_buffer(src_flat) if src_flat is not None else None)
    sources = descs[:k]
    trainer_group = dist.new_group(list(range(k)))
    for m in a.dst_tp:
        if m > world:
            continue
        dst_ranks = list(range(world - m, world))
        me = rank - (world - m) if rank in dst_ranks else -1
        dst_flat, plan = None, None
        if me >= 0:
            dst_flat = torch.empty(ParamLayout(param_shapes(cfg, m, me)).numel, dtype=torch.bfloat16, device=dev)
            addrs = [int(src_flat.data_ptr()) if (r == rank and src_flat is not None) else open_buffer(d, dev)
                     for r, d in enumerate(sources)]
            plan = DeviceReshard(cfg, k, m, me, addrs, dst_flat)
        slice_bytes = plan.bytes if plan is not None else 0
        # bytes each receiving GPU must pull over NVLink (its own trainer shard, if any, is local)
        remote = 0
        if plan is not None:
            remote = sum(r.rows * r.row_elems * 2 for r in plan.rects if r.src != rank)
        peer_ms = _time(lambda: plan.run() if plan is not None else None, dev, a.iters)
        # correctness: the bucket slice equals slicing the full model assembled on the host side of the plan
        if plan is not None and m <= 2:
            srcs = [torch.empty(ParamLayout(param_shapes(cfg, k, r)).numel, dtype=torch.bfloat16, device=dev)
                    for r in range(k)]
            for r, t in enumerate(srcs):
                _fill(t, 1000 + r)
            want = torch.empty_like(dst_flat)
            apply_plan(plan.rects, srcs, want)
            ok = bool(torch.equal(want, dst_flat))
            del srcs, want
        else:
            ok = None
        nccl_ms = None
        if not a.skip_nccl:
            bucket = dist.new_group(sorted(set([0] + dst_ranks)))
            full = torch.empty(ParamLayout(param_shapes(cfg, 1, 0)).numel, dtype=torch.bfloat16, device=dev) \
                if (rank == 0 or me >= 0) else None
            gathered = [torch.empty_like(src_flat) for _ in range(k)] if rank < k else None
            rects_full = build_plan(cfg, k, 1, 0) if rank == 0 else None
            rects_dst = build_plan(cfg, 1, m, me) if me >= 0 else None
            chunk = a.chunk_mb * (1 << 20) // 2

            def nccl():
                if rank < k:
                    dist.all_gather(gathered, src_flat, group=trainer_group)
                if rank == 0:
                    apply_plan(rects_full, gathered, full)
                if full is not None:
                    for s in range(0, full.numel(), chunk):
                        dist.broadcast(full[s:s + chunk], src=0, group=bucket)
                if me >= 0:
                    apply_plan(rects_dst, [full], dst_flat)

            nccl_ms = _time(nccl, dev, a.iters)
            del full, gathered
        busiest = torch.tensor([float(remote)], device=dev)
        dist.all_reduce(busiest, op=dist.ReduceOp.MAX)
        per_gpu = torch.tensor([float(slice_bytes)], device=dev)
        dist.all_reduce(per_gpu, op=dist.ReduceOp.MAX)
        oks = [None] * world
        dist.all_gather_object(oks, ok)
        bound_ms = float(busiest) / (NVLINK_GBS * 1e9) * 1e3
        if rank == 0:
            print(json.dumps({
                "metric": "weight sync", "model": a.model, "src_tp": k, "dst_tp": m, "ranks": world,
                "bytes_per_bucket_rank": int(per_gpu), "peer_ms": round(peer_ms, 3),
                "peer_gb_per_s_per_gpu": round(float(per_gpu) / (peer_ms / 1e3) / 1e9, 1),
                "nvlink_bound_ms": round(bound_ms, 3), "peer_fraction_of_bound": round(bound_ms / peer_ms, 3),
                "nccl_ms": None if nccl_ms is None else round(nccl_ms, 3),
                "speedup_vs_nccl": None if nccl_ms is None else round(nccl_ms / peer_ms, 2),
                "bit_exact": [o for o in oks if o is not None]}), flush=True)
        del dst_flat, plan
        torch.cuda.empty_cache()
        dist.barrier()
    dist.barrier()
    dist.destroy_process_group()


if __name__ == "__main__":
    main()
