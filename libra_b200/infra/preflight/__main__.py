"""Operational CLIs.

    nccl        all-gather health check over every GPU of the box (reference
                scripts/nccl_allgather_preflight.py:30-53), spawned with one
                process per GPU, a short process-group timeout, max over ranks.
    nvlink      device-timed peer copy bandwidth of every ordered GPU pair
                (one process; flags pairs below a fraction of the expected
                per-direction NVLink bandwidth).
    grp         startup Global Resource Planner preflight from a config
                (reference scripts/run_global_resource_preflight.py).
    placement   initial rollout/train placement of a config, printed as JSON
                (reference scripts/plan_initial_grp_placement.py).
    validate-ehp  check the Elastic Hybrid Pool settings of a config
                (reference scripts/validate_ehp_ab_config.py).
    merge-trees merge C-MLFQ prefix-tree JSON files (reference
                scripts/merge_cmlfq_prefix_trees.py).
    scan        list this box's GPUs and their settings (read only; reference
                scripts/scan_cluster_nodes.py).
"""

from __future__ import annotations

import argparse
import json
import os
import subprocess
import sys
import time


def _nccl_worker(rank: int, world: int, port: int, numel: int, iters: int, out: str) -> None:
    import datetime

    import torch
    import torch.distributed as dist

    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=60))
    x = torch.full((numel,), float(rank), device="cuda", dtype=torch.bfloat16)
    y = torch.empty(numel * world, device="cuda", dtype=torch.bfloat16)
    dist.all_gather_into_tensor(y, x)
    torch.cuda.synchronize()
    ok = all(float(y[r * numel]) == float(r) for r in range(world))
    s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    s.record()
    for _ in range(iters):
        dist.all_gather_into_tensor(y, x)
    e.record()
    torch.cuda.synchronize()
    ms = torch.tensor([s.elapsed_time(e) / iters], device="cuda")
    dist.all_reduce(ms, op=dist.ReduceOp.MAX)
    okt = torch.tensor([1 if ok else 0], device="cuda")
    dist.all_reduce(okt, op=dist.ReduceOp.MIN)
    if rank == 0:
        bytes_ = numel * 2 * world * (world - 1) / world
        with open(out, "w") as f:
            json.dump({"ok": bool(okt.item()), "world": world, "numel": numel, "ms": ms.item(),
                       "bus_gbs": bytes_ / (ms.item() / 1e3) / 1e9}, f)
    dist.destroy_process_group()


def cmd_nccl(a) -> int:
    import tempfile

    import torch
    import torch.multiprocessing as mp

    world = a.gpus or torch.cuda.device_count()
    if world < 1:
        print(json.dumps({"ok": False, "error": "no CUDA device"}))
        return 1
    out = tempfile.mktemp(suffix=".json")
    mp.start_processes(_nccl_worker, args=(world, a.port, a.numel, a.iters, out), nprocs=world, join=True,
                       start_method="spawn")
    res = json.load(open(out))
    print(json.dumps(res))
    return 0 if res["ok"] else 1


def classify_links(pairs: list, expect_gbs: float, min_fraction: float) -> dict:
    """Judge measured peer-copy bandwidths: a pair is slow below
    ``min_fraction * expect_gbs``.  ``pairs`` holds dicts with src, dst, gbs."""
    floor = expect_gbs * min_fraction
    slow = [p for p in pairs if p["gbs"] < floor]
    vals = [p["gbs"] for p in pairs]
    return {"ok": bool(pairs) and not slow, "pairs": len(pairs), "min_gbs": min(vals) if vals else 0.0,
            "max_gbs": max(vals) if vals else 0.0, "median_gbs": sorted(vals)[len(vals) // 2] if vals else 0.0,
            "floor_gbs": floor, "slow": slow}


def measure_peer_copy(src_dev: int, dst_dev: int, nbytes: int, iters: int, bidirectional: bool = False) -> float:
    """Device-timed copy from GPU ``src_dev`` into GPU ``dst_dev`` over NVLink
    (peer access enabled by the runtime copy engine path), GB/s per direction.
    Bidirectional: both directions run at once on two streams, and the figure
    is per direction.  Timed with CUDA events on the copying streams after one
    warm-up copy, and the slower direction is reported."""
    import torch

    n = nbytes // 2
    a = torch.empty(n, dtype=torch.bfloat16, device=f"cuda:{src_dev}").fill_(1.0)
    b = torch.empty(n, dtype=torch.bfloat16, device=f"cuda:{dst_dev}")
    jobs = [(a, b, src_dev)]
    if bidirectional:
        a2 = torch.empty(n, dtype=torch.bfloat16, device=f"cuda:{dst_dev}").fill_(2.0)
        b2 = torch.empty(n, dtype=torch.bfloat16, device=f"cuda:{src_dev}")
        jobs.append((a2, b2, dst_dev))
    streams = [torch.cuda.Stream(device=d) for _, _, d in jobs]
    for (x, y, d), s in zip(jobs, streams):
        with torch.cuda.stream(s):
            y.copy_(x, non_blocking=True)
    for d in {src_dev, dst_dev}:
        torch.cuda.synchronize(d)
    evs = []
    for (x, y, d), s in zip(jobs, streams):
        with torch.cuda.device(d), torch.cuda.stream(s):
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record(s)
            for _ in range(iters):
                y.copy_(x, non_blocking=True)
            e1.record(s)
            evs.append((e0, e1))
    for d in {src_dev, dst_dev}:
        torch.cuda.synchronize(d)
    ms = max(e0.elapsed_time(e1) for e0, e1 in evs) / iters
    ok = bool((b[:: max(1, n // 64)] == 1.0).all())
    if not ok:
        raise RuntimeError(f"peer copy {src_dev}->{dst_dev} delivered wrong data")
    return n * 2 / (ms / 1e3) / 1e9


def cmd_nvlink(a) -> int:
    """Peer copy bandwidth between every ordered GPU pair of the box (the B200
    replacement of the all-gather health check: on one NVSwitch box every
    pair should see the same bandwidth, so one slow pair marks a bad link)."""
    import torch

    world = a.gpus or torch.cuda.device_count()
    if world < 2:
        print(json.dumps({"ok": False, "error": f"needs two or more CUDA devices, found {world}"}))
        return 1
    pairs = []
    for s in range(world):
        for d in range(world):
            if s == d or (a.first_only and s != 0):
                continue
            if not torch.cuda.can_device_access_peer(s, d):
                pairs.append({"src": s, "dst": d, "gbs": 0.0, "error": "no peer access"})
                continue
            gbs = measure_peer_copy(s, d, a.mbytes << 20, a.iters, bidirectional=a.bidirectional)
            pairs.append({"src": s, "dst": d, "gbs": round(gbs, 1)})
    res = classify_links(pairs, a.expect_gbs, a.min_fraction)
    res.update({"world": world, "bytes": a.mbytes << 20, "bidirectional": a.bidirectional, "results": pairs})
    print(json.dumps(res))
    return 0 if res["ok"] else 1


def cmd_grp(a) -> int:
    from libra_b200.config import AsyncRLConfig
    from libra_b200.infra.cost_model.preflight_planner import PreflightPlanner

    from libra_b200.infra.cost_model.preflight_planner import synthetic_history
    from libra_b200.infra.cost_model.startup_profile import load_length_profile_records

    cfg = AsyncRLConfig.from_file(a.config)
    hist = load_length_profile_records(a.profile) if a.profile else synthetic_history(num_requests=a.requests)
    res = PreflightPlanner(cfg).run(hist)
    print(json.dumps(res.to_dict(), default=str, indent=1))
    return 0


def cmd_placement(a) -> int:
    from libra_b200.config import AsyncRLConfig
    from libra_b200.infra.cost_model.global_resource_planner import GlobalResourcePlanner
    from libra_b200.infra.cost_model.preflight_planner import synthetic_history

    cfg = AsyncRLConfig.from_file(a.config)
    grp = GlobalResourcePlanner.from_config(cfg)
    d = grp.plan_if_needed(max(grp.warmup_steps, 0) + grp.plan_interval, cfg,
                           batch=synthetic_history(num_requests=a.requests))
    plan = d.candidate_plan or d.current_plan
    if plan is not None and a.apply:
        grp.apply_plan_to_config(plan, cfg)
    print(json.dumps({"decision": d.to_dict(), "instances": [vars(i) for i in cfg.heterogeneous_rollout.instances]},
                     default=str, indent=1))
    return 0


def validate_ehp(cfg) -> list:
    g = cfg.global_resource_planner
    problems = []
    width = max(1, cfg.train_tp_size) * max(1, cfg.train_pp_size) * max(1, getattr(cfg, "train_cp_size", 1))
    if g.elastic_hybrid_replica_size_gpus and g.elastic_hybrid_replica_size_gpus != width:
        problems.append(f"elastic_hybrid_replica_size_gpus={g.elastic_hybrid_replica_size_gpus} must equal one DP "
                        f"replica ({width} GPUs)")
    if g.runtime_reconfigure_training and not g.runtime_training_pool_only:
        problems.append("runtime_reconfigure_training needs runtime_training_pool_only (fixed core topology)")
    if g.elastic_hybrid_max_workers and g.elastic_hybrid_max_workers * width > cfg.rollout_gpus:
        problems.append("elastic_hybrid_max_workers x replica width exceeds rollout_gpus")
    if g.elastic_hybrid_borrow_train_rollout_ratio <= g.elastic_hybrid_release_train_rollout_ratio:
        problems.append("borrow ratio must exceed release ratio (hysteresis)")
    if g.hybrid_worker_launch_enabled and not g.runtime_reconfigure_training:
        problems.append("hybrid_worker_launch_enabled without runtime_reconfigure_training never launches workers")
    return problems


def cmd_validate_ehp(a) -> int:
    from libra_b200.config import AsyncRLConfig

    probs = validate_ehp(AsyncRLConfig.from_file(a.config))
    print(json.dumps({"ok": not probs, "problems": probs}, indent=1))
    return 0 if not probs else 1


def cmd_merge_trees(a) -> int:
    from libra_b200.infra.scheduling.cmlfq_prefix_tree import CausalPrefixTree

    merged = CausalPrefixTree()
    for path in a.inputs:
        t = CausalPrefixTree()
        t.load(path)
        merged.merge(t)
    merged.save(a.output)
    print(json.dumps({"inputs": len(a.inputs), "output": a.output}))
    return 0


def cmd_scan(a) -> int:
    q = "index,name,memory.total,clocks.max.sm,clocks.sm,power.limit,persistence_mode,mig.mode.current"
    try:
        out = subprocess.run(["nvidia-smi", f"--query-gpu={q}", "--format=csv,noheader"], capture_output=True,
                             text=True, timeout=30).stdout
    except (FileNotFoundError, subprocess.SubprocessError) as exc:
        print(json.dumps({"error": str(exc)}))
        return 1
    rows = [dict(zip(q.split(","), [x.strip() for x in line.split(",")])) for line in out.splitlines() if line.strip()]
    print(json.dumps({"host": os.uname().nodename, "gpus": rows}, indent=1))
    return 0


def main(argv=None) -> int:
    ap = argparse.ArgumentParser(prog="python -m libra_b200.infra.preflight")
    sub = ap.add_subparsers(dest="cmd", required=True)
    p = sub.add_parser("nccl")
    p.add_argument("--gpus", type=int, default=0)
    p.add_argument("--numel", type=int, default=16 * 1024 * 1024)
    p.add_argument("--iters", type=int, default=10)
    p.add_argument("--port", type=int, default=29531)
    p.set_defaults(fn=cmd_nccl)
    p = sub.add_parser("nvlink")
    p.add_argument("--gpus", type=int, default=0)
    p.add_argument("--mbytes", type=int, default=256, help="copy size per pair, MiB")
    p.add_argument("--iters", type=int, default=10)
    p.add_argument("--bidirectional", action="store_true")
    p.add_argument("--first-only", action="store_true", help="only pairs from GPU 0")
    p.add_argument("--expect-gbs", type=float, default=770.0, help="expected per-direction peer copy GB/s")
    p.add_argument("--min-fraction", type=float, default=0.6)
    p.set_defaults(fn=cmd_nvlink)
    p = sub.add_parser("grp")
    p.add_argument("--config", required=True)
    p.add_argument("--profile", default="", help="length-profile JSONL (else a synthetic history)")
    p.add_argument("--requests", type=int, default=64)
    p.set_defaults(fn=cmd_grp)
    p = sub.add_parser("validate-ehp")
    p.add_argument("--config", required=True)
    p.set_defaults(fn=cmd_validate_ehp)
    p = sub.add_parser("placement")
    p.add_argument("--config", required=True)
    p.add_argument("--requests", type=int, default=64)
    p.add_argument("--apply", action="store_true")
    p.set_defaults(fn=cmd_placement)
    p = sub.add_parser("merge-trees")
    p.add_argument("inputs", nargs="+")
    p.add_argument("--output", required=True)
    p.set_defaults(fn=cmd_merge_trees)
    p = sub.add_parser("scan")
    p.set_defaults(fn=cmd_scan)
    a = ap.parse_args(argv)
    return a.fn(a)


if __name__ == "__main__":
    sys.exit(main())
