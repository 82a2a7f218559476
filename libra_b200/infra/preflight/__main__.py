"""Operational CLIs.

    nccl        all-gather health check over every GPU of the box (reference
                scripts/nccl_allgather_preflight.py:30-53), spawned with one
                process per GPU, a short process-group timeout, max over ranks.
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
