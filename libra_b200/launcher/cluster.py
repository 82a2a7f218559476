"""Cluster/box planning and command builders.

Same role as the reference's ``launcher/slurm_utils.py`` (node discovery,
per-node train/rollout GPU split, rollout endpoints and launch commands,
torchrun command, automatic plan).  Defaults are for 8-GPU B200 boxes; the
rollout command starts our own server (``libra_b200.engine.server``) and a
single-node trainer rendezvous on 127.0.0.1.
"""

from __future__ import annotations

import os
import shlex
import socket
import subprocess
import sys
from dataclasses import dataclass, field
from typing import Dict, List, Optional


def is_slurm_env() -> bool:
    return bool(os.environ.get("SLURM_NODELIST") or os.environ.get("SLURM_JOB_NODELIST"))


def get_nodes() -> List[str]:
    """Hosts of the allocation (Slurm) or this host."""
    nodelist = os.environ.get("SLURM_NODELIST") or os.environ.get("SLURM_JOB_NODELIST", "")
    if not nodelist:
        return [socket.gethostname()]
    try:
        out = subprocess.run(["scontrol", "show", "hostnames", nodelist], capture_output=True, text=True, check=True,
                             timeout=30).stdout
        nodes = [n.strip() for n in out.splitlines() if n.strip()]
        return nodes or [socket.gethostname()]
    except (FileNotFoundError, subprocess.SubprocessError):
        return [socket.gethostname()]


def get_slurm_info() -> Dict[str, object]:
    e = os.environ
    return {"job_id": e.get("SLURM_JOB_ID", e.get("SLURM_JOBID", "")), "job_name": e.get("SLURM_JOB_NAME", ""),
            "nodelist": e.get("SLURM_NODELIST", ""), "num_nodes": int(e.get("SLURM_NNODES", "1")),
            "num_tasks": int(e.get("SLURM_NTASKS", "1")), "gpus": e.get("SLURM_GPUS", ""),
            "partition": e.get("SLURM_JOB_PARTITION", "")}


@dataclass
class NodeGPUAllocation:
    node: str
    train_gpu_ids: List[int]
    rollout_gpu_ids: List[int]
    gpus_per_node: int = 8


def compute_gpu_allocation(nodes: List[str], gpus_per_node: int = 8, train_gpus_per_node: int = 4,
                           rollout_gpus_per_node: int = 4) -> List[NodeGPUAllocation]:
    """Training takes the low GPU ids of every node, rollout the next ones."""
    if train_gpus_per_node + rollout_gpus_per_node > gpus_per_node:
        raise ValueError(f"train ({train_gpus_per_node}) + rollout ({rollout_gpus_per_node}) GPUs exceed "
                         f"gpus_per_node ({gpus_per_node})")
    return [NodeGPUAllocation(n, list(range(train_gpus_per_node)),
                              list(range(train_gpus_per_node, train_gpus_per_node + rollout_gpus_per_node)),
                              gpus_per_node) for n in nodes]


def _instances(alloc: NodeGPUAllocation, tp_list: List[int]):
    gpus, out = list(alloc.rollout_gpu_ids), []
    for tp in tp_list:
        if len(gpus) < tp:
            break
        out.append((gpus[:tp], tp))
        gpus = gpus[tp:]
    return out


def build_rollout_endpoints(allocations: List[NodeGPUAllocation], tp_size: int = 1, base_port: int = 8000,
                            tp_list: Optional[List[int]] = None) -> List[str]:
    eps, port = [], base_port
    for a in allocations:
        for _ in _instances(a, tp_list or [tp_size] * (len(a.rollout_gpu_ids) // max(tp_size, 1))):
            eps.append(f"{a.node}:{port}")
            port += 1
    return eps


def build_rollout_launch_commands(allocations: List[NodeGPUAllocation], model: str = "qwen3-4b",
                                  checkpoint: str = "", tp_size: int = 1, base_port: int = 8000,
                                  kv_memory_fraction: float = 0.85, tp_list: Optional[List[int]] = None,
                                  extra_args: str = "", python: str = "") -> List[Dict[str, object]]:
    py = shlex.quote(python or sys.executable)
    cmds, port = [], base_port
    for a in allocations:
        for gpus, tp in _instances(a, tp_list or [tp_size] * (len(a.rollout_gpu_ids) // max(tp_size, 1))):
            dev = ",".join(map(str, gpus))
            launch = f"{py} -m torch.distributed.run --standalone --nproc-per-node {tp} -m" if tp > 1 else f"{py} -m"
            cmd = (f"CUDA_VISIBLE_DEVICES={dev} {launch} libra_b200.engine.server --model {shlex.quote(model)} "
                   + (f"--checkpoint {shlex.quote(checkpoint)} " if checkpoint else "")
                   + f"--host 0.0.0.0 --port {port} --tp {tp} --kv-memory-fraction {kv_memory_fraction}")
            if extra_args:
                cmd += " " + extra_args
            cmds.append({"node": a.node, "port": port, "gpu_ids": gpus, "gpu_ids_str": dev, "tp": tp, "command": cmd})
            port += 1
    return cmds


def build_torchrun_command(allocations: List[NodeGPUAllocation], train_script: str, master_addr: str = "",
                           master_port: int = 29500, extra_args: str = "", python: str = "") -> Dict[str, object]:
    n = len(allocations)
    nproc = len(allocations[0].train_gpu_ids) if allocations else 1
    if not master_addr:
        master_addr = "127.0.0.1" if n <= 1 else allocations[0].node
    dev = ",".join(map(str, allocations[0].train_gpu_ids)) if allocations else "0"
    py = shlex.quote(python or sys.executable)
    rdzv = (f"--standalone --local-addr 127.0.0.1" if n <= 1 else
            f"--nnodes={n} --rdzv-backend=c10d --rdzv-endpoint={master_addr}:{master_port}")
    cmd = f"CUDA_VISIBLE_DEVICES={dev} {py} -m torch.distributed.run {rdzv} --nproc-per-node={nproc} {train_script}"
    if extra_args:
        cmd += " " + extra_args
    return {"num_nodes": n, "nproc_per_node": nproc, "master_addr": master_addr, "master_port": master_port,
            "train_gpu_ids_str": dev, "command": cmd}


def auto_plan_cluster(train_gpus: int, rollout_gpus: int, tp_size: int = 1, base_port: int = 8000,
                      gpus_per_node: int = 8, nodes: Optional[List[str]] = None,
                      tp_list: Optional[List[int]] = None) -> Dict[str, object]:
    nodes = nodes or get_nodes()
    n = len(nodes)
    if train_gpus % n or rollout_gpus % n:
        raise ValueError(f"train ({train_gpus}) and rollout ({rollout_gpus}) GPUs must split evenly over {n} nodes")
    allocs = compute_gpu_allocation(nodes, gpus_per_node, train_gpus // n, rollout_gpus // n)
    eps = build_rollout_endpoints(allocs, tp_size, base_port, tp_list)
    return {"nodes": nodes, "num_nodes": n, "allocations": allocs, "endpoints": eps, "endpoints_str": ",".join(eps),
            "is_slurm": is_slurm_env(), "train_gpus": train_gpus, "rollout_gpus": rollout_gpus}


def print_cluster_plan(plan: Dict[str, object]) -> None:
    print(f"nodes={plan['num_nodes']} slurm={plan['is_slurm']} train_gpus={plan['train_gpus']} "
          f"rollout_gpus={plan['rollout_gpus']}")
    for a in plan["allocations"]:
        print(f"  {a.node}: train={a.train_gpu_ids} rollout={a.rollout_gpu_ids}")
    print(f"  endpoints: {plan['endpoints_str']}")
