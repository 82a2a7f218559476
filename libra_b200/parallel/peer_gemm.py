"""Tensor-parallel GEMM fused with its all-reduce over NVLink peer memory.

The row-parallel linear of Megatron-style tensor parallelism (attention output
projection, MLP down projection) computes a partial ``a_r w_r^T`` on every
rank and all-reduces it; the reference reaches this through Megatron-Core's
``RowParallelLinear`` (NCCL all-reduce after cuBLAS, engine/megatron_core_
train_engine.py:887-903).  Here one kernel (``gemm_allreduce`` in
``ops/csrc/gemm_tcgen05.cu``) does both: the CTA-pair GEMM's epilogue stores
each 256-row block of the partial locally and signals the rank that owns the
block, the owner pulls the partials over NVLink, sums them in fp32 and writes
the sum to every rank, and each rank copies the finished blocks (plus the
residual) into its output.  Each byte crosses NVLink once per direction, as in a reduce-scatter +
all-gather, and the transfers overlap the GEMM tiles still running.

``PeerGemmAllReduce`` owns one symmetric buffer per (group, N): partial
``[max_rows, N]``, gathered sum ``[max_rows, N]`` and the arrival counters,
shared through CUDA IPC handles and opened in this device's context.  Calls
must be made in the same order on every rank of the group.
"""

from __future__ import annotations

from typing import Dict, Optional, Tuple

import torch
import torch.distributed as dist

from libra_b200 import ops

MAX_RANKS = 8
ROW_BLOCK = 256


class PeerGemmAllReduce:
    def __init__(self, group, max_rows: int, n_cols: int, device):
        self.group = group
        self.n = dist.get_world_size(group) if dist.is_initialized() else 1
        self.me = dist.get_rank(group) if dist.is_initialized() else 0
        if self.n > MAX_RANKS:
            raise ValueError(f"at most {MAX_RANKS} ranks")
        if n_cols % 8:
            raise ValueError("N must be a multiple of 8")
        self.max_rows, self.n_cols = int(max_rows), int(n_cols)
        slot = self.max_rows * self.n_cols * 2
        self.recv_bytes = (slot + 255) // 256 * 256
        self.gath_bytes = (slot + 255) // 256 * 256
        max_rb = (self.max_rows + ROW_BLOCK - 1) // ROW_BLOCK
        flag_bytes = (4 * max_rb * 4 + 255) // 256 * 256
        self.buf = torch.zeros(self.recv_bytes + self.gath_bytes + flag_bytes, dtype=torch.uint8, device=device)
        bases = [int(self.buf.data_ptr())]
        self._opened = []
        if self.n > 1:
            C = ops.ext()
            handles = [None] * self.n
            dist.all_gather_object(handles, C.ipc_export(self.buf), group=self.group)
            bases = []
            with torch.cuda.device(self.buf.device):
                for r, (h, off) in enumerate(handles):
                    if r == self.me:
                        bases.append(int(self.buf.data_ptr()))
                    else:
                        base = C.ipc_open(h)
                        self._opened.append(base)
                        bases.append(base + int(off))
        self.recv = bases
        self.gath = [b + self.recv_bytes for b in bases]
        self.flags = [b + self.recv_bytes + self.gath_bytes for b in bases]
        self.calls = 0
        if self.n > 1:
            torch.cuda.synchronize(self.buf.device)
            dist.barrier(group=self.group)

    def close(self) -> None:
        for base in self._opened:
            ops.ext().ipc_close(base)
        self._opened = []

    def __call__(self, a: torch.Tensor, w: torch.Tensor, residual: Optional[torch.Tensor] = None,
                 b_mn: bool = False) -> torch.Tensor:
        """sum over ranks of a_r @ w_r^T (w_r: [N, K], or [K, N] with ``b_mn``) + residual."""
        a2 = a.reshape(-1, a.shape[-1])
        if not a2.is_contiguous():
            a2 = a2.contiguous()
        N = w.shape[1] if b_mn else w.shape[0]
        if N != self.n_cols or a2.shape[0] > self.max_rows:
            raise ValueError(f"buffer is for N={self.n_cols}, up to {self.max_rows} rows; got N={N}, "
                             f"{a2.shape[0]} rows")
        y = torch.empty(a2.shape[0], N, dtype=a.dtype, device=a.device)
        res = residual.reshape(-1, N).contiguous() if residual is not None else None
        ops.ext().gemm_allreduce(a2, w, bool(b_mn), res, y, self.recv, self.gath, self.flags, self.me,
                                 self.calls & 1, self.max_rows, 0, ops.error_flag(a.device))
        self.calls += 1
        return y.view(*a.shape[:-1], N)

    def reduce_scatter(self, a: torch.Tensor, w: torch.Tensor, residual: Optional[torch.Tensor] = None,
                       b_mn: bool = False) -> torch.Tensor:
        """This rank's row shard of sum over ranks of a_r @ w_r^T (+ residual shard):
        rows [me * M/n, (me+1) * M/n).  M must be a multiple of 256 * n."""
        a2 = a.reshape(-1, a.shape[-1]).contiguous()
        M = a2.shape[0]
        N = w.shape[1] if b_mn else w.shape[0]
        if N != self.n_cols or M > self.max_rows or M % (ROW_BLOCK * self.n):
            raise ValueError(f"reduce-scatter needs N={self.n_cols}, M <= {self.max_rows} and M a multiple of "
                             f"{ROW_BLOCK * self.n}; got N={N}, M={M}")
        y = torch.empty(M // self.n, N, dtype=a.dtype, device=a.device)
        res = residual.reshape(-1, N).contiguous() if residual is not None else None
        ops.ext().gemm_allreduce(a2, w, bool(b_mn), res, y, self.recv, self.gath, self.flags, self.me,
                                 self.calls & 1, self.max_rows, M // self.n, ops.error_flag(a.device))
        self.calls += 1
        return y


class PeerAllGatherGemm:
    """y = [a_0; a_1; ...; a_{n-1}] @ w^T for row shards a_q of the group
    (sequence-parallel column-parallel linear, K1) in one kernel: peers' shards
    are copied over NVLink into a local buffer by the GEMM's epilogue warps while
    its first tiles (the local shard's rows) run.  Shards go through two
    alternating symmetric slots per rank; calls in the same order on every rank."""

    def __init__(self, group, shard_rows: int, k_cols: int, device):
        self.group = group
        self.n = dist.get_world_size(group) if dist.is_initialized() else 1
        self.me = dist.get_rank(group) if dist.is_initialized() else 0
        if self.n > MAX_RANKS or shard_rows % ROW_BLOCK or k_cols % 8:
            raise ValueError("at most 8 ranks, shard rows a multiple of 256, K a multiple of 8")
        self.shard_rows, self.k_cols = int(shard_rows), int(k_cols)
        self.slot_bytes = (self.shard_rows * self.k_cols * 2 + 255) // 256 * 256
        self.buf = torch.zeros(2 * self.slot_bytes + 256, dtype=torch.uint8, device=device)
        bases = [int(self.buf.data_ptr())]
        self._opened = []
        if self.n > 1:
            C = ops.ext()
            handles = [None] * self.n
            dist.all_gather_object(handles, C.ipc_export(self.buf), group=self.group)
            bases = []
            with torch.cuda.device(self.buf.device):
                for r, (h, off) in enumerate(handles):
                    if r == self.me:
                        bases.append(int(self.buf.data_ptr()))
                    else:
                        base = C.ipc_open(h)
                        self._opened.append(base)
                        bases.append(base + int(off))
        self.slots = [(b, b + self.slot_bytes) for b in bases]
        self.ready = [b + 2 * self.slot_bytes for b in bases]
        self.gath = torch.empty(self.n * self.shard_rows, self.k_cols, dtype=torch.bfloat16, device=device)
        self.counter = torch.zeros(1, dtype=torch.int32, device=device)
        self.calls = 0
        if self.n > 1:
            torch.cuda.synchronize(self.buf.device)
            dist.barrier(group=self.group)

    def close(self) -> None:
        for base in self._opened:
            ops.ext().ipc_close(base)
        self._opened = []

    def __call__(self, a: torch.Tensor, w: torch.Tensor, b_mn: bool = False) -> torch.Tensor:
        if a.shape != (self.shard_rows, self.k_cols):
            raise ValueError(f"shard must be [{self.shard_rows}, {self.k_cols}], got {tuple(a.shape)}")
        self.calls += 1
        p = self.calls & 1
        slot = self.buf[p * self.slot_bytes:p * self.slot_bytes + self.shard_rows * self.k_cols * 2]
        slot.view(torch.bfloat16).view(self.shard_rows, self.k_cols).copy_(a)
        N = w.shape[1] if b_mn else w.shape[0]
        y = torch.empty(self.n * self.shard_rows, N, dtype=a.dtype, device=a.device)
        ops.ext().gemm_allgather(a.contiguous(), w, bool(b_mn), y, [sl[p] for sl in self.slots], self.ready,
                                 self.gath, self.counter, self.me, self.calls, ops.error_flag(a.device))
        return y


_REGISTRY: Dict[Tuple[int, int], PeerGemmAllReduce] = {}


def enable_fused_row_parallel(group, max_rows: int, n_cols_list, device) -> None:
    """Create the peer buffers for the row-parallel GEMMs of a TP group (one per
    output width); afterwards ``row_parallel_linear`` on that group runs the
    fused kernel.  Collective: call on every rank of the group."""
    for n_cols in sorted(set(int(c) for c in n_cols_list)):
        key = (id(group), n_cols)
        if key not in _REGISTRY:
            _REGISTRY[key] = PeerGemmAllReduce(group, max_rows, n_cols, device)


def fused_for(group, n_cols: int, rows: int) -> Optional[PeerGemmAllReduce]:
    f = _REGISTRY.get((id(group), int(n_cols)))
    return f if f is not None and rows <= f.max_rows else None


def disable_fused_row_parallel() -> None:
    for f in _REGISTRY.values():
        f.close()
    _REGISTRY.clear()


class _RowParallelFused(torch.autograd.Function):
    """Forward: fused GEMM + all-reduce (+ residual).  Backward needs no
    collective: dA_r = dY W_r and dW_r = dY^T A_r on every rank."""

    @staticmethod
    def forward(ctx, a, w, residual, fused):
        a2 = a.reshape(-1, a.shape[-1])
        if not a2.is_contiguous():
            a2 = a2.contiguous()
        y = fused(a2, w, residual)
        ctx.save_for_backward(a2, w)
        ctx.in_shape = a.shape
        ctx.has_residual = residual is not None
        return y.view(*a.shape[:-1], w.shape[0])

    @staticmethod
    def backward(ctx, dy):
        a2, w = ctx.saved_tensors
        dy2 = dy.reshape(-1, w.shape[0]).contiguous()
        da = ops.gemm(dy2, w, b_mn=True).view(ctx.in_shape) if ctx.needs_input_grad[0] else None
        dw = ops._accumulate_wgrad(w, dy2, a2) if ctx.needs_input_grad[1] else None
        return da, dw, (dy if ctx.has_residual else None), None


def row_parallel_fused(a, w, residual, fused: PeerGemmAllReduce):
    return _RowParallelFused.apply(a, w, residual, fused)


def _bench(argv=None) -> None:
    """torchrun --nproc-per-node N -m libra_b200.parallel.peer_gemm --rows 16384 --cols 2560 --inner 2048
    [--mode ar|rs|ag|all]: device time of each fused kernel against our GEMM + the NCCL collective
    (max over ranks), and the fraction of its roofline: the slower of the GEMM at the measured
    1622 TFLOP/s burst peak and the bytes that must cross NVLink at 770 GB/s per direction.

    ar: y = sum_r a_r w_r^T on every rank (M x N bf16 all-reduced);
    rs: this rank's M/n rows of that sum (reduce-scatter);
    ag: y = [a_0; ...; a_{n-1}] w^T from row shards a_r of M/n rows (all-gather of A, K columns)."""
    import argparse
    import datetime
    import json
    import os

    ap = argparse.ArgumentParser()
    ap.add_argument("--rows", dest="m", type=int, default=16384)
    ap.add_argument("--cols", dest="n", type=int, default=2560)
    ap.add_argument("--inner", dest="k", type=int, default=2048)
    ap.add_argument("--iters", type=int, default=20)
    ap.add_argument("--mode", default="ar", choices=["ar", "rs", "ag", "all"])
    ap.add_argument("--peak-tflops", type=float, default=1622.0)
    ap.add_argument("--link-gbs", type=float, default=770.0)
    args = ap.parse_args(argv)
    rank = int(os.environ.get("RANK", "0"))
    torch.cuda.set_device(int(os.environ.get("LOCAL_RANK", "0")))
    dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                            device_id=torch.device("cuda", torch.cuda.current_device()))
    world = dist.get_world_size()
    M, N, K = args.m, args.n, args.k
    g = torch.Generator(device="cuda").manual_seed(rank)
    a = torch.randn(M, K, device="cuda", generator=g).bfloat16()
    w = (torch.randn(N, K, device="cuda", generator=g) / K ** 0.5).bfloat16()

    def timed(fn):
        for _ in range(3):
            fn()
        torch.cuda.synchronize()
        dist.barrier()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        for _ in range(args.iters):
            fn()
        e1.record()
        torch.cuda.synchronize()
        t = torch.tensor([e0.elapsed_time(e1) / args.iters], device="cuda")
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return t.item()

    modes = ["ar", "rs", "ag"] if args.mode == "all" else [args.mode]
    for mode in modes:
        if mode in ("ar", "rs"):
            f = PeerGemmAllReduce(dist.group.WORLD, M, N, "cuda")
            flops = 2.0 * M * N * K
            link = (world - 1) / world * M * N * 2 * (2 if mode == "ar" else 1)  # bytes into (and out of) a rank
            if mode == "ar":
                fused, base = (lambda: f(a, w)), None

                def base():
                    y = ops.gemm(a, w)
                    dist.all_reduce(y)
                    return y
            else:
                out = torch.empty(M // world, N, dtype=torch.bfloat16, device="cuda")
                fused = lambda: f.reduce_scatter(a, w)  # noqa: E731

                def base():
                    dist.reduce_scatter_tensor(out, ops.gemm(a, w))
                    return out
        else:
            S = M // world
            f = PeerAllGatherGemm(dist.group.WORLD, S, K, "cuda")
            shard = a[:S].contiguous()
            full = torch.empty(M, K, dtype=torch.bfloat16, device="cuda")
            flops = 2.0 * M * N * K
            link = (world - 1) * S * K * 2
            fused = lambda: f(shard, w)  # noqa: E731

            def base():
                dist.all_gather_into_tensor(full, shard)
                return ops.gemm(full, w)
        tf, tb = timed(fused), timed(base)
        ops.check_kernel_errors()
        bound = max(flops / (args.peak_tflops * 1e12), link / (args.link_gbs * 1e9)) * 1e3
        if rank == 0:
            print(json.dumps({"kernel": {"ar": "gemm_allreduce", "rs": "gemm_reduce_scatter",
                                         "ag": "allgather_gemm"}[mode], "ranks": world, "M": M, "N": N, "K": K,
                              "fused_ms": round(tf, 4), "gemm_plus_nccl_ms": round(tb, 4),
                              "speedup": round(tb / tf, 3), "roofline_ms": round(bound, 4),
                              "fused_of_roofline": round(bound / tf, 3), "nccl_of_roofline": round(bound / tb, 3),
                              "fused_tflops_per_gpu": round(flops / tf / 1e9, 1)}), flush=True)
        f.close()
        dist.barrier()
    dist.destroy_process_group()


if __name__ == "__main__":
    _bench()
