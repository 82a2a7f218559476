"""Tensor-parallel all-reduce over NVLink peer memory (rollout decode path).

Each TP rank allocates one device buffer (two partial-output slots + a flag
area), shares it with its peers through CUDA IPC handles exchanged over the
process group, and maps the peers' buffers.  The row-parallel GEMM writes its
partial output straight into the current slot (``partial(rows)``);
``reduce_add_rmsnorm`` then runs one kernel on every rank that synchronises on
the peer flags and sums the N partials over NVLink, adding the residual and
applying the next RMSNorm (``ops/csrc/tp_allreduce.cu``).  Replaces the NCCL
all-reduce + separate add + RMSNorm of the reference's rollout path (inside
vLLM).  One buffer per process group and shape; calls must be issued in the
same order on every rank.
"""

from __future__ import annotations

import torch
import torch.distributed as dist

from libra_b200 import ops

MAX_CTAS = 512
MAX_RANKS = 8
WARPS = 8


class PeerAllReduce:
    def __init__(self, group, max_rows: int, hidden: int, device):
        self.group = group
        self.n = dist.get_world_size(group) if dist.is_initialized() else 1
        self.me = dist.get_rank(group) if dist.is_initialized() else 0
        if self.n > MAX_RANKS:
            raise ValueError(f"at most {MAX_RANKS} ranks")
        self.max_rows, self.hidden = int(max_rows), int(hidden)
        self.slot_bytes = (self.max_rows * self.hidden * 2 + 255) // 256 * 256
        flag_bytes = MAX_CTAS * MAX_RANKS * 4
        self.buf = torch.zeros(2 * self.slot_bytes + flag_bytes, dtype=torch.uint8, device=device)
        self.data_ptrs = [int(self.buf.data_ptr())]
        self._opened = []
        if self.n > 1:
            # map every peer's buffer into THIS device's context, so kernels
            # running here can load from it over NVLink
            C = ops.ext()
            handles = [None] * self.n
            dist.all_gather_object(handles, C.ipc_export(self.buf), group=self.group)
            self.data_ptrs = []
            with torch.cuda.device(self.buf.device):
                for r, (h, off) in enumerate(handles):
                    if r == self.me:
                        self.data_ptrs.append(int(self.buf.data_ptr()))
                    else:
                        base = C.ipc_open(h)
                        self._opened.append(base)
                        self.data_ptrs.append(base + int(off))
        self.flag_ptrs = [p + 2 * self.slot_bytes for p in self.data_ptrs]
        self.epoch = 0
        if self.n > 1:
            torch.cuda.synchronize(device)
            dist.barrier(group=self.group)

    def close(self) -> None:
        for base in self._opened:
            ops.ext().ipc_close(base)
        self._opened = []

    def _slot(self, epoch: int) -> int:
        return epoch % 2

    def partial(self, rows: int) -> torch.Tensor:
        """bf16 [rows, hidden] view the next call reduces (write the partial here)."""
        if rows > self.max_rows:
            raise ValueError(f"{rows} rows exceed the buffer's {self.max_rows}")
        off = self._slot(self.epoch + 1) * self.slot_bytes
        return self.buf[off:off + rows * self.hidden * 2].view(torch.bfloat16).view(rows, self.hidden)

    def reduce_add_rmsnorm(self, residual: torch.Tensor, weight: torch.Tensor, eps: float):
        """(x, h): x = residual + sum of partials, h = rmsnorm(x) * weight."""
        rows = residual.shape[0]
        self.epoch += 1
        grid = max(1, min(MAX_CTAS, (rows + WARPS - 1) // WARPS))
        return ops.ext().tp_allreduce_add_rmsnorm(self.data_ptrs, self.flag_ptrs, self.me,
                                                  self._slot(self.epoch) * self.slot_bytes,
                                                  residual.contiguous(), weight, float(eps), self.epoch, grid,
                                                  ops.error_flag(residual.device))
