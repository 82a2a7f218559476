"""Pipeline parallelism: 1F1B schedule over point-to-point activation exchange.

Reference: the Megatron3D engine's own 1F1B (``engine/megatron_train_engine.py``,
p2p at ``:399-430``).  A stage is a callable ``forward(mb, x) -> y`` (x is None
on the first stage, which embeds its micro-batch itself); the last stage's
output is the scalar loss of the micro-batch.  Activations are [tokens, H]
with a per-micro-batch token count, so every transfer is preceded by its shape
(two int64s).  Schedule per stage with S stages, M micro-batches, rank r:
warm-up min(S - r - 1, M) forwards, then alternate one forward / one backward,
then drain the remaining backwards - at most S - r activations stay alive.
"""

from __future__ import annotations

from typing import Any, Callable, List, Optional, Sequence

import torch
import torch.distributed as dist


class P2P:
    def __init__(self, group, prev_rank: Optional[int], next_rank: Optional[int], dtype=torch.bfloat16,
                 device=None):
        self.group, self.prev, self.next = group, prev_rank, next_rank
        self.dtype, self.device = dtype, device
        self._pending: List = []  # (work, tensors kept alive until the send completes)

    def _send(self, t: torch.Tensor, dst: int) -> None:
        # Sends are non-blocking: in the 1F1B steady state a stage sends its
        # activation forward while its neighbour sends a gradient back.
        shape = torch.tensor(list(t.shape) + [0] * (2 - t.dim()), dtype=torch.int64, device=t.device)
        t = t.contiguous()
        self._pending.append((dist.isend(shape, dst, group=self.group), shape))
        self._pending.append((dist.isend(t, dst, group=self.group), t))

    def wait_sends(self) -> None:
        for work, _ in self._pending:
            work.wait()
        self._pending.clear()

    def _recv(self, src: int, dtype) -> torch.Tensor:
        shape = torch.empty(2, dtype=torch.int64, device=self.device)
        dist.recv(shape, src, group=self.group)
        t = torch.empty(int(shape[0]), int(shape[1]), dtype=dtype, device=self.device)
        dist.recv(t, src, group=self.group)
        return t

    def send_forward(self, y):
        if self.next is not None:
            self._send(y.detach(), self.next)

    def recv_forward(self):
        return None if self.prev is None else self._recv(self.prev, self.dtype)

    def send_backward(self, g):
        if self.prev is not None:
            self._send(g, self.prev)

    def recv_backward(self):
        return None if self.next is None else self._recv(self.next, self.dtype)


def one_f_one_b(stage_forward: Callable[[Any, Optional[torch.Tensor]], torch.Tensor], micro_batches: Sequence[Any],
                p2p: P2P, num_stages: int, stage_rank: int) -> List[float]:
    """Run forward+backward of every micro-batch; returns the last stage's losses."""
    M = len(micro_batches)
    warm = min(num_stages - stage_rank - 1, M)
    last = stage_rank == num_stages - 1
    inputs: List[Optional[torch.Tensor]] = []
    outputs: List[torch.Tensor] = []
    losses: List[float] = []

    def fwd(i: int) -> None:
        x = p2p.recv_forward()
        if x is not None:
            x = x.requires_grad_(True)
        y = stage_forward(micro_batches[i], x)
        if last:
            losses.append(float(y.detach()))
        else:
            p2p.send_forward(y)
        inputs.append(x)
        outputs.append(y)

    def bwd() -> None:
        x, y = inputs.pop(0), outputs.pop(0)
        if last:
            y.backward()
        else:
            g = p2p.recv_backward()
            y.backward(g)
        if x is not None:
            p2p.send_backward(x.grad)

    for i in range(warm):
        fwd(i)
    for i in range(warm, M):
        fwd(i)
        bwd()
    for _ in range(warm):
        bwd()
    p2p.wait_sends()
    return losses


class PipelineStage:
    """Layers [first, last) of a Qwen3Model as one pipeline stage."""

    def __init__(self, model, first_layer: int, last_layer: int, is_first: bool, is_last: bool, loss_fn=None):
        self.model, self.first, self.last = model, first_layer, last_layer
        self.is_first, self.is_last, self.loss_fn = is_first, is_last, loss_fn

    @staticmethod
    def split_layers(num_layers: int, num_stages: int) -> List[range]:
        base, extra = divmod(num_layers, num_stages)
        out, start = [], 0
        for s in range(num_stages):
            n = base + (1 if s < extra else 0)
            out.append(range(start, start + n))
            start += n
        return out

    def __call__(self, mb, x):
        m = self.model
        batch = mb["batch"]
        if self.is_first:
            x = m.embed(batch.tokens)
        for i in range(self.first, self.last):
            x = m._layer(i, x, batch.positions, batch.cu_seqlens, batch.max_seqlen, batch.tiles)
        if not self.is_last:
            return x
        from libra_b200 import ops

        h = ops.rmsnorm(x, m.p["norm"], m.cfg.rms_norm_eps)
        rows = h.index_select(0, batch.action_rows)
        logp = ops.lm_head_logprob(rows, m.lm_head_weight, batch.action_targets, mb.get("temperature", 1.0))
        return self.loss_fn(logp, mb)


def allreduce_tied_embedding_grad(param: torch.Tensor, group) -> None:
    """With tied word embeddings the first stage (embedding) and the last stage
    (LM head) each hold part of the gradient; sum them (reference: Megatron's
    embedding group)."""
    g = getattr(param, "main_grad", None)
    if g is None:
        if param.grad is None:
            param.grad = torch.zeros_like(param)
        g = param.grad
    dist.all_reduce(g, group=group)
