"""Captured decode steps of the rollout engine.

A decode step (one new token for every running sequence) launches ~10 kernels
per layer; at rollout batch sizes each kernel runs for a few microseconds, so
issuing them one by one from Python would leave the GPU idle most of the
step.  ``DecodeGraphs`` records the whole step — embedding, every layer, the
final norm, LM head and the sampler — as one CUDA graph per batch size of a
ladder (1, 2, 4, 8, 16, 24, ... up to ``max_batch``) and replays the smallest
graph that fits the running batch.

Everything the graph reads lives in static device buffers that the host
refreshes before each replay: input tokens, positions, KV slot of the new
token, sequence lengths, block tables, temperatures, seeds.  Rows past the
live batch are padding: they attend to a one-token scratch block that no
sequence owns and their sampled tokens are ignored.  The attention kernel's
split layout is fixed by ``max_model_len`` (not by the current lengths) and
its split workspace is preallocated, so the same graph serves every step of a
generation.

Dense models on one GPU take the fused decode path: every linear layer is the
decode GEMM (gemm_decode: the weight is the 128-row tcgen05 operand and the
batch the N dimension, stream-K over all SMs, fp32 accumulator), so every SM
streams every weight however few rows the batch has; the work after it is one
fused kernel
(q/k norm + RoPE + KV-cache write; residual add + RMSNorm; SwiGLU; sampling),
which also clears the accumulator for its next use.  Attention is the
stream-K paged decode kernel, whose grid is one CTA per SM whatever the
lengths.  Per layer: 4 GEMMs + 5 kernels, chained with programmatic dependent
launch (``LIBRA_DECODE_PDL=0`` turns it off), so each GEMM starts loading its
weights while the kernel before it finishes.  ``LIBRA_DECODE_FUSED=0`` keeps
the unfused kernels (bf16 GEMM epilogues, split-layout attention).

The vLLM servers of the reference do the same with their CUDA-graph mode
(the reference's launch scripts run them with ``--enforce-eager`` instead);
this engine always captures unless ``LIBRA_DECODE_GRAPHS=0``.
"""

from __future__ import annotations

import math
import os
from typing import Dict, List, Optional

import numpy as np
import torch

from libra_b200 import ops


def default_buckets(max_batch: int) -> List[int]:
    ladder = [1, 2, 4, 8, 16, 24, 32, 40, 48, 56, 64, 80, 96, 112, 128, 160, 192, 224, 256, 320, 384, 448, 512]
    out = [b for b in ladder if b < max_batch] + [max_batch]
    return sorted(set(out))


def graphs_enabled() -> bool:
    return os.environ.get("LIBRA_DECODE_GRAPHS", "1") != "0"


class DecodeGraphs:
    """One CUDA graph per batch-size bucket for the single-token decode step."""

    def __init__(self, runner, max_batch: int = 256, max_model_len: int = 8192, split_len: int = 512,
                 buckets: Optional[List[int]] = None):
        self.r = runner
        cfg, dev, kv = runner.cfg, runner.device, runner.kv
        self.cfg, self.device, self.kv = cfg, dev, kv
        self.max_batch = int(max_batch)
        self.bs = kv.block_size
        self.max_blocks = -(-int(max_model_len) // self.bs)
        self.split_len = int(split_len)
        self.S = -(-int(max_model_len) // self.split_len)
        self.buckets = buckets or default_buckets(self.max_batch)
        B, nq = self.max_batch, runner.nq
        # scratch KV block for padding rows (never owned by a sequence)
        self.scratch_block = kv.alloc.allocate()
        # host staging (pinned) and device buffers
        self.h64 = torch.zeros(4, B, dtype=torch.long).pin_memory()     # token, slot, seed, position
        self.h32 = torch.zeros(2, B, dtype=torch.int32).pin_memory()    # position, length
        self.hf = torch.zeros(B, dtype=torch.float32).pin_memory()      # temperature
        self.htbl = torch.full((B, self.max_blocks), self.scratch_block, dtype=torch.int32).pin_memory()
        self.n64, self.n32, self.nf, self.ntbl = (self.h64.numpy(), self.h32.numpy(), self.hf.numpy(),
                                                  self.htbl.numpy())
        self.d64 = torch.zeros(4, B, dtype=torch.long, device=dev)
        self.d32 = torch.zeros(2, B, dtype=torch.int32, device=dev)
        self.df = torch.zeros(B, dtype=torch.float32, device=dev)
        self.dtbl = torch.full((B, self.max_blocks), self.scratch_block, dtype=torch.int32, device=dev)
        self.out_tok = torch.zeros(B, dtype=torch.long, device=dev)
        self.out_lp = torch.zeros(B, dtype=torch.float32, device=dev)
        self.h_out_tok = torch.zeros(B, dtype=torch.long).pin_memory()
        self.h_out_lp = torch.zeros(B, dtype=torch.float32).pin_memory()
        self.attn_out = torch.zeros(B, nq, cfg.head_dim, dtype=torch.bfloat16, device=dev)
        self.part_out = torch.zeros(B, nq, self.S, cfg.head_dim, dtype=torch.float32, device=dev)
        self.part_ml = torch.zeros(B, nq, self.S, 2, dtype=torch.float32, device=dev)
        self.fused = self._fused_supported()
        # programmatic dependent launch between the kernels of the fused step
        self.pdl = self.fused and os.environ.get("LIBRA_DECODE_PDL", "1") != "0"
        if self.fused:
            H, F = cfg.hidden_size, cfg.intermediate_size
            V = runner.lm_head.shape[0]
            nkv = runner.nkv
            f32 = dict(dtype=torch.float32, device=dev)
            bf = dict(dtype=torch.bfloat16, device=dev)
            # stream-K accumulators: zero now, and every consumer leaves them zero
            self.acc_qkv = torch.zeros(B, (nq + 2 * nkv) * cfg.head_dim, **f32)
            self.acc_h = torch.zeros(B, H, **f32)
            self.acc_gu = torch.zeros(B, 2 * F, **f32)
            self.acc_logits = torch.zeros(B, V, **f32)
            self.xbuf = torch.zeros(B, H, **bf)
            self.hbuf = torch.zeros(B, H, **bf)
            self.qbuf = torch.zeros(B, nq, cfg.head_dim, **bf)
            self.abuf = torch.zeros(B, F, **bf)
            self.attn_ws = ops.decode_workspace(B, nq, cfg.head_dim, dev)
        self._pad_rows(0, B)
        # per-row cache of what the block-table staging row holds: (seq_id, blocks written)
        self._row_owner: List[Optional[str]] = [None] * B
        self._row_nblocks = [0] * B
        self.graphs: Dict[int, torch.cuda.CUDAGraph] = {}
        self.pool = None
        self.replays = 0
        self.io_bytes = {"h2d": 0, "d2h": 0}

    def _fused_supported(self) -> bool:
        r, cfg = self.r, self.cfg
        if os.environ.get("LIBRA_DECODE_FUSED", "1") == "0" or self.device.type != "cuda":
            return False
        return (not cfg.is_moe and r.tp_size == 1 and cfg.head_dim == 128 and self.bs == 16
                and cfg.num_attention_heads % cfg.num_key_value_heads == 0
                and cfg.num_attention_heads // cfg.num_key_value_heads in (1, 2, 4, 5, 8)
                and cfg.num_key_value_heads <= 8 and cfg.hidden_size % 8 == 0 and cfg.hidden_size <= 8192)

    def reset_accumulators(self) -> None:
        """Zero the stream-K accumulators and attention counters (after a
        failed replay, whose consumers may not have run)."""
        if self.fused:
            for t in (self.acc_qkv, self.acc_h, self.acc_gu, self.acc_logits, self.attn_ws[2]):
                t.zero_()

    # ------------------------------------------------------------------ forward recorded in the graphs
    def _forward_fused(self, b: int) -> None:
        r, cfg, p = self.r, self.cfg, self.r.p
        eps = cfg.rms_norm_eps
        pdl = self.pdl
        gemm = ops.gemm_decode
        tok, slot, seed, pos64 = self.d64[0, :b], self.d64[1, :b], self.d64[2, :b], self.d64[3, :b]
        pos32, lens = self.d32[0, :b], self.d32[1, :b]
        x, h = self.xbuf[:b], self.hbuf[:b]
        acc_h = self.acc_h[:b]
        torch.index_select(p["embed_tokens"], 0, tok, out=x)
        # acc_h is zero here, so this is the first layer's input RMSNorm
        ops.decode_residual_norm(x, acc_h, p["layers.0.input_layernorm"], h, eps, pdl=pdl)
        part_o, part_ml, counters = self.attn_ws
        L = cfg.num_hidden_layers
        for layer in range(L):
            pre = f"layers.{layer}."
            gemm(h, p[pre + "qkv_proj"], self.acc_qkv[:b], pdl=pdl)
            ops.decode_qkv_post(self.acc_qkv[:b], p[pre + "q_norm"], p[pre + "k_norm"], pos32, r.cos, r.sin, slot,
                                self.qbuf[:b], self.kv.k[layer], self.kv.v[layer], eps, pdl=pdl)
            attn = ops.decode_attention(self.qbuf[:b], self.kv.k[layer], self.kv.v[layer], self.dtbl, lens,
                                        self.attn_out[:b], part_o, part_ml, counters, r.scale, pdl=pdl)
            gemm(attn.view(b, -1), p[pre + "o_proj"], acc_h, pdl=pdl)
            ops.decode_residual_norm(x, acc_h, p[pre + "post_attention_layernorm"], h, eps, pdl=pdl)
            gemm(h, p[pre + "gate_up_proj"], self.acc_gu[:b], pdl=pdl)
            ops.decode_swiglu(self.acc_gu[:b], self.abuf[:b], pdl=pdl)
            gemm(self.abuf[:b], p[pre + "down_proj"], acc_h, pdl=pdl)
            nxt = p[f"layers.{layer + 1}.input_layernorm"] if layer + 1 < L else p["norm"]
            ops.decode_residual_norm(x, acc_h, nxt, h, eps, pdl=pdl)
        gemm(h, r.lm_head, self.acc_logits[:b], pdl=pdl)
        ops.sample_tokens(self.acc_logits[:b], self.df[:b], seed, pos64, self.out_tok[:b], self.out_lp[:b], pdl=pdl)

    def _forward(self, b: int) -> None:
        if self.fused:
            return self._forward_fused(b)
        r, cfg, p = self.r, self.cfg, self.r.p
        tok, slot, seed, pos64 = self.d64[0, :b], self.d64[1, :b], self.d64[2, :b], self.d64[3, :b]
        pos32, lens = self.d32[0, :b], self.d32[1, :b]
        x = p["embed_tokens"].index_select(0, tok)
        for layer in range(cfg.num_hidden_layers):
            pre = f"layers.{layer}."
            h = ops.rmsnorm(x, p[pre + "input_layernorm"], cfg.rms_norm_eps)
            qkv = ops.linear(h, p[pre + "qkv_proj"])
            q, k, v = ops.qk_norm_rope(qkv, p[pre + "q_norm"], p[pre + "k_norm"], pos32, r.cos, r.sin, r.nq, r.nkv,
                                       cfg.rms_norm_eps)
            self.kv.write(layer, slot, k, v)
            attn = ops.paged_decode(q, self.kv.k[layer], self.kv.v[layer], self.dtbl, lens, self.attn_out[:b],
                                    self.part_out, self.part_ml, self.split_len, r.scale)
            x = ops.linear(attn.reshape(b, -1), p[pre + "o_proj"], residual=x)
            h = ops.rmsnorm(x, p[pre + "post_attention_layernorm"], cfg.rms_norm_eps)
            x = ops.linear(ops.linear_swiglu(h, p[pre + "gate_up_proj"]), p[pre + "down_proj"], residual=x)
        last = ops.rmsnorm(x, p["norm"], cfg.rms_norm_eps)
        logits = ops.linear(last, r.lm_head)
        ops.sample_tokens(logits, self.df[:b], seed, pos64, self.out_tok[:b], self.out_lp[:b])

    @torch.no_grad()
    def capture(self) -> None:
        """Record one graph per bucket, largest first (they share one memory pool)."""
        stream = torch.cuda.Stream(self.device)
        stream.wait_stream(torch.cuda.current_stream(self.device))
        with torch.cuda.stream(stream):
            for b in sorted(self.buckets, reverse=True):
                self._upload(b)
                self._forward(b)   # warm-up: kernel attributes, tensor-map encoders, allocator
                torch.cuda.synchronize(self.device)
                g = torch.cuda.CUDAGraph()
                with torch.cuda.graph(g, pool=self.pool, stream=stream):
                    self._forward(b)
                if self.pool is None:
                    self.pool = g.pool()
                self.graphs[b] = g
        torch.cuda.current_stream(self.device).wait_stream(stream)
        torch.cuda.synchronize(self.device)

    # ------------------------------------------------------------------ host side of a step
    def bucket(self, n: int) -> int:
        for b in self.buckets:
            if b >= n:
                return b
        raise ValueError(f"decode batch {n} exceeds the captured maximum {self.max_batch}")

    def _pad_rows(self, lo: int, hi: int) -> None:
        if hi <= lo:
            return
        slot0 = self.scratch_block * self.bs
        self.n64[0, lo:hi] = 0
        self.n64[1, lo:hi] = slot0
        self.n64[2, lo:hi] = 0
        self.n64[3, lo:hi] = 0
        self.n32[0, lo:hi] = 0
        self.n32[1, lo:hi] = 1
        self.nf[lo:hi] = 0.0
        self.ntbl[lo:hi, 0] = self.scratch_block

    def set_row(self, i: int, seq_id: str, token: int, length: int, temperature: float, seed: int) -> None:
        """Row ``i`` decodes the token at position ``length - 1`` of ``seq_id``
        (whose KV blocks must already cover ``length`` tokens)."""
        blocks = self.kv.seqs[seq_id].blocks
        pos = length - 1
        n64 = self.n64
        n64[0, i] = token
        n64[1, i] = blocks[pos // self.bs] * self.bs + pos % self.bs
        n64[2, i] = seed
        n64[3, i] = pos
        self.n32[0, i] = pos
        self.n32[1, i] = length
        self.nf[i] = temperature
        nb = len(blocks)
        if self._row_owner[i] == seq_id:
            have = self._row_nblocks[i]
            if nb > have:
                self.ntbl[i, have:nb] = blocks[have:nb]
                self._row_nblocks[i] = nb
        else:
            self.ntbl[i, :nb] = blocks
            self._row_owner[i] = seq_id
            self._row_nblocks[i] = nb

    def _upload(self, b: int) -> None:
        self.d64[:, :b].copy_(self.h64[:, :b], non_blocking=True)
        self.d32[:, :b].copy_(self.h32[:, :b], non_blocking=True)
        self.df[:b].copy_(self.hf[:b], non_blocking=True)
        self.dtbl[:b].copy_(self.htbl[:b], non_blocking=True)

    def run(self, n: int):
        """Replay the bucket graph for rows 0..n-1; returns (tokens, logprobs) as lists."""
        b = self.bucket(n)
        if n < b:
            self._pad_rows(n, b)
            for i in range(n, b):
                self._row_owner[i] = None
        self._upload(b)
        self.io_bytes["h2d"] += b * (4 * 8 + 2 * 4 + 4 + 4 * self.max_blocks)
        self.io_bytes["d2h"] += n * 12
        self.graphs[b].replay()
        self.replays += 1
        self.h_out_tok[:n].copy_(self.out_tok[:n], non_blocking=True)
        self.h_out_lp[:n].copy_(self.out_lp[:n], non_blocking=True)
        torch.cuda.current_stream(self.device).synchronize()
        return self.h_out_tok[:n].tolist(), self.h_out_lp[:n].tolist()
