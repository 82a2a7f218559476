"""Analytic cost model of one asynchronous GRPO step on an NVSwitch box.

The decomposition follows the reference (``infra/cost_model/model.py``):

* **Rollout** — per instance: per-token KV bytes ``2 L ceil(kv/tp) d b``; KV pool
  = tp x HBM - weights - workspace; prefill step = FLOPs / (tp peak MFU) +
  per-layer TP sync; decode step = (weights/tp + active KV) / (tp BW util) +
  per-layer TP sync; steady batch = capacity / (prompt + gen/2); requests are
  assigned greedily longest-first to the instance that finishes them first;
  cluster makespan = max over instances of (prefill + decode time).
* **Training** — memory per GPU, forward/backward time per micro-batch, 1F1B
  pipeline, exposed DP communication; global step = max(T_train, T_rollout).

What is re-derived for B200 (this framework's engine, not Megatron's):

* Memory: flat bf16 params (2P/tp), flat fp32 gradients (4P/tp), fp32
  master + Adam (12P, sharded over DP with the distributed optimizer),
  activations of a packed micro-batch (``act_bytes_per_token_layer``; stored,
  not recomputed, unless ``recompute``), and the LM-head logits kept in bf16
  only for action rows (fused logprob: no fp32 [tokens, vocab] temporary).
* Compute: FLOP-based (6 N T + attention) against the measured sustained bf16
  GEMM rate times a training MFU (``prefill_mfu`` reused for the fused
  kernels), instead of alpha/beta per-op fits.  The reference's alpha/beta/
  gamma model stays available with ``use_profiled_coefficients=True``.
* Communication: NVLink 5 peer bandwidth for TP (fused AG->GEMM / GEMM->RS
  overlap most of it: ``tp_overlap``), DP reduce-scatter + all-gather
  (overlapped with backward: ``dp_overlap``) and MoE all-to-all.
"""

from __future__ import annotations

import math
from dataclasses import dataclass, field
from typing import Any, Dict, List, Optional, Tuple

from libra_b200.infra.cost_model.memory_budget import estimate_recompute_logprobs_memory


@dataclass
class RequestInfo:
    prompt_length: int
    gen_length: int

    @property
    def total_length(self) -> int:
        return self.prompt_length + self.gen_length


@dataclass
class InstanceConfig:
    tp: int
    token_capacity: int = 0
    assigned_requests: List[RequestInfo] = field(default_factory=list)


@dataclass
class TrainParallelConfig:
    tp: int = 1
    pp: int = 1
    dp: int = 1
    b_micro: int = 4
    zero_level: int = 1  # 1 = distributed optimizer (master/Adam sharded over DP)
    cp: int = 1
    ep: int = 1

    @property
    def n_gpus(self) -> int:
        return self.tp * self.pp * self.cp * self.dp


@dataclass
class RolloutClusterConfig:
    tp_list: List[int] = field(default_factory=list)

    @property
    def n_gpus(self) -> int:
        return sum(self.tp_list)

    @property
    def n_instances(self) -> int:
        return len(self.tp_list)


@dataclass
class CostModelResult:
    t_train: float = 0.0
    t_rollout: float = 0.0
    t_global: float = 0.0
    is_oom: bool = False
    oom_source: str = ""
    details: Dict[str, Any] = field(default_factory=dict)


def _mean(xs):
    xs = list(xs)
    return float(sum(xs)) / len(xs) if xs else 0.0


# =============================================================================== rollout
class RolloutCostModel:
    def __init__(self, num_params: float, d_model: int, n_layers: int, n_kv_heads: int, head_dim: int,
                 dtype_bytes: int, flops_peak: float, mem_bw: float, mem_capacity: float, tp_comm_overhead: float,
                 prefill_mfu: float = 0.55, decode_bw_util: float = 0.85, prefill_chunk_size: int = 1024,
                 kv_frag_rate: float = 0.04, act_workspace_bytes: float = 1.0e9, max_queue_limit: int = 256,
                 effective_num_params: Optional[float] = None, n_heads: int = 0,
                 decode_layer_overhead_s: float = 0.0, decode_row_layer_s: float = 0.0):
        self.P = num_params
        self.P_active = effective_num_params or num_params
        self.d_model, self.n_layers = d_model, n_layers
        self.n_kv_heads, self.head_dim, self.dtype_bytes = n_kv_heads, head_dim, dtype_bytes
        self.n_heads = n_heads or max(1, d_model // max(head_dim, 1))
        self.flops_peak, self.mem_bw, self.mem_capacity = flops_peak, mem_bw, mem_capacity
        self.tp_comm_overhead = tp_comm_overhead
        self.prefill_mfu, self.decode_bw_util = prefill_mfu, decode_bw_util
        self.L_chunk = prefill_chunk_size
        self.kv_frag_rate, self.act_workspace = kv_frag_rate, act_workspace_bytes
        self.max_queue_limit = max_queue_limit
        self.decode_layer_overhead_s = decode_layer_overhead_s
        self.decode_row_layer_s = decode_row_layer_s

    def compute_token_kv_bytes(self, tp: int) -> float:
        """KV bytes per token held by ONE GPU of a TP group (heads replicated if tp > kv)."""
        return 2.0 * self.n_layers * max(1, self.n_kv_heads // tp) * self.head_dim * self.dtype_bytes

    def compute_kv_pool(self, tp: int) -> float:
        return max(tp * self.mem_capacity - self.P * self.dtype_bytes - self.act_workspace, 0.0)

    def compute_token_capacity(self, tp: int) -> int:
        per_tok = self.compute_token_kv_bytes(tp) * tp  # whole TP group
        if per_tok <= 0:
            return 0
        return int(self.compute_kv_pool(tp) / per_tok * (1.0 - self.kv_frag_rate))

    def _tp_sync(self, tp: int) -> float:
        return 2.0 * self.n_layers * self.tp_comm_overhead if tp > 1 else 0.0

    def compute_prefill_step_time(self, B_prefill: int, L_chunk: int, tp: int) -> float:
        tokens = B_prefill * L_chunk
        linear = 2.0 * self.P_active * tokens
        attn = 4.0 * self.n_layers * B_prefill * L_chunk * L_chunk * self.n_heads * self.head_dim / 2.0
        return (linear + attn) / (tp * self.flops_peak * max(self.prefill_mfu, 1e-6)) + self._tp_sync(tp)

    def compute_decode_step_time(self, total_active_tokens: int, tp: int) -> float:
        read = self.P_active * self.dtype_bytes / tp + total_active_tokens * self.compute_token_kv_bytes(tp)
        return read / (self.mem_bw * max(self.decode_bw_util, 1e-6)) + self._tp_sync(tp)

    def compute_steady_state_batch(self, tp: int, avg_prompt_len: float, avg_gen_len: float) -> float:
        occupancy = avg_prompt_len + avg_gen_len / 2.0
        if occupancy <= 0:
            return 1.0
        return max(1.0, min(float(self.max_queue_limit), self.compute_token_capacity(tp) / occupancy))

    def compute_instance_throughput(self, tp: int, avg_prompt_len: float, avg_gen_len: float) -> float:
        b = self.compute_steady_state_batch(tp, avg_prompt_len, avg_gen_len)
        t = self.compute_decode_step_time(int(b * (avg_prompt_len + avg_gen_len / 2.0)), tp)
        return b / t if t > 0 else float("inf")

    def greedy_throughput_allocation(self, requests: List[RequestInfo], cluster: RolloutClusterConfig) -> List[InstanceConfig]:
        """Longest request first, onto the instance that would finish it earliest."""
        insts = [InstanceConfig(tp=tp) for tp in cluster.tp_list]
        if not requests or not insts:
            return insts
        ap, ag = _mean(r.prompt_length for r in requests), _mean(r.gen_length for r in requests)
        rate = [self.compute_instance_throughput(i.tp, ap, ag) for i in insts]
        load = [0.0] * len(insts)
        for req in sorted(requests, key=lambda r: r.total_length, reverse=True):
            finish = [(load[i] + req.total_length) / rate[i] if rate[i] > 0 else float("inf")
                      for i in range(len(insts))]
            best = min(range(len(insts)), key=finish.__getitem__)
            insts[best].assigned_requests.append(req)
            load[best] += req.total_length
        return insts

    def simulate_instance_makespan(self, requests: List[RequestInfo], tp: int) -> float:
        """Step-by-step makespan of one instance that admits every request at
        once (up to the steady batch) and decodes one token per running
        sequence per step, the batch shrinking as sequences finish; a finished
        sequence's slot goes to the next waiting request.  Step time = fixed
        latency + running rows x per-row time + (weights / tp + resident KV) /
        (bandwidth x utilisation).  Between two finish events the running set is
        constant and its KV grows by one token per sequence per step, so each
        segment is summed in closed form."""
        import heapq

        ap, ag = _mean(r.prompt_length for r in requests), _mean(r.gen_length for r in requests)
        cap = max(1, int(self.compute_steady_state_batch(tp, ap, ag)))
        kv_tok = self.compute_token_kv_bytes(tp)
        w = self.P_active * self.dtype_bytes / tp
        bw = self.mem_bw * max(self.decode_bw_util, 1e-6)
        fixed = self.n_layers * self.decode_layer_overhead_s + self._tp_sync(tp)
        row = self.n_layers * self.decode_row_layer_s
        waiting = list(requests)
        prefill = sum(r.prompt_length for r in requests) / max(self.L_chunk, 1) * \
            self.compute_prefill_step_time(1, self.L_chunk, tp)
        heap: List[Tuple[int, int]] = []  # (finish step, request index)
        ctx0 = {}                         # request index -> (start step, prompt length)
        step, nxt, total, kv_at_step = 0, 0, 0.0, 0.0

        def admit(at: int) -> None:
            nonlocal nxt
            while nxt < len(waiting) and len(heap) < cap:
                r = waiting[nxt]
                heapq.heappush(heap, (at + max(1, r.gen_length), nxt))
                ctx0[nxt] = (at, r.prompt_length)
                nxt += 1

        admit(0)
        while heap:
            end = heap[0][0]
            k = end - step
            if k > 0:
                n = len(heap)
                # resident KV tokens at the first step of the segment
                kv0 = sum(p + (step - s0) for s0, p in (ctx0[i] for _, i in heap))
                kv_sum = k * kv0 + n * k * (k - 1) / 2.0
                total += k * (fixed + n * row) + (k * w + kv_sum * kv_tok) / bw
                step = end
            while heap and heap[0][0] == step:
                _, i = heapq.heappop(heap)
                del ctx0[i]
            admit(step)
        return prefill + total

    def compute_instance_makespan(self, requests: List[RequestInfo], tp: int) -> float:
        if not requests:
            return 0.0
        if self.decode_layer_overhead_s > 0.0 or self.decode_row_layer_s > 0.0:
            return self.simulate_instance_makespan(requests, tp)
        ap, ag = _mean(r.prompt_length for r in requests), _mean(r.gen_length for r in requests)
        b = self.compute_steady_state_batch(tp, ap, ag)
        prefill = sum(r.prompt_length for r in requests) / max(self.L_chunk, 1) * \
            self.compute_prefill_step_time(1, self.L_chunk, tp)
        decode = sum(r.gen_length for r in requests) / max(b, 1.0) * \
            self.compute_decode_step_time(int(b * (ap + ag / 2.0)), tp)
        return prefill + decode

    def check_oom(self, max_total_seq: int, tp: int) -> bool:
        return max_total_seq > self.compute_token_capacity(tp)

    def evaluate_cluster(self, cluster: RolloutClusterConfig, requests: List[RequestInfo]) -> Tuple[float, dict]:
        if not cluster.tp_list:
            return float("inf"), {"error": "empty cluster"}
        if requests:
            longest, widest = max(r.total_length for r in requests), max(cluster.tp_list)
            if self.check_oom(longest, widest):
                return float("inf"), {"oom": True, "max_seq": longest, "max_tp": widest,
                                      "token_capacity": self.compute_token_capacity(widest)}
        insts = self.greedy_throughput_allocation(requests, cluster)
        times = [self.compute_instance_makespan(i.assigned_requests, i.tp) for i in insts]
        span = max(times) if times else 0.0
        return span, {"instance_times": times, "n_instances": len(insts),
                      "requests_per_instance": [len(i.assigned_requests) for i in insts], "makespan": span,
                      "token_capacities": [self.compute_token_capacity(i.tp) for i in insts]}


# =============================================================================== training
class TrainingCostModel:
    def __init__(self, num_params: float, d_model: int, n_layers: int, n_kv_heads: int, head_dim: int,
                 dtype_bytes: int, flops_peak: float, mem_bw: float, mem_capacity: float, bw_intra_node: float,
                 bw_inter_node: float, gpus_per_node: int, latency_inter_node: float = 5e-6,
                 alpha_mlp_fwd: float = 3.5e-8, beta_mlp_fwd: float = 1.0e-5, alpha_mlp_bwd: float = 7.0e-8,
                 beta_mlp_bwd: float = 2.0e-5, alpha_attn_fwd: float = 1.5e-12, beta_attn_fwd: float = 2.5e-8,
                 gamma_attn_fwd: float = 8.0e-6, alpha_attn_bwd: float = 3.0e-12, beta_attn_bwd: float = 5.0e-8,
                 gamma_attn_bwd: float = 1.5e-5, rho_compute_bound: float = 0.08, rho_memory_bound: float = 0.45,
                 theta_slowdown: float = 1.0, train_mem_frag_rate: float = 0.08, train_workspace_bytes: float = 0.5e9,
                 effective_num_params: Optional[float] = None, vocab_size: int = 151936, max_seq_length: int = 2048,
                 recompute_logprobs: bool = True, recompute_micro_batch_size: int = 1,
                 recompute_logits_dtype_bytes: int = 4, recompute_workspace_factor: float = 1.5,
                 memory_safety_margin_bytes: float = 0.0, n_heads: int = 0, intermediate_size: int = 0,
                 train_mfu: float = 0.55, recompute_activations: bool = False, tp_overlap: float = 0.8,
                 dp_overlap: float = 0.7, fused_logprob: bool = True, use_profiled_coefficients: bool = False,
                 num_experts: int = 1, top_k: int = 1):
        self.P = num_params
        self.P_active = effective_num_params or num_params
        self.d_model, self.n_layers, self.n_kv_heads, self.head_dim = d_model, n_layers, n_kv_heads, head_dim
        self.n_heads = n_heads or max(1, d_model // max(head_dim, 1))
        self.ffn = intermediate_size or 4 * d_model
        self.dtype_bytes = dtype_bytes
        self.flops_peak, self.mem_bw, self.mem_capacity = flops_peak, mem_bw, mem_capacity
        self.bw_intra, self.bw_inter, self.gpus_per_node = bw_intra_node, bw_inter_node, gpus_per_node
        self.latency_inter = latency_inter_node
        self.coef = dict(alpha_mlp_fwd=alpha_mlp_fwd, beta_mlp_fwd=beta_mlp_fwd, alpha_mlp_bwd=alpha_mlp_bwd,
                         beta_mlp_bwd=beta_mlp_bwd, alpha_attn_fwd=alpha_attn_fwd, beta_attn_fwd=beta_attn_fwd,
                         gamma_attn_fwd=gamma_attn_fwd, alpha_attn_bwd=alpha_attn_bwd, beta_attn_bwd=beta_attn_bwd,
                         gamma_attn_bwd=gamma_attn_bwd)
        self.rho_compute, self.rho_memory, self.theta = rho_compute_bound, rho_memory_bound, theta_slowdown
        self.mem_frag_rate, self.workspace = train_mem_frag_rate, train_workspace_bytes
        self.vocab_size = max(1, int(vocab_size))
        self.max_seq_length = max(1, int(max_seq_length))
        self.recompute_logprobs = bool(recompute_logprobs)
        self.recompute_micro_batch_size = max(1, int(recompute_micro_batch_size))
        self.recompute_logits_dtype_bytes = max(1, int(recompute_logits_dtype_bytes))
        self.recompute_workspace_factor = max(1.0, float(recompute_workspace_factor))
        self.memory_safety_margin_bytes = max(0.0, float(memory_safety_margin_bytes))
        self.train_mfu = train_mfu
        self.recompute_activations = recompute_activations
        self.tp_overlap, self.dp_overlap = tp_overlap, dp_overlap
        self.fused_logprob = fused_logprob
        self.use_profiled_coefficients = use_profiled_coefficients
        self.num_experts, self.top_k = num_experts, top_k

    # ------------------------------------------------------------------ memory
    def act_bytes_per_token_layer(self, tp: int) -> float:
        """bf16 tensors saved for backward per token and layer (packed, no padding)."""
        h = self.d_model
        q = self.n_heads * self.head_dim / tp
        kv = max(1, self.n_kv_heads // tp) * self.head_dim
        ffn = self.ffn / tp * (self.top_k if self.num_experts > 1 else 1)
        elems = 4 * h + 2 * (q + 2 * kv) + 2 * q + 3 * ffn
        return elems * self.dtype_bytes

    def estimate_memory_per_gpu(self, config: TrainParallelConfig, b_micro: int, L: int) -> float:
        tp, pp, dp = config.tp, config.pp, config.dp
        mp = max(tp * pp, 1)
        m_params = 2.0 * self.P / mp
        m_grads = 4.0 * self.P / mp
        m_opt = 12.0 * self.P / (mp * (dp if config.zero_level >= 1 else 1))
        layers = self.n_layers / max(pp, 1)
        tokens = b_micro * L
        if self.recompute_activations:
            m_act = tokens * self.d_model * self.dtype_bytes * layers + tokens * self.act_bytes_per_token_layer(tp)
        else:
            m_act = tokens * self.act_bytes_per_token_layer(tp) * layers
        if self.fused_logprob:
            # bf16 logits of the action rows of one micro-batch, one vocab shard
            m_logits = tokens * self.vocab_size / tp * 2.0
        else:
            m_logits = 0.0
        total = m_params + m_grads + m_opt + m_act + m_logits + self.workspace
        if self.recompute_logprobs and not self.fused_logprob:
            total += estimate_recompute_logprobs_memory(
                batch_size=min(b_micro, self.recompute_micro_batch_size), sequence_length=max(L, self.max_seq_length),
                vocab_size=self.vocab_size, tensor_parallel_size=tp,
                logits_dtype_bytes=self.recompute_logits_dtype_bytes,
                workspace_factor=self.recompute_workspace_factor).total_bytes
        return total

    def check_memory_oom(self, config: TrainParallelConfig, b_micro: int, L: int) -> bool:
        avail = self.mem_capacity * (1.0 - self.mem_frag_rate) - self.memory_safety_margin_bytes
        return self.estimate_memory_per_gpu(config, b_micro, L) > avail

    # ------------------------------------------------------------------ compute
    def layer_flops_fwd(self, tokens: float, L: int) -> float:
        """Linear + causal attention FLOPs of one layer forward for ``tokens`` tokens."""
        linear = 2.0 * (self.P_active - 2.0 * self.vocab_size * self.d_model) / self.n_layers * tokens
        attn = 2.0 * self.n_heads * self.head_dim * tokens * L  # QK^T + PV, causal half of 4*
        return max(linear, 0.0) + attn

    def _profiled_layer_time(self, L: int, b: int, tp: int, bwd: bool) -> float:
        c = self.coef
        tag = "bwd" if bwd else "fwd"
        mlp = (c[f"alpha_mlp_{tag}"] * L + c[f"beta_mlp_{tag}"]) * b / max(tp, 1)
        attn = (c[f"alpha_attn_{tag}"] * L * L + c[f"beta_attn_{tag}"] * L + c[f"gamma_attn_{tag}"]) * b / max(tp, 1)
        return mlp + attn

    def interference(self, t: float, compute_bound: bool, bg_ratio: float) -> float:
        rho = self.rho_compute if compute_bound else self.rho_memory
        return t * (1.0 + rho * bg_ratio ** self.theta)

    def compute_tp_comm(self, tp: int, b_micro: int, L: int) -> float:
        """Per-layer exposed TP traffic (AG + RS of the activations, twice per layer)."""
        if tp <= 1:
            return 0.0
        act = b_micro * L * self.d_model * self.dtype_bytes
        vol = 2.0 * 2.0 * (tp - 1) / tp * act
        return vol / self.bw_intra * (1.0 - self.tp_overlap)

    def compute_ep_comm(self, config: TrainParallelConfig, b_micro: int, L: int) -> float:
        if self.num_experts <= 1 or config.ep <= 1:
            return 0.0
        tokens = b_micro * L
        vol = 2.0 * tokens * self.top_k * self.d_model * self.dtype_bytes * (config.ep - 1) / config.ep
        return vol / self.bw_intra * (1.0 - self.tp_overlap)

    def compute_pp_comm(self, config: TrainParallelConfig, L: int) -> float:
        if config.pp <= 1:
            return 0.0
        bw = self.bw_intra if config.n_gpus <= self.gpus_per_node else self.bw_inter
        return config.b_micro * L * self.d_model * self.dtype_bytes / bw + self.latency_inter

    def compute_dp_comm(self, config: TrainParallelConfig) -> float:
        """Reduce-scatter of fp32 grads + all-gather of bf16 params (distributed optimizer)."""
        if config.dp <= 1:
            return 0.0
        per_rank = self.P / (config.tp * config.pp)
        bw = self.bw_intra if config.n_gpus <= self.gpus_per_node else self.bw_inter
        return (config.dp - 1) / config.dp * per_rank * (4.0 + 2.0) / bw

    def compute_stage_fwd_time(self, L: int, config: TrainParallelConfig) -> float:
        layers = self.n_layers // max(config.pp, 1)
        b = config.b_micro
        if self.use_profiled_coefficients:
            per = self.interference(self._profiled_layer_time(L, b, config.tp, False), True, 0.2 if config.dp > 1 else 0.0)
        else:
            per = self.layer_flops_fwd(b * L, L) / (config.tp * self.flops_peak * self.train_mfu)
        return layers * (per + self.compute_tp_comm(config.tp, b, L) + self.compute_ep_comm(config, b, L))

    def compute_stage_bwd_time(self, L: int, config: TrainParallelConfig) -> float:
        fwd = self.compute_stage_fwd_time(L, config)
        if self.use_profiled_coefficients:
            layers = self.n_layers // max(config.pp, 1)
            bwd = layers * self._profiled_layer_time(L, config.b_micro, config.tp, True)
        else:
            bwd = 2.0 * fwd
        return bwd + (fwd if self.recompute_activations else 0.0)

    def compute_logprob_time(self, L: int, config: TrainParallelConfig, bwd: bool) -> float:
        flops = 2.0 * config.b_micro * L * self.d_model * self.vocab_size / config.tp * (3.0 if bwd else 1.0)
        return flops / (self.flops_peak * self.train_mfu)

    def compute_pipeline_time(self, T_fwd: float, T_bwd: float, n_micro: int, pp: int) -> float:
        if pp <= 1:
            return n_micro * (T_fwd + T_bwd)
        return (pp - 1) * T_fwd + max(0, n_micro - pp + 1) * (T_fwd + T_bwd) + (pp - 1) * T_bwd

    def compute_iteration_time(self, config: TrainParallelConfig, B_global: int, L: int) -> Tuple[float, dict]:
        b_dp = max(1, B_global // config.dp)
        n_micro = max(1, b_dp // config.b_micro)
        t_fwd = self.compute_stage_fwd_time(L, config) + self.compute_logprob_time(L, config, False) / config.pp
        t_bwd = self.compute_stage_bwd_time(L, config) + self.compute_logprob_time(L, config, True) / config.pp
        t_pipe = self.compute_pipeline_time(t_fwd, t_bwd, n_micro, config.pp)
        t_recompute = n_micro * t_fwd if self.recompute_logprobs else 0.0
        t_pp = (config.pp - 1) * self.compute_pp_comm(config, L)
        t_dp = self.compute_dp_comm(config)
        t_opt = 30.0 * self.P / (config.tp * config.pp * config.dp) / self.mem_bw
        t_iter = t_pipe + t_recompute + t_pp + t_dp * (1.0 - self.dp_overlap) + t_opt
        return t_iter, {"t_fwd_per_micro": t_fwd, "t_bwd_per_micro": t_bwd, "t_pipeline": t_pipe,
                        "t_recompute_logprobs": t_recompute, "t_pp_comm": t_pp, "t_dp_comm": t_dp,
                        "t_dp_exposed": t_dp * (1.0 - self.dp_overlap), "t_optimizer": t_opt, "n_micro": n_micro,
                        "b_per_dp": b_dp, "layers_per_pp": self.n_layers // max(config.pp, 1)}


# =============================================================================== combined
class CostModel:
    """Rollout + training cost for a (train config, rollout TP list) candidate."""

    def __init__(self, hardware=None, model_arch=None, profiling=None, *, max_seq_length: int = 2048,
                 recompute_logprobs: bool = True, recompute_micro_batch_size: int = 1,
                 recompute_logits_dtype_bytes: int = 4, recompute_workspace_factor: float = 1.5,
                 memory_safety_margin_bytes: float = 0.0, train_mfu: Optional[float] = None,
                 recompute_activations: bool = False):
        from libra_b200.config import HardwareConfig, ModelArchConfig, ProfilingConfig

        hw = hardware or HardwareConfig()
        ma = model_arch or ModelArchConfig()
        pf = profiling or ProfilingConfig()
        peak = hw.flops_peak_sustained or hw.flops_peak
        bw = hw.hbm_copy_bw or hw.mem_bw
        link = hw.nvlink_peer_bw or hw.bw_intra_node
        self.rollout_model = RolloutCostModel(
            ma.num_params, ma.d_model, ma.n_layers, ma.n_kv_heads, ma.head_dim, ma.dtype_bytes, peak, bw,
            hw.mem_capacity, hw.tp_comm_overhead, pf.prefill_mfu, pf.decode_bw_util, pf.prefill_chunk_size,
            pf.kv_frag_rate, pf.act_workspace_bytes, effective_num_params=ma.effective_num_params, n_heads=ma.n_heads,
            decode_layer_overhead_s=pf.decode_layer_overhead_s, decode_row_layer_s=pf.decode_row_layer_s)
        self.training_model = TrainingCostModel(
            ma.num_params, ma.d_model, ma.n_layers, ma.n_kv_heads, ma.head_dim, ma.dtype_bytes, peak, bw,
            hw.mem_capacity, link, hw.bw_inter_node, hw.gpus_per_node, hw.latency_inter_node,
            pf.alpha_mlp_fwd, pf.beta_mlp_fwd, pf.alpha_mlp_bwd, pf.beta_mlp_bwd, pf.alpha_attn_fwd,
            pf.beta_attn_fwd, pf.gamma_attn_fwd, pf.alpha_attn_bwd, pf.beta_attn_bwd, pf.gamma_attn_bwd,
            pf.rho_compute_bound, pf.rho_memory_bound, pf.theta_slowdown, pf.train_mem_frag_rate,
            pf.train_workspace_bytes, effective_num_params=ma.effective_num_params, vocab_size=ma.vocab_size,
            max_seq_length=max_seq_length, recompute_logprobs=recompute_logprobs,
            recompute_micro_batch_size=recompute_micro_batch_size,
            recompute_logits_dtype_bytes=recompute_logits_dtype_bytes,
            recompute_workspace_factor=recompute_workspace_factor,
            memory_safety_margin_bytes=memory_safety_margin_bytes, n_heads=ma.n_heads,
            intermediate_size=(ma.expert_intermediate_size if ma.is_moe else ma.intermediate_size),
            train_mfu=train_mfu if train_mfu is not None else pf.prefill_mfu,
            recompute_activations=recompute_activations,
            num_experts=ma.num_experts if ma.is_moe else 1, top_k=ma.num_activated_experts if ma.is_moe else 1)
        self.hw, self.ma, self.prof = hw, ma, pf

    def evaluate_rollout(self, cluster: RolloutClusterConfig, requests: List[RequestInfo]) -> Tuple[float, dict]:
        return self.rollout_model.evaluate_cluster(cluster, requests)

    def evaluate_training(self, config: TrainParallelConfig, B_global: int, L: int) -> Tuple[float, dict]:
        return self.training_model.compute_iteration_time(config, B_global, L)

    def check_train_oom(self, config: TrainParallelConfig, B_global: int, L: int) -> bool:
        return self.training_model.check_memory_oom(config, config.b_micro, L)

    def evaluate(self, train_config: TrainParallelConfig, rollout_cluster: RolloutClusterConfig,
                 requests: List[RequestInfo], B_global: int = 32) -> CostModelResult:
        res = CostModelResult()
        L = int(_mean(r.total_length for r in requests)) if requests else 1024
        if self.check_train_oom(train_config, B_global, L):
            res.is_oom, res.oom_source = True, "train"
            res.t_train = res.t_rollout = res.t_global = float("inf")
            res.details["train_oom"] = True
            res.details["train_mem_per_gpu"] = self.training_model.estimate_memory_per_gpu(
                train_config, train_config.b_micro, L)
            return res
        res.t_train, res.details["training"] = self.evaluate_training(train_config, B_global, L)
        res.t_rollout, res.details["rollout"] = self.evaluate_rollout(rollout_cluster, requests)
        if math.isinf(res.t_rollout):
            res.is_oom, res.oom_source, res.t_global = True, "rollout", float("inf")
            return res
        res.t_global = max(res.t_train, res.t_rollout)
        res.details.update({"t_train": res.t_train, "t_rollout": res.t_rollout,
                            "train_config": {"tp": train_config.tp, "pp": train_config.pp, "dp": train_config.dp,
                                             "b_micro": train_config.b_micro},
                            "rollout_config": rollout_cluster.tp_list})
        return res
