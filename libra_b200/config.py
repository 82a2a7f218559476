"""Configuration schema for libra_b200.

The key names, nesting and defaults of every section below are kept identical to
the reference's schema (``config.py:130-737`` in NetX-lab/Libra) so that an
experiment YAML written for the reference loads here unchanged.  The loader
itself is a fresh design:

* ``ConfigSection`` gives every dataclass section ``from_dict``/``from_file`` with
  one numeric-string coercion rule (``_coerce_scalar``).
* YAML composition (``base_config`` / ``hardware_config`` / ``model_arch_config``,
  reference ``config.py:76-115``) is done by ``compose_config_dict``.
* Topology validation (reference ``config.py:739-937``) lives in
  ``AsyncRLConfig._validate_topology`` / ``_validate_weight_sync`` /
  ``_validate_backend`` so each rule group can be read and tested on its own.

B200 additions (not in the reference) are additive keys with defaults that keep
reference behaviour: ``hardware.hbm_copy_bw`` (measured copy bandwidth) and
``hardware.flops_peak_sustained``.
"""

from __future__ import annotations

import copy
import dataclasses
import json
import os
from dataclasses import dataclass, field, fields
from typing import Any, Optional

COMPOSE_KEYS = ("base_config", "hardware_config", "model_arch_config")


# ---------------------------------------------------------------------------
# generic helpers
# ---------------------------------------------------------------------------

def _coerce_scalar(value: Any) -> Any:
    """Turn numeric strings ("1e-6", "8") into numbers; leave everything else.

    YAML 1.1 reads ``1e-6`` as a string, so the coercion matters for learning
    rates and bandwidth figures.  Integers stay integers only when written
    without a dot or exponent.
    """
    if not isinstance(value, str):
        return value
    text = value.strip()
    try:
        number = float(text)
    except (ValueError, OverflowError):
        return value
    if number.is_integer() and not any(c in text.lower() for c in ".e"):
        return int(number)
    return number


def merge_dicts(base: dict, override: dict) -> dict:
    """Recursive dict merge; ``override`` wins, nested dicts are merged."""
    out = copy.deepcopy(base)
    for key, value in override.items():
        if isinstance(value, dict) and isinstance(out.get(key), dict):
            out[key] = merge_dicts(out[key], value)
        else:
            out[key] = copy.deepcopy(value)
    return out


def read_config_file(path: str) -> dict:
    """Read a .yaml/.yml/.json file into a dict."""
    if not os.path.isfile(path):
        raise FileNotFoundError(f"config file not found: {path}")
    suffix = os.path.splitext(path)[1].lower()
    with open(path, "r", encoding="utf-8") as handle:
        if suffix in (".yaml", ".yml"):
            import yaml

            return yaml.safe_load(handle) or {}
        if suffix == ".json":
            return json.load(handle)
    raise ValueError(f"cannot read a {suffix or 'suffix-less'} config file ({path}): expected YAML or JSON")


def _abs_from(path: str, directory: str) -> str:
    return path if os.path.isabs(path) else os.path.normpath(os.path.join(directory, path))


def compose_config_dict(raw: dict, directory: str, visited: Optional[set] = None) -> dict:
    """Resolve ``base_config`` inheritance and the hardware/model include files.

    Order of precedence (lowest first): the base chain, the hardware include
    (merged under ``hardware``), the model include (under ``model_arch``), then
    the file's own keys.
    """
    visited = set() if visited is None else visited
    result: dict = {}
    base = raw.get("base_config")
    if base is not None:
        base_path = _abs_from(base, directory)
        if base_path in visited:
            raise ValueError(f"base_config chain loops back to {base_path} (cyclic config inheritance)")
        visited.add(base_path)
        result = compose_config_dict(read_config_file(base_path), os.path.dirname(base_path), visited)
    for include_key, section in (("hardware_config", "hardware"), ("model_arch_config", "model_arch")):
        include = raw.get(include_key)
        if include is not None:
            included = read_config_file(_abs_from(include, directory))
            result[section] = merge_dicts(result.get(section, {}), included)
    own = {k: v for k, v in raw.items() if k not in COMPOSE_KEYS}
    return merge_dicts(result, own)


class ConfigSection:
    """Mixin: dict/file constructors that ignore unknown keys and coerce numbers."""

    @classmethod
    def from_dict(cls, data: Optional[dict]):
        if not data:
            return cls()
        known = {f.name for f in fields(cls)}
        kwargs = {k: _coerce_scalar(v) for k, v in data.items() if k in known}
        return cls(**kwargs)

    @classmethod
    def from_file(cls, path: str):
        return cls.from_dict(read_config_file(path))


# ---------------------------------------------------------------------------
# sections
# ---------------------------------------------------------------------------

@dataclass
class HardwareConfig(ConfigSection):
    """Per-GPU hardware figures used by the cost model (reference ``config.py:130``)."""

    flops_peak: float = 312e12
    mem_bw: float = 2.0e12
    mem_capacity: float = 80e9
    bw_intra_node: float = 400e9
    bw_inter_node: float = 200e9
    gpus_per_node: int = 8
    tp_comm_overhead: float = 5e-6
    latency_inter_node: float = 5e-6
    # B200 additions: measured sustained GEMM rate and plain copy bandwidth.
    flops_peak_sustained: float = 0.0
    hbm_copy_bw: float = 0.0
    nvlink_peer_bw: float = 0.0


@dataclass
class ModelArchConfig(ConfigSection):
    """Architecture summary used by the planner (reference ``config.py:154``)."""

    num_params: float = 3e9
    d_model: int = 2048
    n_layers: int = 36
    n_heads: int = 16
    n_kv_heads: int = 2
    vocab_size: int = 151936
    intermediate_size: int = 11008
    dtype_bytes: int = 2
    head_dim: int = 0
    is_moe: bool = False
    active_num_params: float = 0.0
    num_experts: int = 1
    num_shared_experts: int = 0
    num_activated_experts: int = 1
    expert_intermediate_size: int = 0
    shared_expert_intermediate_size: int = 0

    def __post_init__(self):
        if self.head_dim <= 0:
            self.head_dim = self.d_model // max(self.n_heads, 1)
        if self.expert_intermediate_size <= 0:
            self.expert_intermediate_size = self.intermediate_size

    @property
    def activated_expert_ratio(self) -> float:
        if not self.is_moe or self.num_experts <= 1:
            return 1.0
        return min(1.0, self.num_activated_experts / max(self.num_experts, 1))

    @property
    def effective_num_params(self) -> float:
        if not self.is_moe:
            return self.num_params
        if self.active_num_params > 0:
            return self.active_num_params
        return self.num_params * self.activated_expert_ratio


@dataclass
class ProfilingConfig(ConfigSection):
    """Profiled alpha/beta/gamma op-time coefficients (reference ``config.py:213``)."""

    alpha_mlp_fwd: float = 3.5e-8
    beta_mlp_fwd: float = 1.0e-5
    alpha_mlp_bwd: float = 7.0e-8
    beta_mlp_bwd: float = 2.0e-5
    alpha_attn_fwd: float = 1.5e-12
    beta_attn_fwd: float = 2.5e-8
    gamma_attn_fwd: float = 8.0e-6
    alpha_attn_bwd: float = 3.0e-12
    beta_attn_bwd: float = 5.0e-8
    gamma_attn_bwd: float = 1.5e-5
    rho_compute_bound: float = 0.08
    rho_memory_bound: float = 0.45
    theta_slowdown: float = 1.0
    prefill_mfu: float = 0.55
    decode_bw_util: float = 0.85
    # B200 additions (0 keeps the reference's steady-batch rollout model): fixed latency of one decode
    # step per layer (kernel chain, pipeline fill) and the extra time per running sequence per layer;
    # when either is set, an instance's makespan is simulated step by step (continuous batching, the
    # batch shrinking as sequences finish) instead of assuming a full steady batch
    decode_layer_overhead_s: float = 0.0
    decode_row_layer_s: float = 0.0
    prefill_chunk_size: int = 1024
    kv_frag_rate: float = 0.04
    act_workspace_bytes: float = 1.0e9
    train_mem_frag_rate: float = 0.08
    train_workspace_bytes: float = 0.5e9


@dataclass
class HeterogeneousInstanceConfig(ConfigSection):
    """One rollout instance (a TP bucket member)."""

    instance_id: str = ""
    tp: int = 1
    gpus: list = field(default_factory=list)
    description: str = ""
    host: str = ""
    port: int = 0


def _default_length_thresholds() -> dict:
    return {"short": 5000, "medium": 10000, "long": 15000}


def _default_routing_rules() -> dict:
    return {"short": [1, 2], "medium": [2, 4], "long": [4, 8], "extra_long": [8, 4]}


def _default_two_buckets() -> dict:
    return {
        "short": {"tp_degrees": [1, 2], "max_tokens": 5000},
        "long": {"tp_degrees": [4, 8], "max_tokens": 50000},
    }


@dataclass
class SchedulingConfig(ConfigSection):
    """Rollout scheduler options (reference ``config.py:280``)."""

    scheduler_type: str = "length_aware"
    length_thresholds: dict = field(default_factory=_default_length_thresholds)
    routing_rules: dict = field(default_factory=_default_routing_rules)
    load_balance_strategy: str = "least_connections"
    max_queue_length: int = 100
    enable_fallback: bool = True
    adaptive_routing: bool = True
    request_timeout: float = 600.0
    la_mlfq_buckets: dict = field(default_factory=_default_two_buckets)
    la_mlfq_migration_threshold: int = 3000
    la_mlfq_scout_timeout: float = 30.0
    la_mlfq_history_ttl: int = 5
    cmlfq_buckets: dict = field(default_factory=_default_two_buckets)
    cmlfq_rebuild_interval: int = 50
    cmlfq_migration_profile_path: str = ""
    cmlfq_tree_path: str = ""
    cmlfq_tree_persist_interval: int = 1
    cmlfq_shared_load_dir: str = ""
    cmlfq_shared_load_ttl_s: float = 60.0
    cmlfq_shared_load_heartbeat_s: float = 10.0
    cmlfq_payload_small_threshold: int = 500
    cmlfq_payload_large_threshold: int = 5000


@dataclass
class HeterogeneousRolloutConfig(ConfigSection):
    """Heterogeneous TP-bucket rollout cluster (reference ``config.py:353``)."""

    enabled: bool = False
    total_gpus: int = 0
    available_gpus: list = field(default_factory=list)
    instances: list = field(default_factory=list)
    scheduling: SchedulingConfig = field(default_factory=SchedulingConfig)
    vllm_base_port: int = 8000
    vllm_host: str = "127.0.0.1"
    startup_timeout: int = 300
    max_model_len: int = 0
    gpu_memory_utilization: float = 0.90
    enable_thinking: bool = False

    def __post_init__(self):
        self.instances = [
            inst if isinstance(inst, HeterogeneousInstanceConfig)
            else HeterogeneousInstanceConfig.from_dict(
                dict(inst, gpus=list(inst.get("gpus", []))) if isinstance(inst, dict) else {}
            )
            for inst in self.instances
        ]
        if isinstance(self.scheduling, dict):
            self.scheduling = SchedulingConfig.from_dict(self.scheduling)
        if self.total_gpus <= 0 and self.instances:
            self.total_gpus = sum(inst.tp for inst in self.instances)
        for index, inst in enumerate(self.instances):
            if not inst.instance_id:
                inst.instance_id = f"hetero_tp{inst.tp}_{index}"

    @property
    def n_instances(self) -> int:
        return len(self.instances)

    @property
    def tp_list(self) -> list:
        return [inst.tp for inst in self.instances]

    @classmethod
    def from_dict(cls, data: Optional[dict]):
        if not data:
            return cls()
        data = dict(data)
        gpu_block = data.pop("gpu", None)
        if isinstance(gpu_block, dict):
            for key in ("total_gpus", "available_gpus"):
                if key in gpu_block:
                    data.setdefault(key, gpu_block[key])
        return super().from_dict(data)


@dataclass
class GlobalResourcePlannerConfig(ConfigSection):
    """Global Resource Planner + elastic executor options (reference ``config.py:436``)."""

    enabled: bool = False
    train_backend: str = "analytic"
    rollout_backend: str = "analytic"
    plan_interval: int = 10
    warmup_steps: int = 1
    min_history_size: int = 8
    min_gain_ratio: float = 0.05
    reconfiguration_cost_s: float = 15.0
    max_history_size: int = 4096
    allowed_rollout_tp: list = field(default_factory=lambda: [1, 2, 4, 8])
    rollout_node_tp_pattern: list = field(default_factory=list)
    require_heterogeneous_rollout_tp: bool = False
    allowed_train_tp: list = field(default_factory=list)
    allowed_train_pp: list = field(default_factory=list)
    fixed_train_gpus: int = 0
    initial_allocation_strategy: str = "grp"
    initial_allocation_applied: bool = False
    allocation_granularity_gpus: int = 1
    min_train_gpus: int = 1
    min_rollout_gpus: int = 1
    micro_batch_sizes: list = field(default_factory=list)
    startup_profile_enabled: bool = True
    startup_profile_sample_size: int = 64
    startup_profile_strategy: str = "spread"
    startup_profile_seed: int = 0
    startup_profile_samples_per_prompt: int = 1
    startup_profile_dataset_jsonl: str = ""
    startup_profile_history_jsonl: str = ""
    startup_profile_summary_json: str = ""
    startup_profile_reuse_existing: bool = True
    startup_profile_allow_synthetic_fallback: bool = False
    memory_budget_check_enabled: bool = True
    memory_budget_dry_run_enabled: bool = True
    memory_budget_safety_margin_bytes: float = 2.0e9
    memory_budget_logits_dtype_bytes: int = 4
    memory_budget_workspace_factor: float = 1.5
    apply_to_runtime: bool = True
    verbose: bool = False
    runtime_length_profile_enabled: bool = True
    runtime_length_profile_jsonl: str = ""
    runtime_async_planning: bool = True
    runtime_max_pending_plans: int = 1
    runtime_dynamic_reconfiguration_enabled: bool = True
    runtime_online_replanning: bool = True
    runtime_replan_cooldown_steps: int = 1
    runtime_queue_pressure_threshold: float = 0.75
    runtime_active_rollout_pressure_threshold: float = 0.85
    runtime_rejected_rollout_delta_threshold: int = 8
    runtime_rollout_train_imbalance_threshold: float = 1.25
    simulator_allow_fallback: bool = True
    simulator_timeout_s: float = 120.0
    simulator_cache_dir: str = "./logs/global_resource_planner/simulator_cache"
    sailor_path: str = "../sailor"
    sailor_python: str = "python"
    sailor_train_command: str = ""
    vidur_path: str = "../vidur"
    vidur_python: str = "python"
    vidur_rollout_command: str = ""
    vidur_model_name: str = "meta-llama/Meta-Llama-3-8B"
    vidur_device: str = "a100"
    vidur_qps: float = 1000000.0
    vidur_scheduler: str = "sarathi"
    vidur_batch_size_cap: int = 512
    vidur_chunk_size: int = 512
    vidur_time_limit_s: float = 0.0
    runtime_manage_rollout_processes: bool = False
    runtime_adopt_existing_rollout_processes: bool = True
    runtime_drain_before_reconfigure: bool = True
    runtime_drain_timeout_s: float = 3600.0
    runtime_rollout_reconfigure_strategy: str = "diff"
    runtime_cluster_swap_enabled: bool = False
    runtime_prewarm_no_spare_fallback_strategy: str = "restart_all"
    runtime_rollout_log_dir: str = ""
    runtime_rollout_manifest_path: str = ""
    runtime_rollout_pid_registry_path: str = ""
    runtime_wait_rollout_process_start_ready: bool = False
    runtime_post_rollout_stop_grace_s: float = 0.0
    runtime_reconfigure_training: bool = False
    runtime_training_pool_only: bool = True
    runtime_training_pool_target_gpus: int = 0
    runtime_training_pool_plan_only: bool = True
    runtime_batch_collection_timeout_s: float = 0.0
    runtime_batch_collection_max_retries: int = 0
    runtime_use_nccl_barrier_after_rollout: bool = False
    runtime_use_nccl_barrier_before_weight_sync: bool = False
    runtime_coordinate_reconfiguration_ranks: bool = True
    runtime_coordinate_batch_source_only: bool = True
    runtime_peer_request_wait_s: float = 45.0
    vllm_launch_command_template: str = ""
    vllm_stop_command_template: str = ""
    vllm_ready_timeout_s: float = 300.0
    vllm_stop_timeout_s: float = 30.0
    hybrid_worker_launch_enabled: bool = False
    hybrid_training_prewarm_enabled: bool = False
    hybrid_training_prewarm_count: int = 0
    hybrid_training_prewarm_worker_ids: list = field(default_factory=list)
    hybrid_worker_python: str = "python"
    hybrid_worker_command_template: str = ""
    hybrid_worker_task_dir: str = "./logs/elastic_training_tasks"
    hybrid_worker_ready_timeout_s: float = 60.0
    hybrid_worker_remote_control_enabled: bool = False
    hybrid_worker_remote_control_dir: str = ""
    elastic_hybrid_planning_enabled: bool = False
    elastic_hybrid_require_planner_signal: bool = False
    elastic_hybrid_max_workers: int = 0
    elastic_hybrid_replica_size_gpus: int = 0
    elastic_hybrid_min_rollout_gpus: int = 0
    elastic_hybrid_borrow_train_rollout_ratio: float = 1.15
    elastic_hybrid_release_train_rollout_ratio: float = 0.90
    elastic_hybrid_max_rollout_pressure: float = 0.80
    elastic_hybrid_join_timeout_s: float = 180.0
    elastic_hybrid_signal_ttl_steps: int = 20
    elastic_hybrid_require_isolated_ccl: bool = False
    gradient_transport_backend: str = "tcp"
    decouple_communication_domains: bool = True
    gradient_server_host: str = "127.0.0.1"
    gradient_server_public_host: str = ""
    gradient_server_port: int = 0
    gradient_server_authkey: str = "rl-framework-elastic"
    native_rdma_device: str = "mlx5_0"
    native_rdma_gid_index: int = 0
    native_rdma_ib_port: int = 1
    native_rdma_max_bytes: int = 67108864
    hybrid_worker_mode: str = "megatron_core"
    hybrid_worker_config_path: str = ""
    hybrid_worker_endpoint_dir: str = ""
    hybrid_lockstep_gradient_sync: bool = True
    hybrid_active_gradient_timeout_s: float = 300.0
    hybrid_update_timeout_s: float = 300.0


_NESTED_SECTIONS = {
    "hardware": HardwareConfig,
    "model_arch": ModelArchConfig,
    "profiling": ProfilingConfig,
    "heterogeneous_rollout": HeterogeneousRolloutConfig,
    "global_resource_planner": GlobalResourcePlannerConfig,
}

TRAIN_BACKENDS = ("fsdp", "megatron3d", "megatron_core")


@dataclass
class AsyncRLConfig:
    """Top-level experiment configuration (reference ``config.py:593``).

    ``train_backend`` keeps the reference's three names.  In this framework all
    three select the native B200 engine (``libra_b200.engine.train_engine``);
    the name only changes which reference rules are validated, so reference
    YAML files keep passing or failing exactly as they did.
    """

    model_path: str
    tokenizer_path: str = ""
    rollout_backend: str = "vllm"
    train_gpus: int = 4
    rollout_gpus: int = 4
    rollout_gpu_ids: str = ""
    tp_size: int = 1
    vllm_tp_size: int = 1
    train_backend: str = "megatron_core"
    train_tp_size: int = 0
    train_pp_size: int = 1
    train_dp_size: int = 0
    train_cp_size: int = 1
    train_ep_size: int = 1
    expert_tensor_parallel_size: int = 1
    pipeline_schedule: str = "1f1b"
    virtual_pipeline_model_parallel_size: int = 0
    sequence_parallel: bool = True
    use_distributed_optimizer: bool = True
    megatron_grad_reduce_in_fp32: bool = False
    megatron_use_precision_aware_optimizer: bool = False
    megatron_optimizer_cpu_offload: bool = False
    megatron_optimizer_offload_fraction: float = 0.0
    megatron_optimizer_pin_cpu_grads: bool = True
    megatron_optimizer_pin_cpu_params: bool = True
    megatron_checkpoint_format: str = "torch_dist"
    megatron_fully_parallel_save: bool = True
    megatron_async_save: bool = False
    megatron_streaming_export: bool = True
    megatron_use_transformer_engine: bool = False
    megatron_use_cpu_initialization: bool = False
    megatron_recompute_num_layers: int = 1
    max_concurrent_rollouts: int = 64
    max_head_offpolicyness: int = 4
    queue_size: int = 256
    enable_rollout_tracing: bool = False
    sync_interval: int = 1
    recompute_logprobs: bool = True
    recompute_micro_batch_size: int = 1
    phase_trace_enabled: bool = False
    phase_trace_dir: str = ""
    weight_sync_mode: str = "disk"
    sync_path: str = "./logs/async_rl_weights"
    rollout_weight_sync_mode: str = "none"
    rollout_weight_sync_control_dir: str = ""
    rollout_weight_sync_timeout_s: float = 1200.0
    rollout_weight_sync_export_only: bool = True
    rollout_weight_reload_method: str = "restart"
    rollout_weight_reload_strategy: str = "parallel"
    rollout_nccl_host: str = ""
    rollout_nccl_port: int = 29620
    rollout_nccl_chunk_mb: int = 256
    rollout_nccl_rate_limit_gbps: float = 0.0
    rollout_weight_sync_poll_interval_s: float = 0.05
    require_rollout_weight_sync: bool = False
    learning_rate: float = 1e-6
    ppo_epochs: int = 1
    batch_size: int = 32
    micro_batch_size: int = 4
    kl_coef: float = 0.001
    clip_epsilon: float = 0.2
    gamma: float = 1.0
    max_new_tokens: int = 1024
    r2e_max_turns: int = 3
    r2e_max_prompt_tokens: int = 0
    r2e_stop_reward: float = 0.5
    n_samples: int = 4
    temperature: float = 1.0
    top_p: float = 1.0
    dataset_name: str = "openai/gsm8k"
    dataset_split: str = "train"
    max_seq_length: int = 2048
    total_steps: int = 100
    eval_interval: int = 10
    save_interval: int = 10
    seed: int = 42
    ray_address: str = "auto"
    vllm_host: str = "127.0.0.1"
    vllm_port: int = 8000
    vllm_num_instances: int = 0
    vllm_endpoints: str = ""
    num_nodes: int = 1
    gpus_per_node_override: int = 0
    train_gpus_per_node: int = 0
    rollout_gpus_per_node: int = 0
    master_addr: str = ""
    master_port: int = 29500
    log_dir: str = "./logs"
    wandb_project: str = "RL_Framework"
    wandb_run_name: str = "run1"
    keep_latest_checkpoints: int = 5
    enable_history_collection: bool = False
    history_output_dir: str = ""
    history_save_raw_lengths: bool = False
    history_flush_interval: int = 10
    history_experiment_name: str = ""
    hardware: HardwareConfig = field(default_factory=HardwareConfig)
    model_arch: ModelArchConfig = field(default_factory=ModelArchConfig)
    profiling: ProfilingConfig = field(default_factory=ProfilingConfig)
    n_total_gpus: int = 0
    heterogeneous_rollout: HeterogeneousRolloutConfig = field(default_factory=HeterogeneousRolloutConfig)
    global_resource_planner: GlobalResourcePlannerConfig = field(default_factory=GlobalResourcePlannerConfig)

    # -- validation ---------------------------------------------------------

    def __post_init__(self):
        for name, section_cls in _NESTED_SECTIONS.items():
            value = getattr(self, name)
            if isinstance(value, dict):
                setattr(self, name, section_cls.from_dict(value))
        if not self.tokenizer_path:
            self.tokenizer_path = self.model_path
        if not 0.0 <= self.r2e_stop_reward <= 1.0:
            raise ValueError("r2e_stop_reward must be between 0 and 1")
        self._validate_topology()
        self._validate_weight_sync()
        self._validate_backend()
        self._fill_derived()

    def _model_parallel_width(self) -> int:
        width = self.train_tp_size * self.train_pp_size
        if self.train_backend == "megatron_core":
            width *= self.train_cp_size
        return width

    def _validate_topology(self) -> None:
        if self.train_tp_size <= 0:
            self.train_tp_size = max(1, self.tp_size)
        else:
            self.tp_size = self.train_tp_size
        if self.train_pp_size <= 0:
            raise ValueError("train_pp_size must be greater than zero")
        if self.train_dp_size <= 0:
            width = self._model_parallel_width()
            if self.train_gpus % width:
                raise ValueError(
                    "train_gpus must be divisible by the configured model-parallel size: "
                    f"train_gpus={self.train_gpus}, model_parallel={width}"
                )
            self.train_dp_size = self.train_gpus // width
        if self.train_backend not in TRAIN_BACKENDS:
            raise ValueError("train_backend must be 'fsdp', 'megatron3d', or 'megatron_core'")
        if self.train_gpus <= 0:
            raise ValueError("train_gpus must be greater than zero")
        if self.pipeline_schedule != "1f1b":
            raise ValueError("pipeline_schedule currently supports only '1f1b'")
        if self.virtual_pipeline_model_parallel_size != 0:
            raise ValueError("virtual_pipeline_model_parallel_size currently supports only 0")
        topology = self._model_parallel_width() * self.train_dp_size
        if topology != self.train_gpus:
            raise ValueError(
                "The training topology must match train_gpus: "
                f"topology_size={topology}, train_gpus={self.train_gpus}"
            )
        if self.batch_size % (self.train_dp_size * self.micro_batch_size):
            raise ValueError(
                "batch_size must be divisible by train_dp_size * micro_batch_size: "
                f"{self.batch_size} vs {self.train_dp_size}*{self.micro_batch_size}"
            )

    def _validate_weight_sync(self) -> None:
        choices = {
            "weight_sync_mode": ("disk", "nccl"),
            "rollout_weight_sync_mode": ("none", "restart", "nccl"),
            "rollout_weight_reload_method": ("restart", "inplace"),
            "rollout_weight_reload_strategy": ("parallel", "serial"),
        }
        for key, allowed in choices.items():
            if getattr(self, key) not in allowed:
                quoted = ", ".join(f"'{a}'" for a in allowed[:-1]) + f", or '{allowed[-1]}'"
                if len(allowed) == 2:
                    quoted = f"'{allowed[0]}' or '{allowed[1]}'"
                raise ValueError(f"{key} must be {quoted}")
        if self.rollout_weight_sync_mode != "nccl":
            return
        if self.train_backend != "megatron_core":
            raise ValueError("NCCL rollout sync requires train_backend='megatron_core'")
        if self.weight_sync_mode != "nccl":
            raise ValueError("NCCL rollout sync requires weight_sync_mode='nccl'")
        if self.rollout_weight_reload_strategy != "parallel":
            raise ValueError("NCCL rollout reload requires parallel strategy")
        if self.rollout_nccl_chunk_mb <= 0:
            raise ValueError("rollout_nccl_chunk_mb must be greater than zero")
        if self.rollout_nccl_rate_limit_gbps < 0:
            raise ValueError("rollout_nccl_rate_limit_gbps cannot be negative")
        if self.rollout_weight_sync_poll_interval_s <= 0:
            raise ValueError("rollout_weight_sync_poll_interval_s must be greater than zero")

    def _engine_constraints(self):
        """(holds, message) pairs: what the native training engine can run.

        Every ``train_backend`` value selects the same engine, so the rules
        are the engine's: tensor parallelism must divide the heads, the FFN
        and the vocabulary; experts are spread over expert-parallel ranks
        inside the data-parallel group; pipeline stages (with TP=1, EP=1) hold
        contiguous layer ranges; one context shard per rank; checkpoints in
        the ``torch_dist`` layout."""
        arch = self.model_arch
        tp, ep = self.train_tp_size, self.train_ep_size
        heads, kv = arch.n_heads, arch.n_kv_heads
        yield (self.train_pp_size == 1 or (tp == 1 and ep == 1),
               f"train_pp_size={self.train_pp_size}: pipeline stages run with train_tp_size=1 and train_ep_size=1")
        yield (self.train_pp_size <= arch.n_layers,
               f"train_pp_size={self.train_pp_size} exceeds the model's {arch.n_layers} layers")
        yield (self.train_cp_size == 1,
               f"train_cp_size={self.train_cp_size}: sequences are not split across ranks; long contexts run as "
               "packed variable-length attention on one rank")
        yield (heads % tp == 0 and (kv % tp == 0 or tp % kv == 0),
               f"train_tp_size={tp} must divide num_attention_heads={heads} and divide or be a multiple of "
               f"num_key_value_heads={kv}")
        yield (arch.intermediate_size % tp == 0 and arch.vocab_size % tp == 0,
               f"train_tp_size={tp} must divide intermediate_size={arch.intermediate_size} and "
               f"vocab_size={arch.vocab_size}")
        yield ep >= 1 and self.expert_tensor_parallel_size >= 1, "train_ep_size and expert_tensor_parallel_size must be >= 1"
        yield (self.expert_tensor_parallel_size == 1,
               f"expert_tensor_parallel_size={self.expert_tensor_parallel_size}: each expert lives whole on one "
               "expert-parallel rank")
        if ep > 1:
            yield arch.num_experts > 1, f"train_ep_size={ep} needs a mixture-of-experts model (num_experts > 1)"
            yield (arch.num_experts % ep == 0,
                   f"num_experts={arch.num_experts} must split evenly over train_ep_size={ep}")
            yield (self.train_dp_size % ep == 0,
                   f"train_ep_size={ep} must divide the data-parallel size {self.train_dp_size} (experts are "
                   "exchanged inside the data-parallel group)")
        yield (0.0 <= self.megatron_optimizer_offload_fraction <= 1.0,
               "megatron_optimizer_offload_fraction must lie in [0, 1]")
        yield (self.megatron_optimizer_offload_fraction == 0.0 or self.megatron_optimizer_cpu_offload,
               "megatron_optimizer_offload_fraction > 0 moves part of the optimizer state to the host: it needs "
               "megatron_optimizer_cpu_offload=true")
        yield (self.megatron_checkpoint_format == "torch_dist",
               f"megatron_checkpoint_format={self.megatron_checkpoint_format!r}: checkpoints are written as "
               "torch_dist (DCP) directories")
        yield (not (self.weight_sync_mode == "nccl" and self.rollout_weight_sync_mode not in ("nccl", "none")),
               "weight_sync_mode='nccl' pushes weights straight into the rollout engines; pair it with "
               "rollout_weight_sync_mode='nccl'")

    def _validate_backend(self) -> None:
        for holds, message in self._engine_constraints():
            if not holds:
                raise ValueError(message)

    def _fill_derived(self) -> None:
        for directory in (self.sync_path, self.log_dir):
            try:
                os.makedirs(directory, exist_ok=True)
            except OSError:
                # Shared paths may exist only on the launch node; components
                # create their own directories when they first write.
                pass
        if self.n_total_gpus <= 0:
            self.n_total_gpus = self.train_gpus + self.rollout_gpus
        if self.num_nodes > 1:
            if self.train_gpus_per_node <= 0:
                self.train_gpus_per_node = self.train_gpus // self.num_nodes
            if self.rollout_gpus_per_node <= 0:
                self.rollout_gpus_per_node = self.rollout_gpus // self.num_nodes
        if not self.master_addr:
            self.master_addr = _first_slurm_host() or "localhost"

    # -- construction -------------------------------------------------------

    @classmethod
    def from_dict(cls, data: dict) -> "AsyncRLConfig":
        data = dict(data)
        sections = {name: data.pop(name, None) for name in _NESTED_SECTIONS}
        known = {f.name for f in fields(cls)} - set(_NESTED_SECTIONS)
        kwargs = {k: _coerce_scalar(v) for k, v in data.items() if k in known}
        for name, section_cls in _NESTED_SECTIONS.items():
            kwargs[name] = section_cls.from_dict(sections[name])
        return cls(**kwargs)

    @classmethod
    def from_file(cls, path: str) -> "AsyncRLConfig":
        raw = read_config_file(path)
        return cls.from_dict(compose_config_dict(raw, os.path.dirname(os.path.abspath(path))))

    from_yaml = from_file
    from_json = from_file

    def to_dict(self) -> dict:
        return dataclasses.asdict(self)

    def to_yaml(self, path: str) -> None:
        import yaml

        os.makedirs(os.path.dirname(path) or ".", exist_ok=True)
        with open(path, "w", encoding="utf-8") as handle:
            yaml.dump(self.to_dict(), handle, default_flow_style=False, allow_unicode=True)

    def to_json(self, path: str) -> None:
        os.makedirs(os.path.dirname(path) or ".", exist_ok=True)
        with open(path, "w", encoding="utf-8") as handle:
            json.dump(self.to_dict(), handle, indent=2, ensure_ascii=False)


def _first_slurm_host() -> str:
    nodelist = os.environ.get("SLURM_NODELIST", "")
    if not nodelist:
        return ""
    import subprocess

    try:
        out = subprocess.run(
            ["scontrol", "show", "hostnames", nodelist], capture_output=True, text=True, check=True
        ).stdout.split()
        return out[0] if out else "localhost"
    except Exception:
        return "localhost"


def load_config(config_path: Optional[str] = None) -> AsyncRLConfig:
    """Load from an explicit path or ``$ASYNC_RL_CONFIG``."""
    path = config_path or os.environ.get("ASYNC_RL_CONFIG")
    if not path:
        raise ValueError("no config given: pass a path to load_config(), --config on the command line, or set "
                         "ASYNC_RL_CONFIG")
    return AsyncRLConfig.from_file(path)


def parse_args_and_load_config() -> AsyncRLConfig:
    import argparse

    parser = argparse.ArgumentParser(description="Asynchronous RL training")
    parser.add_argument("--config", type=str, default=None,
                        help="Configuration file path (.yaml/.yml/.json). Defaults to ASYNC_RL_CONFIG.")
    args, _ = parser.parse_known_args()
    return load_config(args.config)


@dataclass
class ResourceConfig:
    """Legacy rollout resource knobs (reference ``config.py:1055``)."""

    max_concurrent_requests: int = 32
    batch_size: int = 32
    gpu_allocation: int = 4
    target_rollout_time: float = 30.0


@dataclass
class GenerationConfig:
    """Sampling parameters for one generate call."""

    max_new_tokens: int = 1024
    temperature: float = 1.0
    top_p: float = 1.0
    top_k: int = -1
    do_sample: bool = True
    stop_token_ids: list = field(default_factory=list)
