import os

import pytest

from libra_b200.config import AsyncRLConfig, compose_config_dict, load_config, merge_dicts

CFG_DIR = os.path.join(os.path.dirname(os.path.dirname(__file__)), "libra_b200", "configs")


def test_presets_load(tmp_path):
    cfg = AsyncRLConfig.from_file(os.path.join(CFG_DIR, "qwen3_4b_grpo_8xb200.yaml"))
    assert cfg.train_tp_size == 2 and cfg.train_dp_size == 2
    assert cfg.hardware.flops_peak == pytest.approx(1.622e15)
    assert cfg.model_arch.d_model == 2560 and cfg.model_arch.head_dim == 128
    assert cfg.heterogeneous_rollout.tp_list == [1, 1, 2]
    assert cfg.heterogeneous_rollout.instances[2].instance_id == "hetero_tp2_2"
    assert cfg.heterogeneous_rollout.scheduling.scheduler_type == "cmlfq"
    tiny = AsyncRLConfig.from_file(os.path.join(CFG_DIR, "tiny_cpu_gloo.yaml"))
    assert tiny.train_dp_size == 2 and tiny.n_total_gpus == 3


def test_numeric_string_coercion():
    cfg = AsyncRLConfig.from_dict({"model_path": "x", "learning_rate": "1e-6", "batch_size": "32",
                                   "hardware": {"flops_peak": "2.25e15", "gpus_per_node": "8"}})
    assert cfg.learning_rate == 1e-6 and cfg.batch_size == 32
    assert isinstance(cfg.hardware.gpus_per_node, int)


@pytest.mark.parametrize("kw,msg", [
    ({"train_gpus": 3, "train_tp_size": 2}, "divisible"),
    ({"batch_size": 30}, "batch_size must be divisible"),
    ({"weight_sync_mode": "foo"}, "weight_sync_mode"),
    ({"rollout_weight_sync_mode": "nccl"}, "requires weight_sync_mode"),
    ({"train_pp_size": 2, "train_tp_size": 2, "train_gpus": 4}, "pipeline stages run with train_tp_size=1"),
    ({"train_cp_size": 2, "train_gpus": 8}, "train_cp_size=2: sequences are not split"),
    ({"train_backend": "deepspeed"}, "train_backend"),
    ({"megatron_optimizer_offload_fraction": 0.5}, "needs megatron_optimizer_cpu_offload=true"),
    ({"train_ep_size": 2, "train_gpus": 2}, "needs a mixture-of-experts model"),
    ({"train_tp_size": 3, "train_gpus": 3, "batch_size": 3, "micro_batch_size": 1}, "train_tp_size=3 must divide"),
])
def test_validation_errors(kw, msg, tmp_path):
    base = {"model_path": "m", "sync_path": str(tmp_path / "s"), "log_dir": str(tmp_path / "l")}
    with pytest.raises(ValueError, match=msg):
        AsyncRLConfig.from_dict({**base, **kw})


def test_composition_order(tmp_path):
    (tmp_path / "hw.yaml").write_text("flops_peak: 1.0\nmem_bw: 2.0\n")
    (tmp_path / "base.yaml").write_text("model_path: a\nbatch_size: 8\nmicro_batch_size: 1\nhardware: {mem_bw: 5.0}\n")
    (tmp_path / "exp.yaml").write_text("base_config: base.yaml\nhardware_config: hw.yaml\nbatch_size: 16\n"
                                       f"sync_path: {tmp_path}/s\nlog_dir: {tmp_path}/l\n")
    cfg = load_config(str(tmp_path / "exp.yaml"))
    assert cfg.batch_size == 16 and cfg.hardware.flops_peak == 1.0 and cfg.hardware.mem_bw == 2.0
    (tmp_path / "cyc.yaml").write_text("base_config: cyc.yaml\n")
    with pytest.raises(ValueError, match="cyclic"):
        load_config(str(tmp_path / "cyc.yaml"))


def test_merge_and_roundtrip(tmp_path):
    assert merge_dicts({"a": {"b": 1, "c": 2}}, {"a": {"c": 3}}) == {"a": {"b": 1, "c": 3}}
    cfg = AsyncRLConfig.from_dict({"model_path": "m", "sync_path": str(tmp_path / "s"), "log_dir": str(tmp_path / "l")})
    cfg.to_yaml(str(tmp_path / "o.yaml"))
    again = AsyncRLConfig.from_file(str(tmp_path / "o.yaml"))
    assert again.to_dict() == cfg.to_dict()


def test_load_config_requires_path(monkeypatch):
    monkeypatch.delenv("ASYNC_RL_CONFIG", raising=False)
    with pytest.raises(ValueError, match="no config given"):
        load_config(None)


def test_parallel_layout_reaches_the_engine():
    """train_tp_size / train_ep_size from the presets arrive in the engine the factory builds."""
    from libra_b200.engine.train_engine import create_train_engine

    c14 = AsyncRLConfig.from_file(os.path.join(CFG_DIR, "qwen3_14b_agentic_tp4.yaml"))
    e14 = create_train_engine(c14)
    assert e14.tp_size == 4 and e14.ep_size == 1 and e14.cfg.hidden_size == 5120
    assert e14.sequence_parallel  # base.yaml turns sequence parallelism on for TP > 1
    c14.megatron_use_precision_aware_optimizer = True
    c14.megatron_optimizer_cpu_offload, c14.megatron_optimizer_offload_fraction = True, 0.25
    e14b = create_train_engine(c14)
    assert e14b.precision_aware_optimizer and e14b.optimizer_offload_fraction == 0.25
    c30 = AsyncRLConfig.from_file(os.path.join(CFG_DIR, "qwen3_30b_a3b_ep8.yaml"))
    e30 = create_train_engine(c30)
    assert e30.tp_size == 1 and e30.ep_size == 8 and e30.cfg.num_experts == 128
    c4 = AsyncRLConfig.from_file(os.path.join(CFG_DIR, "qwen3_4b_grpo_8xb200.yaml"))
    c4.train_tp_size, c4.train_pp_size = 1, 2
    assert create_train_engine(c4).pp_size == 2


def test_presets_give_each_data_parallel_replica_complete_grpo_groups():
    """Every shipped preset splits its batch into whole GRPO groups per
    data-parallel replica (reference tests/test_production_ehp_ab_config.py)
    and names GPUs of one 8-GPU box (a preset may time-share them between
    training and rollout)."""
    import glob
    import os

    from libra_b200.config import AsyncRLConfig

    root = os.path.join(os.path.dirname(os.path.dirname(__file__)), "libra_b200", "configs")
    presets = [f for f in sorted(glob.glob(os.path.join(root, "*.yaml"))) if not f.endswith("base.yaml")]
    assert len(presets) >= 4
    for f in presets:
        c = AsyncRLConfig.from_file(f)
        local = c.batch_size // max(1, c.train_dp_size)
        assert c.batch_size % max(1, c.train_dp_size) == 0 and local % c.n_samples == 0, f
        assert max(c.train_gpus, c.rollout_gpus) <= 8 and 0.0 <= c.r2e_stop_reward <= 1.0, f
        assert all(0 <= g < 8 for inst in c.heterogeneous_rollout.instances for g in inst.gpus), f
