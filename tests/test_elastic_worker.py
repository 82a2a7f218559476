"""End-to-end hybrid replica on CPU: snapshot -> task -> payload over TCP ->
merge before the core step -> lockstep update -> identical weights."""

import threading

import torch

from libra_b200.engine.train_engine import B200TrainEngine
from libra_b200.infra.elastic import worker as hw
from libra_b200.workflow.synthetic import GRPOWorkload, LengthDist


def _wl(vocab):
    return GRPOWorkload("t", vocab_size=vocab, prompts_per_step=2, group_size=4, prompt=LengthDist(12, 0.3, 4, 24),
                        response=LengthDist(16, 0.3, 2, 32))


def test_hybrid_replica_lockstep_over_tcp(tmp_path, monkeypatch):
    monkeypatch.setenv("ELASTIC_TRAINING_STATE_DIR", str(tmp_path / "state"))
    core = B200TrainEngine("tiny", device="cpu", use_distributed_optimizer=False, learning_rate=1e-3)
    core.initialize()
    domain = core.configure_elastic_training()
    server = hw.attach_gradient_server(core, authkey="k")
    try:
        snap = core.get_elastic_state_snapshot_path(core.capture_elastic_state_snapshot("h", "dp0"))
        domain.request_join("h", "dp0")
        domain.mark_active("h")
        wl = _wl(core.cfg.vocab_size)
        hybrid_trajs = wl.trajectories(1)
        hw.write_task(str(tmp_path / "tasks"), "h", core.step_count + 1, hybrid_trajs, state_version=core.current_version,
                      membership_epoch=domain.membership_epoch("h"))
        ep = server.endpoint
        argv = ["--replica-id", "h", "--target-core-id", "dp0", "--snapshot-path", snap, "--gradient-host", ep.host,
                "--gradient-port", str(ep.port), "--authkey", "k", "--task-dir", str(tmp_path / "tasks"),
                "--model", "tiny", "--device", "cpu", "--max-tasks", "1", "--poll-interval", "0.05"]
        holder = {}

        def run():
            import libra_b200.infra.elastic.worker as w

            orig = w._engine

            def capture(args):
                holder["engine"] = orig(args)
                return holder["engine"]

            w._engine = capture
            try:
                holder["rc"] = w.main(argv)
            finally:
                w._engine = orig

        t = threading.Thread(target=run)
        t.start()
        core.elastic_payload_wait_s = 60.0
        core_trajs = wl.trajectories(0)
        core.recompute_logprobs(core_trajs)
        stats = core.grpo_update(core_trajs)
        t.join(60)
        assert holder.get("rc") == 0 and server.received_count == 1
        assert (tmp_path / "tasks" / f"h.step_1.pt.done").exists()
        hyb = holder["engine"]
        torch.testing.assert_close(hyb.flat_param.float(), core.flat_param.float(), rtol=0, atol=0)
        assert stats["n_updates"] == 1.0
    finally:
        server.close()


def test_controller_launches_and_stops_exact_worker(tmp_path):
    import sys

    from libra_b200.infra.elastic.controller import Controller, request_launch, request_stop

    c = Controller(str(tmp_path))
    request_launch(str(tmp_path), "w0", f"{sys.executable} -c 'import time; time.sleep(60)'")
    request_launch(str(tmp_path), "bad", "")
    assert c.poll_once()
    import json

    started = json.loads((tmp_path / ".launch_w0.started").read_text())
    proc = c.workers["w0"]
    assert started["pid"] == proc.pid and proc.poll() is None
    request_stop(str(tmp_path), "w0")
    c.poll_once()
    assert proc.poll() is not None and "w0" not in c.workers
    assert not list(tmp_path.glob(".launch_*.running"))


def test_trainer_dispatches_batch_shares_to_an_active_hybrid(tmp_path, monkeypatch):
    """AsyncRLTrainer with an active hybrid replica (Elastic Hybrid Pool): each
    step half of the GRPO groups go to the hybrid as a task, the core waits for
    its gradient, averages it with its own before the optimizer step, and the
    hybrid applies the same update in lockstep (bit-identical weights)."""
    from libra_b200.config import AsyncRLConfig
    from libra_b200.trainer.async_rl_trainer import AsyncRLTrainer
    from libra_b200.workflow.synthetic import GRPOWorkload, LengthDist, rollout_requests
    from libra_b200.workflow.synthetic_workflows import GRPOLengthWorkflow, grpo_length_dataset

    monkeypatch.setenv("ELASTIC_TRAINING_STATE_DIR", str(tmp_path / "state"))
    tasks = tmp_path / "tasks"
    wl = GRPOWorkload("t", vocab_size=1024, prompts_per_step=2, group_size=4, prompt=LengthDist(20, 0.3, 8, 32),
                      response=LengthDist(10, 0.5, 1, 16))
    reqs = []
    for s in range(3):
        reqs += rollout_requests(wl, s, prompts=2)
    cfg = AsyncRLConfig.from_dict({
        "model_path": "tiny", "rollout_backend": "colocated", "train_gpus": 1, "rollout_gpus": 0,
        "batch_size": 8, "n_samples": 4, "micro_batch_size": 4, "max_concurrent_rollouts": 16,
        "max_head_offpolicyness": 1, "total_steps": 2, "sync_interval": 1, "max_seq_length": 64,
        "learning_rate": 1e-3, "enable_history_collection": False, "log_dir": str(tmp_path / "l"),
        "sync_path": str(tmp_path / "s"), "save_interval": 0,
        "global_resource_planner": {"enabled": False, "hybrid_worker_task_dir": str(tasks),
                                    "hybrid_active_gradient_timeout_s": 120.0},
        "heterogeneous_rollout": {"enabled": False}})
    core = B200TrainEngine("tiny", device="cpu", use_distributed_optimizer=False, learning_rate=1e-3, micro_batch_size=4)
    core.initialize(max_seq_length=64)
    domain = core.configure_elastic_training()
    server = hw.attach_gradient_server(core, authkey="k")
    holder = {}
    try:
        snap = core.get_elastic_state_snapshot_path(core.capture_elastic_state_snapshot("h", "dp0"))
        domain.request_join("h", "dp0")
        domain.mark_active("h")
        ep = server.endpoint
        argv = ["--replica-id", "h", "--target-core-id", "dp0", "--snapshot-path", snap, "--gradient-host", ep.host,
                "--gradient-port", str(ep.port), "--authkey", "k", "--task-dir", str(tasks), "--model", "tiny",
                "--device", "cpu", "--max-tasks", "2", "--poll-interval", "0.05"]

        def run():
            import libra_b200.infra.elastic.worker as w

            orig = w._engine

            def capture(args):
                holder["engine"] = orig(args)
                return holder["engine"]

            w._engine = capture
            try:
                holder["rc"] = w.main(argv)
            finally:
                w._engine = orig

        t = threading.Thread(target=run)
        t.start()
        tr = AsyncRLTrainer(cfg, train_engine=core)
        seen = []
        tr.step_callback = lambda step, stats, batch: seen.append((step, len(batch), tr.last_hybrid_dispatch))
        tr.train(GRPOLengthWorkflow(), grpo_length_dataset(reqs))
        t.join(120)
        assert holder.get("rc") == 0 and server.received_count == 2
        assert [s for s, _, _ in seen] == [0, 1]
        for _, n_core, d in seen:
            assert d is not None and d["hybrids"] == ["h"] and d["hybrid_trajectories"] == 4 and n_core == 4
        assert sorted(p.name for p in tasks.glob("h.step_*.pt.done")) == ["h.step_1.pt.done", "h.step_2.pt.done"]
        torch.testing.assert_close(holder["engine"].flat_param.float(), core.flat_param.float(), rtol=0, atol=0)
    finally:
        server.close()
