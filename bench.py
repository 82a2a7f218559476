"""GRPO training-step benchmark (trained tokens/s) on Qwen3-4B, bf16.

    python bench.py --gpus N --steps K --warmup W [--impl ours|reference]

One step = logprob recompute over the step's trajectories + one GRPO update
(forward, backward, gradient reduction, clip, AdamW) — the work the reference's
trainer does per step (trainer/async_rl_trainer.py:858-870 recompute, then
grpo_update).  Workload: per GPU 8 prompts x group 8 = 64 trajectories per step
(at 8 GPUs: 64 prompts x 8 = 512, the configured global batch); prompt length
lognormal median 300 clipped 64-1024, response lognormal median 1500 clipped at
4096, uniform random token ids, Bernoulli(0.4) rewards, random-init weights.
Weak scaling (per-GPU work fixed).  The metric is tokens/s = sum of (prompt +
response) tokens over all ranks / step time (reference
scripts/analyze_libra_experiment.py:117-131), step time = max over ranks of the
CUDA-event time.

`value` times the engine on device-resident packed micro-batches; `e2e` times
the public API (`recompute_logprobs` + `grpo_update`) with host trajectories,
including the pinned host->device copies and the device->host logprob/stat reads.
"""

from __future__ import annotations

import argparse
import datetime
import json
import os
import sys
import time

import torch
import torch.distributed as dist

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, HERE)

METRIC = "GRPO trained tokens/s"
MODEL = "Qwen3-4B"


def parse_args():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=5)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--mode", choices=["grpo", "train"], default="grpo",
                    help="grpo: full GRPO step (rollout generation + logprob recompute + update + weight sync); "
                         "train: trainer half only (recompute + update)")
    ap.add_argument("--max-running", type=int, default=128, help="rollout engine: concurrent sequences")
    ap.add_argument("--model", default="qwen3-4b")
    ap.add_argument("--prompts-per-gpu", type=int, default=8)
    ap.add_argument("--group", type=int, default=8)
    ap.add_argument("--micro-batch", type=int, default=8, help="trajectories per loss-normalisation group")
    ap.add_argument("--recompute-micro-batch", type=int, default=16)
    ap.add_argument("--max-tokens", type=int, default=16384, help="tokens per execution chunk (update)")
    ap.add_argument("--max-recompute-tokens", type=int, default=65536, help="tokens per execution chunk (recompute)")
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--no-launch-count", action="store_true")
    return ap.parse_args()


def setup_dist(n_gpus: int):
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world > 1:
        torch.cuda.set_device(local)
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=600),
                                device_id=torch.device("cuda", local))
    elif torch.cuda.is_available():
        torch.cuda.set_device(0)
    return rank, world, local


def barrier(world):
    if world > 1:
        dist.barrier()


_RECORD_OUT = None  # the process's original stdout; fd 1 itself is pointed at stderr during the run


def emit(rank, record):
    # the record goes to the process's real stdout; everything else printed during the run, including
    # native libraries writing to fd 1 (NCCL's version banner), goes to stderr
    if rank == 0:
        out = _RECORD_OUT or sys.__stdout__
        out.write(json.dumps(record) + "\n")
        out.flush()


def base_record(args, world, impl):
    global_batch = args.prompts_per_gpu * args.group * world
    return {
        "metric": METRIC, "unit": "tokens/s", "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "bf16",
        "data": "synthetic (seeded random token ids, lognormal lengths, Bernoulli(0.4) rewards, random-init weights)",
        "impl": impl,
        "config": {"model": MODEL, "global_batch": global_batch, "seq_len": "prompt ~LN(300) [64,1024] + response ~LN(1500) [1,4096]",
                   "parallelism": f"dp{world}", "prompts_per_gpu": args.prompts_per_gpu, "group": args.group,
                   "micro_batch_trajectories": args.micro_batch, "max_tokens_per_chunk": args.max_tokens,
                   "l2": "inputs larger than L2 (8 GB of weights and >10 GB of activations per step)"},
    }


def count_launches(fn, prefixes=("libra::",)):
    """Run fn once under torch.profiler: count this repo's kernels and return the
    per-kernel device-time breakdown of the step (all kernels, top 20, ms).
    The profiled step is separate from the timed steps."""
    from torch.profiler import ProfilerActivity, profile

    with profile(activities=[ProfilerActivity.CUDA]) as prof:
        fn()
        torch.cuda.synchronize()
    n = 0
    counts, times = {}, {}
    for ev in prof.events():
        if ev.device_type != torch.autograd.DeviceType.CUDA:
            continue
        key = ev.name.split("(")[0][:70]
        times[key] = times.get(key, 0.0) + ev.device_time_total / 1e3
        if any(p in ev.name for p in prefixes):
            n += 1
            counts[key] = counts.get(key, 0) + 1
    top = dict(sorted(((k, round(v, 2)) for k, v in times.items()), key=lambda kv: -kv[1])[:20])
    return n, counts, top


# ---------------------------------------------------------------------- ours
def run_ours(args, rank, world, local):
    from libra_b200.engine.train_engine import B200TrainEngine
    from libra_b200.utils.timing import ClockSampler, DeviceTimer, max_over_ranks, sum_over_ranks
    from libra_b200.workflow.synthetic import WORKLOADS

    dev = torch.device("cuda", local)
    wl = WORKLOADS["qwen3-4b-grpo"]
    eng = B200TrainEngine(args.model, learning_rate=1e-6, micro_batch_size=args.micro_batch,
                          recompute_micro_batch_size=args.recompute_micro_batch, device=dev, seed=0,
                          max_tokens_per_micro_batch=args.max_tokens,
                          max_tokens_per_recompute_batch=args.max_recompute_tokens)
    eng.initialize(max_seq_length=5120)
    n_steps = args.warmup + args.steps

    def host_step(step):
        return wl.trajectories(step, rank=rank, prompts=args.prompts_per_gpu, pin=True)

    def tokens_of(trajs):
        return sum(int(t["input_ids"].numel()) for t in trajs)

    # ---- device-resident timing ("value") --------------------------------
    staged = []
    for s in range(n_steps):
        trajs = host_step(s)
        upd = [eng.to_device(h) for h in eng.prepare_update(trajs)]
        rec = [eng.to_device(h)["batch"] for _, h in eng.prepare_recompute(trajs)]
        staged.append((tokens_of(trajs), rec, upd))
    torch.cuda.synchronize(dev)

    def device_step(s):
        _, rec, upd = staged[s]
        with torch.no_grad():
            for b in rec:
                eng.model.action_logprobs(b, eng.temperature)
        eng.update_packed(upd, sync_stats=False)

    for s in range(args.warmup):
        device_step(s)
    torch.cuda.synchronize(dev)
    barrier(world)
    sampler = ClockSampler(local).start()
    with DeviceTimer(dev) as t:
        for s in range(args.warmup, n_steps):
            device_step(s)
    barrier(world)
    clocks = sampler.stop()
    ms_step = max_over_ranks(t.ms / args.steps, dev)
    tokens_rank = sum(staged[s][0] for s in range(args.warmup, n_steps)) / args.steps
    tokens_step = sum_over_ranks(tokens_rank, dev)
    value = tokens_step / (ms_step / 1e3)
    from libra_b200 import ops
    ops.check_kernel_errors(dev)

    launches = None
    launch_names, kernel_ms = {}, {}
    if not args.no_launch_count:
        n, launch_names, kernel_ms = count_launches(lambda: device_step(args.warmup))
        launches = int(max_over_ranks(n, dev)) * args.steps
    del staged
    torch.cuda.empty_cache()

    # ---- end-to-end through the public API ("e2e") ------------------------
    e2e = None
    if not args.no_e2e:
        host = [host_step(1000 + s) for s in range(n_steps)]
        def api_step(trajs):
            eng.recompute_logprobs(trajs)
            return eng.grpo_update(trajs)

        for s in range(args.warmup):
            api_step(host[s])
        torch.cuda.synchronize(dev)
        barrier(world)
        eng.io_bytes = {"h2d": 0, "d2h": 0}
        t0 = time.perf_counter()
        for s in range(args.warmup, n_steps):
            api_step(host[s])
        torch.cuda.synchronize(dev)
        e2e_ms = max_over_ranks((time.perf_counter() - t0) * 1e3 / args.steps, dev)
        barrier(world)
        h2d = [eng.io_bytes["h2d"]]
        d2h = [eng.io_bytes["d2h"]]
        e2e_tokens = sum_over_ranks(sum(tokens_of(host[s]) for s in range(args.warmup, n_steps)) / args.steps, dev)
        e2e = {"value": e2e_tokens / (e2e_ms / 1e3), "unit": "tokens/s", "ms_per_step": e2e_ms,
               "h2d_bytes_per_step": int(h2d[0] / args.steps), "d2h_bytes_per_step": int(d2h[0] / args.steps),
               "api": "B200TrainEngine.recompute_logprobs + grpo_update (host trajectories)"}

    rec = base_record(args, world, "ours")
    rec.update({"value": value, "ms_per_step": ms_step, "tokens_per_step": tokens_step, "e2e": e2e,
                "gpu_launches": launches, "clocks": clocks})
    rec["config"]["launch_breakdown_per_step"] = launch_names
    rec["config"]["kernel_ms_per_step_top20"] = kernel_ms
    emit(rank, rec)


def run_ours_grpo(args, rank, world, local):
    """Full GRPO step on every rank: the rank's own rollout engine (sharing the
    GPU with its trainer, with its own weight copy and paged KV cache) generates
    the step's 8 prompts x 8 samples, the trainer recomputes logprobs and takes
    the GRPO update (data-parallel gradient reduction across ranks), then the
    new weights are synced into the rollout engine (one device copy of the flat
    bf16 buffer) and the policy version advances."""
    from libra_b200.engine.rollout.llm_engine import LLMEngine
    from libra_b200.engine.rollout.kv_cache import PagedKVCache
    from libra_b200.engine.rollout.sampler import SamplingParams
    from libra_b200.engine.train_engine import B200TrainEngine
    from libra_b200.utils.timing import ClockSampler, max_over_ranks, sum_over_ranks
    from libra_b200.workflow.synthetic import WORKLOADS, group_normalize, rollout_requests, rollout_trajectory

    dev = torch.device("cuda", local)
    wl = WORKLOADS["qwen3-4b-grpo"]
    eng = B200TrainEngine(args.model, learning_rate=1e-6, micro_batch_size=args.micro_batch,
                          recompute_micro_batch_size=args.recompute_micro_batch, device=dev, seed=0,
                          max_tokens_per_micro_batch=args.max_tokens,
                          max_tokens_per_recompute_batch=args.max_recompute_tokens)
    max_len = wl.prompt.hi + wl.response.hi + 16
    eng.initialize(max_seq_length=max_len)
    rollout_flat = eng.flat_param.clone()
    n_req = args.prompts_per_gpu * args.group
    cfg = eng.cfg
    block = 16
    worst = n_req * -(-max_len // block) + 64
    free, _ = torch.cuda.mem_get_info(dev)
    # the trainer's activations (tens of GB at 16k-token chunks) are not allocated yet: leave them room
    budget_blocks = PagedKVCache.blocks_for_budget(0.25 * free, cfg.num_hidden_layers, block,
                                                   cfg.num_key_value_heads, cfg.head_dim)
    llm = LLMEngine(cfg, eng.layout.views(rollout_flat), kv_blocks=min(worst, budget_blocks), block_size=block,
                    max_model_len=max_len, max_running=args.max_running, max_batch_tokens=16384, flat=rollout_flat)
    n_steps = args.warmup + args.steps

    def ev():
        e = torch.cuda.Event(enable_timing=True)
        e.record()
        return e

    def grpo_step(s):
        reqs = rollout_requests(wl, s, rank=rank, prompts=args.prompts_per_gpu)
        e0 = ev()
        res = llm.generate_sync([r.prompt for r in reqs],
                                [SamplingParams(max_tokens=r.response_len, temperature=1.0) for r in reqs])
        e1 = ev()
        trajs = [rollout_trajectory(r, g.output_tokens, g.output_logprobs, llm.version, pin=True)
                 for r, g in zip(reqs, res)]
        group_normalize(trajs)
        eng.recompute_logprobs(trajs)
        eng.grpo_update(trajs)
        e2 = ev()
        llm.load_flat_weights(eng.flat_param, version=s + 1)
        eng.set_version(s + 1)
        e3 = ev()
        toks = sum(int(t["input_ids"].numel()) for t in trajs)
        return toks, (e0, e1, e2, e3), sum(len(g.output_tokens) for g in res)

    for s in range(args.warmup):
        grpo_step(s)
    torch.cuda.synchronize(dev)
    barrier(world)
    sampler = ClockSampler(local).start()
    t_start, t_end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    t_start.record()
    tok, gen_tok, marks = 0, 0, []
    for s in range(args.warmup, n_steps):
        n, m, g = grpo_step(s)
        tok += n
        gen_tok += g
        marks.append(m)
    t_end.record()
    torch.cuda.synchronize(dev)
    barrier(world)
    clocks = sampler.stop()
    ms_step = max_over_ranks(t_start.elapsed_time(t_end) / args.steps, dev)
    roll = sum(m[0].elapsed_time(m[1]) for m in marks) / args.steps
    train = sum(m[1].elapsed_time(m[2]) for m in marks) / args.steps
    sync = sum(m[2].elapsed_time(m[3]) for m in marks) / args.steps
    tokens_step = sum_over_ranks(tok / args.steps, dev)
    gen_step = sum_over_ranks(gen_tok / args.steps, dev)
    value = tokens_step / (ms_step / 1e3)
    from libra_b200 import ops
    ops.check_kernel_errors(dev)
    launches = None
    if not args.no_launch_count:
        n, _, _ = count_launches(lambda: grpo_step(n_steps), prefixes=("libra::",))
        launches = int(max_over_ranks(n, dev)) * args.steps
    sync_bytes = rollout_flat.numel() * rollout_flat.element_size()
    e2e = None if args.no_e2e else grpo_e2e_through_trainer(args, rank, world, local, eng, llm, wl)
    rec = base_record(args, world, "ours")
    rec["config"]["step"] = ("rollout (own engine, captured decode graphs, temperature 1.0) + logprob recompute + "
                             "GRPO update + weight sync to the rollout engine")
    rec["config"]["rollout"] = f"colocated: one engine per GPU, {args.max_running} concurrent sequences"
    rec.update({"value": value, "ms_per_step": ms_step, "tokens_per_step": tokens_step,
                "generated_tokens_per_step": gen_step,
                "phase_ms": {"rollout": max_over_ranks(roll, dev), "train": max_over_ranks(train, dev),
                             "weight_sync": max_over_ranks(sync, dev)},
                "weight_sync": {"ms": max_over_ranks(sync, dev), "bytes": sync_bytes,
                                "gb_per_s": sync_bytes / (max_over_ranks(sync, dev) / 1e3) / 1e9,
                                "path": "device copy of the flat bf16 parameter buffer into the rollout engine"},
                "gpu_launches": launches, "clocks": clocks, "e2e": e2e})
    emit(rank, rec)


def grpo_e2e_through_trainer(args, rank, world, local, eng, llm, wl):
    """The same GRPO workload end to end through the public orchestrator:
    ``AsyncRLTrainer.train`` with the colocated rollout engine (each rank
    generates its data-parallel share, staleness bound 1), logprob recompute,
    update and weight sync every step.  Timed between step boundaries on every
    rank (synchronize + barrier), max over ranks; counts the host<->device bytes
    of the rollout engine (prompts, decode inputs, sampled tokens) and of the
    trainer (trajectories in, stats out)."""
    from libra_b200.config import AsyncRLConfig
    from libra_b200.engine.rollout_engine import LocalRolloutEngine
    from libra_b200.engine.tokenizer import ByteTokenizer
    from libra_b200.trainer.async_rl_trainer import AsyncRLTrainer
    from libra_b200.utils.timing import max_over_ranks, sum_over_ranks
    from libra_b200.workflow.synthetic import rollout_requests
    from libra_b200.workflow.synthetic_workflows import GRPOLengthWorkflow, grpo_length_dataset

    dev = torch.device("cuda", local)
    warm, steps = max(3, min(args.warmup, 3)), max(2, args.steps // 4)
    reqs = []
    for i in range(warm + steps + 1):
        reqs += rollout_requests(wl, 5000 + i, rank=0, prompts=args.prompts_per_gpu * world)
    dataset = grpo_length_dataset(reqs)
    tmp = os.path.join("/tmp", f"libra_e2e_{os.getpid()}")
    cfg = AsyncRLConfig.from_dict({
        "model_path": args.model, "rollout_backend": "colocated", "train_gpus": world, "rollout_gpus": 0,
        "train_tp_size": 1, "batch_size": args.prompts_per_gpu * args.group * world, "n_samples": args.group,
        "micro_batch_size": args.micro_batch, "max_concurrent_rollouts": args.max_running,
        "max_head_offpolicyness": 1, "total_steps": warm + steps, "sync_interval": 1, "recompute_logprobs": True,
        "max_seq_length": wl.prompt.hi + wl.response.hi + 16, "enable_history_collection": False,
        "log_dir": tmp + "/logs", "sync_path": tmp + "/sync", "save_interval": 0, "eval_interval": 0,
        "global_resource_planner": {"enabled": False}, "heterogeneous_rollout": {"enabled": False}})
    io0 = dict(llm.io_bytes)
    eng.io_bytes = {"h2d": 0, "d2h": 0}
    trainer = AsyncRLTrainer(cfg, train_engine=eng, rollout_engine=LocalRolloutEngine(llm, ByteTokenizer(eng.cfg.vocab_size)))
    marks = {}

    def on_step(step, stats, batch):
        if step == warm - 1 or step == warm + steps - 1:
            torch.cuda.synchronize(dev)
            barrier(world)
            marks[step] = (time.perf_counter(), dict(llm.io_bytes), dict(eng.io_bytes))
        if step >= warm:
            marks.setdefault("tokens", 0)
            marks["tokens"] += sum(int(t["input_ids"].numel()) for t in batch)

    trainer.step_callback = on_step
    trainer.train(GRPOLengthWorkflow(), dataset)
    (t0, r0, e0), (t1, r1, e1) = marks[warm - 1], marks[warm + steps - 1]
    ms = max_over_ranks((t1 - t0) * 1e3 / steps, dev)
    tokens = sum_over_ranks(marks["tokens"] / steps, dev)
    h2d = (r1["h2d"] - r0["h2d"] + e1["h2d"] - e0["h2d"]) / steps
    d2h = (r1["d2h"] - r0["d2h"] + e1["d2h"] - e0["d2h"]) / steps
    return {"value": tokens / (ms / 1e3), "unit": "tokens/s", "ms_per_step": ms, "steps": steps, "warmup": warm,
            "h2d_bytes_per_step": int(max_over_ranks(h2d, dev)), "d2h_bytes_per_step": int(max_over_ranks(d2h, dev)),
            "api": "AsyncRLTrainer.train (rollout_backend=colocated, staleness bound 1, sync every step)"}


# ---------------------------------------------------------------------- reference
def _make_reference_checkpoint(path, model_name, rank, world):
    """Random-init HF Qwen3 checkpoint + a word-level tokenizer (no network)."""
    from transformers import PreTrainedTokenizerFast, Qwen3Config, Qwen3ForCausalLM
    from tokenizers import Tokenizer, pre_tokenizers
    from tokenizers.models import WordLevel

    from libra_b200.models.qwen3 import get_config

    cfg = get_config(model_name)
    if rank == 0 and not os.path.exists(os.path.join(path, "done2")):
        os.makedirs(path, exist_ok=True)
        hf = Qwen3Config(vocab_size=cfg.vocab_size, hidden_size=cfg.hidden_size,
                         intermediate_size=cfg.intermediate_size, num_hidden_layers=cfg.num_hidden_layers,
                         num_attention_heads=cfg.num_attention_heads, num_key_value_heads=cfg.num_key_value_heads,
                         head_dim=cfg.head_dim, rope_theta=cfg.rope_theta, rms_norm_eps=cfg.rms_norm_eps,
                         tie_word_embeddings=cfg.tie_word_embeddings, max_position_embeddings=cfg.max_position_embeddings,
                         torch_dtype="bfloat16")
        with torch.device("cuda"):
            model = Qwen3ForCausalLM(hf).to(torch.bfloat16)
        model.save_pretrained(path, safe_serialization=True)
        del model
        torch.cuda.empty_cache()
        vocab = {f"t{i}": i for i in range(cfg.vocab_size - 2)}
        vocab["<unk>"] = cfg.vocab_size - 2
        vocab["<eos>"] = cfg.vocab_size - 1
        wl = Tokenizer(WordLevel(vocab, unk_token="<unk>"))
        wl.pre_tokenizer = pre_tokenizers.WhitespaceSplit()  # "t5 t9" -> ids 5, 9 (text round-trips)
        tok = PreTrainedTokenizerFast(tokenizer_object=wl, unk_token="<unk>", eos_token="<eos>", pad_token="<eos>")
        tok.save_pretrained(path)
        open(os.path.join(path, "done2"), "w").close()
    barrier(world)


def run_reference(args, rank, world, local):
    ref_root = os.path.join(HERE, "baseline", "_ref")
    if not os.path.isdir(os.path.join(ref_root, "RL_Framework")):
        emit(rank, {"impl": "reference", "unavailable": "baseline/_ref is not installed"})
        return
    sys.path.insert(0, ref_root)
    from RL_Framework.engine.train_engine import FSDPTrainEngine  # the reference's own engine, unmodified

    from libra_b200.utils.timing import ClockSampler, max_over_ranks, sum_over_ranks
    from libra_b200.workflow.synthetic import WORKLOADS

    dev = torch.device("cuda", local)
    ckpt = os.environ.get("LIBRA_REF_CKPT", "/tmp/libra_ref_qwen3_4b")
    _make_reference_checkpoint(ckpt, args.model, rank, world)
    eng = FSDPTrainEngine(model_path=ckpt, learning_rate=1e-6, kl_coef=0.001, clip_epsilon=0.2,
                          micro_batch_size=args.micro_batch)
    eng.initialize(max_seq_length=5120)
    wl = WORKLOADS["qwen3-4b-grpo"]
    n_steps = args.warmup + args.steps

    def tokens_of(trajs):
        return sum(int(t["input_ids"].numel()) for t in trajs)

    def step(s):
        trajs = wl.trajectories(s, rank=rank, prompts=args.prompts_per_gpu, pin=True)
        eng.recompute_logprobs(trajs)
        eng.grpo_update(trajs)
        return tokens_of(trajs)

    for s in range(args.warmup):
        step(s)
    torch.cuda.synchronize(dev)
    barrier(world)
    sampler = ClockSampler(local).start()
    start = torch.cuda.Event(enable_timing=True)
    end = torch.cuda.Event(enable_timing=True)
    start.record()
    tok = 0
    for s in range(args.warmup, n_steps):
        tok += step(s)
    end.record()
    torch.cuda.synchronize(dev)
    barrier(world)
    clocks = sampler.stop()
    ms_step = max_over_ranks(start.elapsed_time(end) / args.steps, dev)
    tokens_step = sum_over_ranks(tok / args.steps, dev)
    rec = base_record(args, world, "reference")
    rec.update({"value": tokens_step / (ms_step / 1e3), "ms_per_step": ms_step, "tokens_per_step": tokens_step,
                "clocks": clocks, "gpu_launches": 0,
                "e2e": {"value": tokens_step / (ms_step / 1e3), "unit": "tokens/s",
                        "api": "RL_Framework FSDPTrainEngine.recompute_logprobs + grpo_update (host trajectories)"}})
    rec["config"]["reference_engine"] = "FSDPTrainEngine (Megatron-Core is not installable offline)"
    emit(rank, rec)


def _start_vllm(ckpt: str, ref_root: str, local: int, port: int, gpu_util: float, max_len: int, log_path: str):
    """vLLM OpenAI server on this rank's GPU, with vLLM's developer routes on so
    /collective_rpc reaches the workers.  The reference's in-place reload
    extension (RL_Framework.vllm_hot_reload.InplaceReloadWorkerExtension) cannot
    be registered on vLLM 0.22, whose Worker already defines reload_weights;
    that built-in method performs the same in-place load of a checkpoint
    directory, so the arm calls it instead."""
    import subprocess

    env = dict(os.environ)
    env.update({"CUDA_VISIBLE_DEVICES": os.environ.get("CUDA_VISIBLE_DEVICES", "").split(",")[local]
                if os.environ.get("CUDA_VISIBLE_DEVICES") else str(local),
                "PYTHONPATH": ref_root + os.pathsep + env.get("PYTHONPATH", ""), "HF_HUB_OFFLINE": "1",
                "TRANSFORMERS_OFFLINE": "1", "VLLM_SERVER_DEV_MODE": "1", "TOKENIZERS_PARALLELISM": "false"})
    for k in ("RANK", "LOCAL_RANK", "WORLD_SIZE", "MASTER_ADDR", "MASTER_PORT", "LOCAL_WORLD_SIZE", "GROUP_RANK",
              "ROLE_RANK", "ROLE_WORLD_SIZE", "TORCHELASTIC_RUN_ID"):
        env.pop(k, None)
    cmd = [sys.executable, "-m", "vllm.entrypoints.openai.api_server", "--model", ckpt, "--host", "127.0.0.1",
           "--port", str(port), "--dtype", "bfloat16", "--gpu-memory-utilization", str(gpu_util),
           "--max-model-len", str(max_len), "--seed", "0"]
    log = open(log_path, "w")
    return subprocess.Popen(cmd, env=env, stdout=log, stderr=subprocess.STDOUT, start_new_session=True)


def _post_json(url: str, body: dict, timeout: float = 600.0):
    import urllib.request

    req = urllib.request.Request(url, data=json.dumps(body).encode(), method="POST",
                                 headers={"Content-Type": "application/json"})
    with urllib.request.urlopen(req, timeout=timeout) as r:
        return r.read()


def run_reference_grpo(args, rank, world, local):
    """The reference's GRPO step on the same workload: rollout through its own
    HTTP client (RL_Framework.engine.rollout_engine.VLLMRolloutEngine) against a
    vLLM 0.22 server on this rank's GPU, logprob recompute + GRPO update through
    its FSDPTrainEngine, and its disk weight sync (FSDPTrainEngine.save_weights)
    followed by its in-place vLLM reload (RL_Framework.vllm_hot_reload)."""
    import asyncio
    import signal

    ref_root = os.path.join(HERE, "baseline", "_ref")
    if not os.path.isdir(os.path.join(ref_root, "RL_Framework")):
        emit(rank, {"impl": "reference", "unavailable": "baseline/_ref is not installed"})
        return
    sys.path.insert(0, ref_root)
    from RL_Framework.engine.rollout_engine import VLLMRolloutEngine
    from RL_Framework.engine.train_engine import FSDPTrainEngine

    from libra_b200.utils.timing import ClockSampler, max_over_ranks, sum_over_ranks
    from libra_b200.workflow.synthetic import WORKLOADS, group_normalize, rollout_requests, rollout_trajectory

    dev = torch.device("cuda", local)
    ckpt = os.environ.get("LIBRA_REF_CKPT", "/tmp/libra_ref_qwen3_4b")
    _make_reference_checkpoint(ckpt, args.model, rank, world)
    wl = WORKLOADS["qwen3-4b-grpo"]
    max_len = wl.prompt.hi + wl.response.hi + 16
    port = 8100 + local
    logdir = os.path.join(HERE, "gpurun_out") if os.path.isdir(os.path.join(HERE, "gpurun_out")) else "/tmp"
    proc = _start_vllm(ckpt, ref_root, local, port, float(os.environ.get("LIBRA_REF_VLLM_UTIL", "0.3")), max_len,
                       os.path.join(logdir, f"ref_vllm_rank{rank}.log"))
    try:
        client = VLLMRolloutEngine("127.0.0.1", port, ckpt)
        client.wait_for_ready(timeout=float(os.environ.get("LIBRA_REF_VLLM_TIMEOUT", "900")))
        barrier(world)
        train = FSDPTrainEngine(model_path=ckpt, learning_rate=1e-6, kl_coef=0.001, clip_epsilon=0.2,
                                micro_batch_size=args.micro_batch)
        train.initialize(max_seq_length=max_len)
        from transformers import AutoTokenizer

        tok = AutoTokenizer.from_pretrained(ckpt)
        sync_root = os.environ.get("LIBRA_REF_SYNC_DIR", "/tmp/libra_ref_sync")
        n_steps = args.warmup + args.steps

        async def rollout(reqs):
            return await asyncio.gather(*[client.generate(" ".join(f"t{t}" for t in r.prompt),
                                                          max_new_tokens=r.response_len, temperature=1.0)
                                          for r in reqs])

        def ev():
            e = torch.cuda.Event(enable_timing=True)
            e.record()
            return e

        def step(s):
            reqs = rollout_requests(wl, s, rank=rank, prompts=args.prompts_per_gpu)
            e0 = ev()
            res = asyncio.run(rollout(reqs))
            e1 = ev()
            trajs = []
            for r, g in zip(reqs, res):
                ids = tok.convert_tokens_to_ids([t.strip() for t in g["tokens"]])
                trajs.append(rollout_trajectory(r, [int(i) for i in ids], [float(x or 0.0) for x in g["logprobs"]],
                                                s, pin=True))
            group_normalize(trajs)
            train.recompute_logprobs(trajs)
            train.grpo_update(trajs)
            e2 = ev()
            # the reference's disk weight sync: rank 0 writes v<step>/ (FSDP full state dict), every
            # instance reloads it in place through the reference's worker extension
            train.save_weights(sync_root, s + 1)
            barrier(world)
            _post_json(f"http://127.0.0.1:{port}/collective_rpc",
                       {"method": "reload_weights", "kwargs": {"weights_path": os.path.join(sync_root, f"v{s + 1}")}})
            _post_json(f"http://127.0.0.1:{port}/reset_prefix_cache", {})
            barrier(world)
            e3 = ev()
            return sum(int(t["input_ids"].numel()) for t in trajs), (e0, e1, e2, e3)

        for s in range(args.warmup):
            step(s)
        torch.cuda.synchronize(dev)
        barrier(world)
        sampler = ClockSampler(local).start()
        t0, t1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        t0.record()
        tokens, marks = 0, []
        for s in range(args.warmup, n_steps):
            n, m = step(s)
            tokens += n
            marks.append(m)
        t1.record()
        torch.cuda.synchronize(dev)
        barrier(world)
        clocks = sampler.stop()
        ms_step = max_over_ranks(t0.elapsed_time(t1) / args.steps, dev)
        phase = {k: max_over_ranks(sum(m[i].elapsed_time(m[i + 1]) for m in marks) / args.steps, dev)
                 for i, k in enumerate(("rollout", "train", "weight_sync"))}
        tokens_step = sum_over_ranks(tokens / args.steps, dev)
        rec = base_record(args, world, "reference")
        rec["config"]["step"] = ("rollout (vLLM 0.22 server through RL_Framework VLLMRolloutEngine) + "
                                 "FSDPTrainEngine.recompute_logprobs + grpo_update + save_weights + in-place reload")
        rec["config"]["reference_engine"] = "FSDPTrainEngine (Megatron-Core is not installable offline)"
        rec.update({"value": tokens_step / (ms_step / 1e3), "ms_per_step": ms_step, "tokens_per_step": tokens_step,
                    "phase_ms": phase, "weight_sync": {"ms": phase["weight_sync"]}, "clocks": clocks,
                    "gpu_launches": 0,
                    "e2e": {"value": tokens_step / (ms_step / 1e3), "unit": "tokens/s",
                            "api": "RL_Framework VLLMRolloutEngine.generate + FSDPTrainEngine"}})
        emit(rank, rec)
    finally:
        try:
            os.killpg(proc.pid, signal.SIGTERM)
            proc.wait(timeout=60)
        except Exception:  # noqa: BLE001 - the server may already be gone
            pass


def main():
    import contextlib

    global _RECORD_OUT
    args = parse_args()
    sys.stdout.flush()
    _RECORD_OUT = os.fdopen(os.dup(1), "w")
    os.dup2(2, 1)  # native writes to fd 1 land on stderr
    with contextlib.redirect_stdout(sys.stderr):  # stdout carries the one JSON record (emit) and nothing else
        _main(args)
    _RECORD_OUT.flush()


def _main(args):
    rank, world, local = setup_dist(args.gpus)
    try:
        if not torch.cuda.is_available():
            emit(rank, {"impl": args.impl, "unavailable": "no CUDA device"})
            return
        if args.impl == "reference":
            run_reference_grpo(args, rank, world, local) if args.mode == "grpo" else run_reference(args, rank, world, local)
        else:
            run_ours_grpo(args, rank, world, local) if args.mode == "grpo" else run_ours(args, rank, world, local)
    finally:
        if world > 1 and dist.is_initialized():
            dist.destroy_process_group()


if __name__ == "__main__":
    main()
