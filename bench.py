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


def emit(rank, record):
    if rank == 0:
        print(json.dumps(record), flush=True)


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


# ---------------------------------------------------------------------- reference
def _make_reference_checkpoint(path, model_name, rank, world):
    """Random-init HF Qwen3 checkpoint + a word-level tokenizer (no network)."""
    from transformers import PreTrainedTokenizerFast, Qwen3Config, Qwen3ForCausalLM
    from tokenizers import Tokenizer
    from tokenizers.models import WordLevel

    from libra_b200.models.qwen3 import get_config

    cfg = get_config(model_name)
    if rank == 0 and not os.path.exists(os.path.join(path, "done")):
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
        tok = PreTrainedTokenizerFast(tokenizer_object=Tokenizer(WordLevel(vocab, unk_token="<unk>")),
                                      unk_token="<unk>", eos_token="<eos>", pad_token="<eos>")
        tok.save_pretrained(path)
        open(os.path.join(path, "done"), "w").close()
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


def main():
    args = parse_args()
    rank, world, local = setup_dist(args.gpus)
    try:
        if not torch.cuda.is_available():
            emit(rank, {"impl": args.impl, "unavailable": "no CUDA device"})
            return
        if args.impl == "reference":
            run_reference(args, rank, world, local)
        else:
            run_ours(args, rank, world, local)
    finally:
        if world > 1 and dist.is_initialized():
            dist.destroy_process_group()


if __name__ == "__main__":
    main()
