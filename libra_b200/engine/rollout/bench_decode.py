"""Decode-step microbenchmark of the rollout engine (one GPU).

    python -m libra_b200.engine.rollout.bench_decode --model qwen3-4b --batch 64 --prompt 300 --steps 200

Builds an engine with random weights, prefills ``batch`` prompts, then times
``steps`` pure decode steps with CUDA events (graph replay + host work per
step), reports ms per step, the host share, and the per-kernel device time of
one profiled step.  Prints one JSON line.
"""

from __future__ import annotations

import argparse
import json
import time

import torch


def main(argv=None) -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--model", default="qwen3-4b")
    ap.add_argument("--batch", type=int, default=64)
    ap.add_argument("--prompt", type=int, default=300)
    ap.add_argument("--steps", type=int, default=200)
    ap.add_argument("--max-len", type=int, default=5136)
    a = ap.parse_args(argv)
    from libra_b200.engine.rollout.kv_cache import PagedKVCache
    from libra_b200.engine.rollout.llm_engine import LLMEngine
    from libra_b200.engine.rollout.sampler import SamplingParams
    from libra_b200.models.qwen3 import ParamLayout, get_config, init_params, param_shapes

    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    cfg = get_config(a.model)
    lay = ParamLayout(param_shapes(cfg))
    flat = torch.empty(lay.numel, dtype=torch.bfloat16, device=dev)
    views = lay.views(flat)
    init_params(cfg, views, seed=0)
    blocks = a.batch * (-(-a.max_len // 16)) + 64
    llm = LLMEngine(cfg, views, kv_blocks=blocks, block_size=16, max_model_len=a.max_len, max_running=128,
                    max_batch_tokens=16384, flat=flat)
    g = torch.Generator().manual_seed(0)
    prompts = [torch.randint(4, cfg.vocab_size, (a.prompt,), generator=g).tolist() for _ in range(a.batch)]
    total = a.steps + 40
    ids = [llm.add_request(p, SamplingParams(max_tokens=total, temperature=1.0)) for p in prompts]
    # prefill + a few decode steps (graph capture happens at the first decode step)
    for _ in range(10):
        llm.step()
    torch.cuda.synchronize()
    host = 0.0
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    t0 = time.perf_counter()
    e0.record()
    for _ in range(a.steps):
        h0 = time.perf_counter()
        llm.step()
        host += time.perf_counter() - h0
    e1.record()
    torch.cuda.synchronize()
    wall = (time.perf_counter() - t0) * 1e3 / a.steps
    ms = e0.elapsed_time(e1) / a.steps
    g_ = llm._graphs
    # the same captured step replayed back to back with no host work in between: the device's share
    graph_ms = None
    if g_ is not None and llm.running:
        b = g_.bucket(len(llm.running))
        for _ in range(3):
            g_.graphs[b].replay()
        torch.cuda.synchronize()
        e2, e3 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e2.record()
        for _ in range(50):
            g_.graphs[b].replay()
        e3.record()
        torch.cuda.synchronize()
        graph_ms = e2.elapsed_time(e3) / 50
        g_.reset_accumulators()
    # one decode step under the profiler: per-kernel device time
    from torch.profiler import ProfilerActivity, profile

    with profile(activities=[ProfilerActivity.CUDA]) as prof:
        llm.step()
        torch.cuda.synchronize()
    kern = {}
    for ev in prof.events():
        if ev.device_type == torch.autograd.DeviceType.CUDA:
            k = ev.name.split("(")[0][:60]
            kern[k] = kern.get(k, 0.0) + ev.device_time_total / 1e3
    top = dict(sorted(((k, round(v, 4)) for k, v in kern.items()), key=lambda kv: -kv[1])[:15])
    ctx = a.prompt + 10 + a.steps
    kv_bytes = a.batch * ctx * cfg.num_hidden_layers * cfg.num_key_value_heads * cfg.head_dim * 2 * 2
    print(json.dumps({"model": a.model, "batch": a.batch, "context_at_end": ctx, "ms_per_step": round(ms, 3),
                      "wall_ms_per_step": round(wall, 3), "host_ms_per_step": round(host * 1e3 / a.steps, 3),
                      "graph_only_ms_per_step": round(graph_ms, 3) if graph_ms is not None else None,
                      "graph_replays": g_.replays if g_ else 0, "weights_gb": flat.numel() * 2 / 1e9,
                      "kv_gb_per_step_at_end": kv_bytes / 1e9, "profiled_step_kernels_ms": top,
                      "profiled_step_device_ms": round(sum(kern.values()), 3)}), flush=True)


if __name__ == "__main__":
    main()
