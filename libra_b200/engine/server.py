"""OpenAI-compatible HTTP front end for one rollout instance.

Routes (the reference serves the same ones from a patched vLLM API server,
``scripts/vllm_hot_reload_api_server.py:41-96``):

* ``POST /v1/completions`` - ``prompt`` as text or token ids, ``max_tokens``,
  ``temperature``, ``top_p``, ``top_k``, ``seed``, ``logprobs``; the choice
  carries ``text``, ``token_ids``, ``prompt_token_ids``,
  ``logprobs.tokens/token_logprobs`` and ``finish_reason``.
* ``GET /health``, ``GET /v1/models``, ``GET /metrics``.
* ``POST /reload_weights`` ``{"checkpoint_path": dir, "version": v}`` - load a
  checkpoint written by the trainer (disk weight sync), under a lock, then drop
  the prefix cache.
* ``POST /reload_weights_peer`` ``{"src_tp": k, "sources": [...], "version": v}``
  - map the trainer ranks' exported flat weight buffers (JSON descriptions of
  CUDA IPC handles, no pickled objects) and reshard this rank's slice into the
  served weights in place with the ``weight_reshard`` kernel (peer-memory
  weight sync).
* ``POST /import_kv`` ``{"path", "tokens", "version", ...}`` - prefix-cache the
  KV blocks another engine exported (``LLMEngine.export_prefix``, a
  safetensors file); with TP every rank takes its own KV heads (C-MLFQ
  migration of a multi-turn request into this instance).

    python -m libra_b200.engine.server --model qwen3-4b --device cuda:4 --port 8000
"""

from __future__ import annotations

import argparse
import asyncio
import json
import os
import time
import uuid
from typing import Any, Dict, Optional

from aiohttp import web

from libra_b200.engine.rollout.sampler import SamplingParams


def build_app(engine, tokenizer, model_name: str = "libra", weight_loader=None) -> web.Application:
    """``engine``: an LLMEngine; ``weight_loader(request_json) -> (params dict, version)``."""
    app = web.Application(client_max_size=64 * 1024 * 1024)
    reload_lock = asyncio.Lock()
    engine.start()

    async def health(_):
        return web.json_response({"status": "ok", "version": engine.version, "instance": engine.instance_id})

    async def models(_):
        return web.json_response({"object": "list", "data": [{"id": model_name, "object": "model"}]})

    async def metrics(_):
        return web.json_response({**engine.stats, **engine.load(), "version": engine.version})

    async def completions(request: web.Request):
        body = await request.json()
        prompt = body.get("prompt", "")
        if isinstance(prompt, list) and prompt and isinstance(prompt[0], list):
            prompt = prompt[0]
        ids = tokenizer.encode(prompt, add_special_tokens=False) if isinstance(prompt, str) else [int(t) for t in prompt]
        stops = list(body.get("stop_token_ids") or [])
        eos = getattr(tokenizer, "eos_token_id", None)
        if eos is not None and eos not in stops and not body.get("ignore_eos", False):
            stops.append(int(eos))
        params = SamplingParams(max_tokens=int(body.get("max_tokens", 16)), temperature=float(body.get("temperature", 1.0)),
                                top_p=float(body.get("top_p", 1.0)), top_k=int(body.get("top_k", -1)),
                                stop_token_ids=stops, seed=body.get("seed"))
        n = max(1, int(body.get("n", 1)))
        results = await asyncio.gather(*(engine.generate(ids, params) for _ in range(n)))
        choices = []
        for i, r in enumerate(results):
            choice = {"index": i, "text": tokenizer.decode(r.output_tokens), "token_ids": r.output_tokens,
                      "prompt_token_ids": ids, "finish_reason": r.finish_reason}
            if body.get("logprobs") is not None:
                choice["logprobs"] = {"tokens": [str(t) for t in r.output_tokens], "token_logprobs": r.output_logprobs}
            choices.append(choice)
        comp = sum(len(r.output_tokens) for r in results)
        return web.json_response({"id": f"cmpl-{uuid.uuid4().hex[:12]}", "object": "text_completion",
                                  "created": int(time.time()), "model": body.get("model") or model_name,
                                  "choices": choices, "usage": {"prompt_tokens": len(ids), "completion_tokens": comp,
                                                                "total_tokens": len(ids) + comp}})

    async def reload(request: web.Request, kind: str):
        if weight_loader is None:
            return web.json_response({"error": "no weight loader configured"}, status=400)
        body = await request.json()
        async with reload_lock:
            t0 = time.perf_counter()
            req = dict(body, kind=kind)
            loop = asyncio.get_running_loop()
            if kind == "peer":
                # in-place reshard into the live weight buffers: runs while the engine is paused
                await loop.run_in_executor(None, lambda: engine.update_weights(
                    {}, req.get("version"), reload_request=req, apply=lambda: weight_loader(req)))
            else:
                params, version = await loop.run_in_executor(None, weight_loader, req)
                if params:
                    await loop.run_in_executor(None, lambda: engine.update_weights(params, version, reload_request=req))
            return web.json_response({"status": "ok", "version": engine.version, "seconds": time.perf_counter() - t0})

    async def import_kv(request: web.Request):
        body = await request.json()
        if not isinstance(body.get("path"), str) or not isinstance(body.get("tokens"), list):
            return web.json_response({"error": "import_kv needs path and tokens"}, status=400)
        loop = asyncio.get_running_loop()
        try:
            n = await loop.run_in_executor(None, engine.import_prefix, body)
        except (OSError, ValueError, KeyError) as exc:
            return web.json_response({"error": str(exc)}, status=400)
        return web.json_response({"status": "ok", "tokens": int(n)})

    app.router.add_get("/health", health)
    app.router.add_get("/v1/models", models)
    app.router.add_get("/metrics", metrics)
    app.router.add_post("/v1/completions", completions)
    app.router.add_post("/reload_weights", lambda r: reload(r, "disk"))
    app.router.add_post("/reload_weights_peer", lambda r: reload(r, "peer"))
    app.router.add_post("/reload_weights_nccl", lambda r: reload(r, "peer"))
    app.router.add_post("/import_kv", import_kv)
    return app


class BackgroundServer:
    """Runs an app on its own event-loop thread (tests, in-process instances)."""

    def __init__(self, app: web.Application, host: str = "127.0.0.1", port: int = 0):
        import threading

        self.app, self.host, self.port = app, host, port
        self._loop = asyncio.new_event_loop()
        self._ready = threading.Event()
        self._thread = threading.Thread(target=self._run, daemon=True, name="rollout-http")
        self._thread.start()
        self._ready.wait(30)

    def _run(self) -> None:
        asyncio.set_event_loop(self._loop)
        self._runner = web.AppRunner(self.app)
        self._loop.run_until_complete(self._runner.setup())
        site = web.TCPSite(self._runner, self.host, self.port)
        self._loop.run_until_complete(site.start())
        self.port = site._server.sockets[0].getsockname()[1]
        self._ready.set()
        self._loop.run_forever()

    def stop(self) -> None:
        async def _down():
            await self._runner.cleanup()

        fut = asyncio.run_coroutine_threadsafe(_down(), self._loop)
        try:
            fut.result(10)
        finally:
            self._loop.call_soon_threadsafe(self._loop.stop)
            self._thread.join(10)


def main(argv=None) -> None:
    import torch

    from libra_b200.engine.checkpointing import load_params_into
    from libra_b200.engine.rollout.llm_engine import LLMEngine
    from libra_b200.engine.tokenizer import load_tokenizer
    from libra_b200.engine.train_engine import B200TrainEngine

    ap = argparse.ArgumentParser(description="libra_b200 rollout server")
    ap.add_argument("--model", default="qwen3-4b")
    ap.add_argument("--checkpoint", default="")
    ap.add_argument("--tokenizer", default="")
    ap.add_argument("--device", default="cuda:0")
    ap.add_argument("--host", default="127.0.0.1")
    ap.add_argument("--port", type=int, default=8000)
    ap.add_argument("--kv-memory-fraction", type=float, default=0.8)
    ap.add_argument("--max-batch-tokens", type=int, default=8192)
    ap.add_argument("--tp", type=int, default=1, help="tensor-parallel degree (one process per GPU via torchrun)")
    a = ap.parse_args(argv)
    tp_group = channel = None
    rank = 0
    device = a.device
    if a.tp > 1:  # launched by torch.distributed.run, one process per GPU of the instance
        import datetime

        import torch.distributed as dist

        local = int(os.environ.get("LOCAL_RANK", "0"))
        if a.device == "cpu" or not torch.cuda.is_available():  # CPU ranks (tests): gloo, fp32 reference ops
            device = "cpu"
            dist.init_process_group("gloo", timeout=datetime.timedelta(seconds=600))
        else:
            torch.cuda.set_device(local)
            device = f"cuda:{local}"
            dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=600),
                                    device_id=torch.device("cuda", local))
        if dist.get_world_size() != a.tp:
            raise SystemExit(f"--tp {a.tp} needs exactly {a.tp} processes, got {dist.get_world_size()}")
        rank, tp_group = dist.get_rank(), dist.group.WORLD
        channel = dist.new_group(backend="gloo")
    holder = B200TrainEngine(a.model, device=device, use_distributed_optimizer=False, tp_size=a.tp)
    holder.initialize()
    holder.release_optimizer_state()

    def load_disk(path: str) -> Dict[str, torch.Tensor]:
        params = {k: v.clone() for k, v in holder.params.items()}
        if a.tp == 1:
            load_params_into(params, path)
            return params
        from libra_b200.models.qwen3 import ParamLayout, param_shapes
        from libra_b200.parallel.tensor_parallel import shard_full_params

        layout = ParamLayout(param_shapes(holder.cfg))  # full (TP=1) shapes, on the host
        full = layout.views(torch.empty(layout.numel, dtype=torch.bfloat16))
        load_params_into(full, path, cfg=holder.cfg)
        for k, v in shard_full_params(full, holder.cfg, a.tp, holder.tp_rank).items():
            params[k].copy_(v)
        return params

    if a.checkpoint:
        for k, v in load_disk(a.checkpoint).items():
            holder.params[k].data.copy_(v)
    tok = load_tokenizer(a.tokenizer or a.checkpoint, holder.cfg.vocab_size)
    llm = LLMEngine(holder.cfg, {k: v.detach() for k, v in holder.params.items()},
                    kv_memory_fraction=a.kv_memory_fraction, max_batch_tokens=a.max_batch_tokens,
                    instance_id=f"{a.host}:{a.port}", eos_token_id=getattr(tok, "eos_token_id", None),
                    tp_group=tp_group, tp_size=a.tp, tp_channel=channel)

    def loader(req: Dict[str, Any]):
        if req.get("kind") == "disk":
            return load_disk(req["checkpoint_path"]), req.get("version")
        from libra_b200.infra.sync.peer_weight_sync import receive_peer_weights

        # this rank's slice for its own TP degree and rank, written in place into the served weights
        receive_peer_weights(req, holder.flat_param, holder.cfg, a.tp, holder.tp_rank)
        return {}, req.get("version")

    if rank > 0:
        llm.tp_reload_hook = loader
        llm.follower_loop()
        return
    web.run_app(build_app(llm, tok, a.model, loader), host=a.host, port=a.port)


if __name__ == "__main__":
    main()
