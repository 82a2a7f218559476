"""Continuous-batching generation engine (the rollout side of libra_b200).

Replaces the vLLM server processes of the reference with an in-process engine
per rollout instance:

* requests wait in a FIFO; each ``step`` admits waiting requests while the
  prefill token budget and KV blocks allow (prefix-cached blocks are reused),
  then runs one mixed batch: prefill/extend tokens of admitted requests plus one
  decode token for every running request;
* sampling (temperature / top-p / top-k, per-request seed) returns the sampled
  token's logprob, as vLLM does with ``logprobs=1``;
* a request finishes on a stop token, ``max_tokens`` or the context limit; its
  KV blocks return to the cache as reusable prefix blocks;
* ``generate`` is a coroutine: the step loop runs on a background thread and
  resolves per-request asyncio futures thread-safely;
* ``update_weights`` swaps in new weights between steps (in-place copy, or a
  new parameter dict) and drops the prefix cache, which is stale afterwards;
  ``pause`` / ``resume`` bracket weight updates.
"""

from __future__ import annotations

import asyncio
import itertools
import threading
import time
import uuid
from collections import deque
from dataclasses import dataclass, field
from typing import Deque, Dict, List, Optional

import torch

from libra_b200 import ops
from libra_b200.engine.rollout.kv_cache import PagedKVCache
from libra_b200.engine.rollout.runner import InferenceRunner, WorkItem
from libra_b200.engine.rollout.sampler import SamplingParams, sample
from libra_b200.models.qwen3 import Qwen3Config
from libra_b200.utils import nvtx


@dataclass
class GenerationResult:
    request_id: str
    prompt_tokens: List[int]
    output_tokens: List[int]
    output_logprobs: List[float]
    finish_reason: str
    metrics: Dict[str, float] = field(default_factory=dict)


@dataclass
class _Request:
    request_id: str
    prompt: List[int]
    params: SamplingParams
    out: List[int] = field(default_factory=list)
    logprobs: List[float] = field(default_factory=list)
    cached: int = 0           # tokens whose KV is in the cache
    future: Optional[asyncio.Future] = None
    loop: Optional[asyncio.AbstractEventLoop] = None
    callback: Optional[object] = None
    generator: Optional[torch.Generator] = None
    t_arrive: float = field(default_factory=time.perf_counter)
    t_first: float = 0.0
    seed: int = 0             # sampler key of the captured decode path

    @property
    def tokens(self) -> List[int]:
        return self.prompt + self.out

    @property
    def n_tokens(self) -> int:
        return len(self.prompt) + len(self.out)

    def token_slice(self, a: int, b: int) -> List[int]:
        P = len(self.prompt)
        if b <= P:
            return self.prompt[a:b]
        if a >= P:
            return self.out[a - P:b - P]
        return self.prompt[a:] + self.out[:b - P]


class LLMEngine:
    def __init__(self, cfg: Qwen3Config, params: Dict[str, torch.Tensor], *, kv_blocks: int = 0,
                 block_size: int = 16, kv_memory_fraction: float = 0.5, max_batch_tokens: int = 8192,
                 max_running: int = 256, max_model_len: int = 0, instance_id: str = "", tp_group=None,
                 tp_size: int = 1, eos_token_id: Optional[int] = None, tp_channel=None,
                 flat: Optional[torch.Tensor] = None):
        """``tp_size > 1``: one engine per TP rank.  TP rank 0 (the driver)
        schedules, samples and serves; the other ranks run ``follower_loop``
        and replay, step by step, the driver's KV-cache operations and model
        steps, which it broadcasts over ``tp_channel`` (a gloo group)."""
        self.cfg = cfg
        self.params = params
        self.flat = flat  # optional single buffer that every parameter views (one-copy weight sync)
        self.device = next(iter(params.values())).device
        self.instance_id = instance_id or f"engine-{uuid.uuid4().hex[:6]}"
        nkv = max(1, cfg.num_key_value_heads // tp_size)
        if kv_blocks <= 0:
            if self.device.type == "cuda":
                free, _ = torch.cuda.mem_get_info(self.device)
                budget = free * kv_memory_fraction
            else:
                budget = 256 * 1024 * 1024
            kv_blocks = PagedKVCache.blocks_for_budget(budget, cfg.num_hidden_layers, block_size, nkv, cfg.head_dim)
        self.kv = PagedKVCache(cfg.num_hidden_layers, kv_blocks, block_size, nkv, cfg.head_dim, self.device,
                               next(iter(params.values())).dtype)
        # a step carries at most the prefill budget plus one decode token per running sequence (a single
        # longer prompt falls back to the unfused all-reduce for its step)
        self.runner = InferenceRunner(cfg, params, self.kv, tp_group, tp_size,
                                      max_step_tokens=max_batch_tokens + max_running)
        self.max_batch_tokens = max_batch_tokens
        self.max_running = max_running
        self.max_model_len = max_model_len or cfg.max_position_embeddings
        self.eos_token_id = eos_token_id
        self.waiting: Deque[_Request] = deque()
        self.running: List[_Request] = []
        self._lock = threading.Lock()
        self._wake = threading.Event()
        self._paused = threading.Event()
        self._idle = threading.Event()
        self._idle.set()
        self._stop = threading.Event()
        self._thread: Optional[threading.Thread] = None
        self.version = 0
        self.stats = {"steps": 0, "prefill_tokens": 0, "decode_tokens": 0, "cached_prefix_tokens": 0,
                      "finished": 0, "busy_s": 0.0}
        self._eager_io = {"h2d": 0, "d2h": 0}  # host<->device bytes of the eager (prefill/extend) steps
        self._ids = itertools.count()
        self.tp_size, self.tp_group, self.tp_channel = tp_size, tp_group, tp_channel
        self.tp_rank = 0
        self._tp_src = 0
        if tp_size > 1:
            import torch.distributed as dist

            self.tp_rank = dist.get_rank(tp_group)
            self._tp_src = dist.get_global_rank(tp_channel, 0) if tp_channel is not None else 0
        self._kv_ops: List[tuple] = []  # KV-cache calls the followers must replay, in order
        self.tp_reload_hook = None  # follower side: callable(request) -> (params, version)
        self.block_size = block_size
        self._graphs = None          # DecodeGraphs, built at the first pure-decode step
        self._graphs_ok = (self.device.type == "cuda" and tp_size == 1 and not cfg.is_moe and cfg.head_dim == 128)
        self._seed_rng = torch.Generator().manual_seed(int(uuid.uuid4().int & 0x7FFFFFFF))

    # ------------------------------------------------------------------ tensor-parallel replay
    def _kv_call(self, op: str, *args):
        """Apply a scheduler-side KV-cache call and record it for the followers."""
        if self.tp_size > 1:
            self._kv_ops.append((op, args))
        if op == "match_prefix":
            return self.kv.match_prefix(*args)
        if op == "free":
            return self.kv.free(*args)
        if op == "clear_cache":
            return self.kv.alloc.clear_cache()
        raise ValueError(op)

    def _broadcast_plan(self, plan: Dict) -> Dict:
        import torch.distributed as dist

        box = [plan]
        dist.broadcast_object_list(box, src=self._tp_src, group=self.tp_channel)
        return box[0]

    def _publish(self, items=None, **extra) -> None:
        if self.tp_size > 1 and self.tp_rank == 0:
            ops, self._kv_ops = self._kv_ops, []
            self._broadcast_plan({"ops": ops, "items": [(i.seq_id, list(i.tokens), i.start) for i in items or []],
                                  **extra})

    def follower_loop(self) -> None:
        """TP rank > 0: replay the driver's steps until it broadcasts a stop."""
        if self.device.type == "cuda":
            torch.cuda.set_device(self.device)
        while True:
            plan = self._broadcast_plan({})
            if plan.get("reload") is not None and self.tp_reload_hook is not None:
                params, version = self.tp_reload_hook(plan["reload"])
                if params:
                    with torch.no_grad():
                        for k, v in params.items():
                            self.params[k].copy_(v)
                if version is not None:
                    self.version = int(version)
            for op, args in plan.get("ops", []):
                getattr(self.kv, op)(*args) if op != "clear_cache" else self.kv.alloc.clear_cache()
            if plan.get("import_kv") is not None:
                try:
                    self._import_prefix_local(plan["import_kv"])
                except (OSError, ValueError, KeyError) as exc:  # the leader hit the same check and reports it
                    print(f"KV import skipped on TP rank {self.tp_rank}: {exc}")
            if plan.get("items"):
                self.runner.step([WorkItem(rid, toks, start) for rid, toks, start in plan["items"]])
            if plan.get("stop"):
                return

    # ------------------------------------------------------------------ request API
    def add_request(self, prompt_tokens: List[int], params: SamplingParams, request_id: str = "",
                    future=None, loop=None, callback=None) -> str:
        rid = request_id or f"{self.instance_id}-{next(self._ids)}"
        gen = None
        if params.seed is not None:
            gen = torch.Generator(device=self.device)
            gen.manual_seed(int(params.seed))
        req = _Request(rid, list(int(t) for t in prompt_tokens), params, future=future, loop=loop, callback=callback,
                       generator=gen)
        req.seed = int(params.seed) if params.seed is not None else int(
            torch.randint(0, 2 ** 62, (1,), generator=self._seed_rng))
        with self._lock:
            self.waiting.append(req)
            self._idle.clear()
        self._wake.set()
        return rid

    async def generate(self, prompt_tokens: List[int], params: Optional[SamplingParams] = None,
                       request_id: str = "") -> GenerationResult:
        loop = asyncio.get_running_loop()
        fut = loop.create_future()
        self.start()
        self.add_request(prompt_tokens, params or SamplingParams(), request_id, future=fut, loop=loop)
        return await fut

    def generate_sync(self, prompts: List[List[int]], params=None) -> List[GenerationResult]:
        """Blocking batch generation on the calling thread (no background loop).
        ``params``: one ``SamplingParams`` for every prompt, or a list with one per prompt."""
        results: Dict[str, GenerationResult] = {}
        plist = params if isinstance(params, (list, tuple)) else [params] * len(prompts)
        if len(plist) != len(prompts):
            raise ValueError("generate_sync: one SamplingParams per prompt")
        ids = [self.add_request(p, sp or SamplingParams(), callback=lambda r: results.__setitem__(r.request_id, r))
               for p, sp in zip(prompts, plist)]
        while len(results) < len(ids):
            self.step()
        return [results[i] for i in ids]

    # ------------------------------------------------------------------ background loop
    def start(self) -> None:
        if self._thread is not None and self._thread.is_alive():
            return
        self._stop.clear()
        self._thread = threading.Thread(target=self._loop, daemon=True, name=f"llm-{self.instance_id}")
        self._thread.start()

    def shutdown(self) -> None:
        self._stop.set()
        self._wake.set()
        if self._thread is not None:
            self._thread.join(timeout=10)
        self._publish(stop=True)

    def _loop(self) -> None:
        if self.device.type == "cuda":
            torch.cuda.set_device(self.device)
        while not self._stop.is_set():
            if self._paused.is_set() or (not self.waiting and not self.running):
                self._idle.set()
                self._wake.wait(timeout=0.05)
                self._wake.clear()
                continue
            try:
                self.step()
            except Exception as exc:  # noqa: BLE001 - fail every in-flight request, keep serving
                self._fail_all(exc)

    def _fail_all(self, exc: Exception) -> None:
        with self._lock:
            reqs = list(self.running) + list(self.waiting)
            self.running.clear()
            self.waiting.clear()
        for r in reqs:
            self._kv_call("free", r.request_id)
            if r.future is not None and r.loop is not None:
                r.loop.call_soon_threadsafe(lambda f=r.future: f.done() or f.set_exception(RuntimeError(str(exc))))

    def pause(self, timeout: float = 600.0) -> None:
        """Stop stepping after the current step (requests stay queued)."""
        self._paused.set()
        deadline = time.monotonic() + timeout
        while self._thread is not None and self._thread.is_alive() and not self._idle.is_set():
            if time.monotonic() > deadline:
                raise TimeoutError("engine did not pause in time")
            time.sleep(0.005)

    def resume(self) -> None:
        self._paused.clear()
        self._wake.set()

    def wait_until_idle(self, timeout: float = 3600.0) -> None:
        deadline = time.monotonic() + timeout
        while self.waiting or self.running:
            if time.monotonic() > deadline:
                raise TimeoutError("engine still has requests")
            time.sleep(0.01)

    # ------------------------------------------------------------------ weights
    @torch.no_grad()
    def update_weights(self, new_params: Dict[str, torch.Tensor], version: Optional[int] = None,
                       copy: bool = True, reload_request: Optional[Dict] = None, apply=None) -> None:
        """Install new weights between steps (copy into the existing buffers, or rebind;
        ``apply()``, when given, writes the buffers in place while the engine is paused).

        With TP, ``reload_request`` is forwarded to the followers, which load
        their own shards through ``tp_reload_hook``; the driver's loop is paused
        first, so the broadcast cannot interleave with a step's."""
        was_paused = self._paused.is_set()
        self.pause()
        try:
            if self.tp_size > 1 and reload_request is not None:
                self._publish(reload=reload_request)
            if apply is not None:  # caller-supplied in-place writer (peer reshard into the live buffers)
                apply()
            if copy:
                for k, v in new_params.items():
                    self.params[k].copy_(v, non_blocking=True)
                if self.device.type == "cuda":
                    torch.cuda.current_stream(self.device).synchronize()
            else:
                self.params = new_params
                self.runner.p = new_params
                self._graphs = None  # the captured steps read the old buffers
            self._kv_call("clear_cache")
            if version is not None:
                self.version = int(version)
        finally:
            if not was_paused:
                self.resume()

    @torch.no_grad()
    def load_flat_weights(self, src_flat: torch.Tensor, version: Optional[int] = None) -> float:
        """Weight sync from a trainer that keeps its parameters in one flat bf16
        buffer with this engine's layout: a single device copy (an NVLink peer
        copy when ``src_flat`` lives on another GPU).  Returns seconds."""
        if self.flat is None or self.flat.numel() != src_flat.numel():
            raise ValueError("load_flat_weights needs an engine built on a flat buffer of the trainer's layout")
        t0 = time.perf_counter()
        was_paused = self._paused.is_set()
        self.pause()
        try:
            self.flat.copy_(src_flat, non_blocking=True)
            if self.device.type == "cuda":
                torch.cuda.current_stream(self.device).synchronize()
            self._kv_call("clear_cache")
            if version is not None:
                self.version = int(version)
        finally:
            if not was_paused:
                self.resume()
        return time.perf_counter() - t0

    @torch.no_grad()
    def migrate_prefix_to(self, other: "LLMEngine", tokens: List[int]) -> int:
        """Copy this engine's cached KV of ``tokens``'s prefix into ``other``'s
        cache (the next turn of a migrated multi-turn request then starts from
        that prefix instead of recomputing it).  Both engines pause for the
        copy; engines on different weight versions do not exchange KV.
        Returns the prefix tokens now cached on ``other``."""
        if other is self or self.version != other.version or self.tp_size != 1 or other.tp_size != 1:
            return 0
        pauses = [(e, e._paused.is_set()) for e in (self, other)]
        for e, _ in pauses:
            e.pause()
        try:
            n = other.kv.import_blocks(self.kv, self.kv.cached_blocks(list(tokens)))
            if other.device.type == "cuda":
                torch.cuda.synchronize(other.device)
        finally:
            for e, was in pauses:
                if not was:
                    e.resume()
        self.stats["migrated_out_tokens"] = self.stats.get("migrated_out_tokens", 0) + n
        return n

    def export_prefix(self, tokens: List[int], path: str) -> Dict:
        """Write this engine's cached KV of ``tokens``'s prefix to ``path``
        (safetensors: ``k`` and ``v`` as [layers, blocks, block_size, kv_heads,
        head_dim]) for another process's engine to import (``import_prefix``);
        returns the JSON request that describes it."""
        from safetensors.torch import save_file

        if self.tp_size != 1:
            raise ValueError("KV export needs a single-rank engine (all KV heads in one cache)")
        was_paused = self._paused.is_set()
        self.pause()
        try:
            blocks = self.kv.cached_blocks(list(tokens))
            k, v = self.kv.export_blocks(blocks)
            save_file({"k": k.contiguous().cpu(), "v": v.contiguous().cpu()}, path)
        finally:
            if not was_paused:
                self.resume()
        n = len(blocks) * self.kv.block_size
        return {"path": path, "tokens": [int(t) for t in tokens[:n]], "version": int(self.version),
                "block_size": self.kv.block_size, "num_layers": self.kv.num_layers,
                "kv_heads": self.cfg.num_key_value_heads, "head_dim": self.kv.head_dim}

    def import_prefix(self, request: Dict) -> int:
        """Prefix-cache KV exported by ``export_prefix`` (another process's
        engine at the same weight version); with TP every rank imports its own
        KV heads, in step with the leader.  Returns the prefix tokens now cached."""
        was_paused = self._paused.is_set()
        self.pause()
        try:
            if self.tp_size > 1:
                self._publish(import_kv=request)
            return self._import_prefix_local(request)
        finally:
            if not was_paused:
                self.resume()

    def _import_prefix_local(self, request: Dict) -> int:
        from safetensors.torch import load_file

        kv, cfg = self.kv, self.cfg
        if int(request.get("version", -1)) != int(self.version):
            return 0  # KV of other weights would be wrong here
        if (int(request["block_size"]), int(request["num_layers"]), int(request["kv_heads"]),
                int(request["head_dim"])) != (kv.block_size, kv.num_layers, cfg.num_key_value_heads, kv.head_dim):
            raise ValueError("exported KV does not match this engine's model or block size")
        data = load_file(str(request["path"]), device=str(self.device))
        k, v = data["k"], data["v"]
        if self.tp_size > 1:  # this rank's KV heads (neighbouring ranks share a head when tp > kv heads)
            kv0 = self.tp_rank * cfg.num_key_value_heads // self.tp_size
            k = k[:, :, :, kv0:kv0 + kv.kv_heads]
            v = v[:, :, :, kv0:kv0 + kv.kv_heads]
        n = kv.import_block_tensors([int(t) for t in request["tokens"]], k, v)
        self.stats["migrated_in_tokens"] = self.stats.get("migrated_in_tokens", 0) + n
        return n

    # ------------------------------------------------------------------ scheduling
    def _admit(self) -> List[_Request]:
        admitted, budget = [], self.max_batch_tokens - len(self.running)
        with self._lock:
            while self.waiting and len(self.running) + len(admitted) < self.max_running:
                r = self.waiting[0]
                if not r.cached and r.request_id not in self.kv.seqs:
                    r.cached = self._kv_call("match_prefix", r.request_id, r.prompt)
                    self.stats["cached_prefix_tokens"] += r.cached
                need = len(r.tokens) - r.cached
                if admitted and need > budget:
                    break
                if not self.kv.can_reserve(r.request_id, len(r.tokens) + 1):
                    if not admitted and not self.running:
                        self.waiting.popleft()
                        self._finish(r, "kv_cache_exhausted")
                        continue
                    break
                self.waiting.popleft()
                admitted.append(r)
                budget -= need
        return admitted

    def _graph_runner(self):
        if self._graphs is None and self._graphs_ok:
            from libra_b200.engine.rollout.decode_graph import DecodeGraphs, graphs_enabled

            if not graphs_enabled():
                self._graphs_ok = False
                return None
            self._graphs = DecodeGraphs(self.runner, max_batch=self.max_running, max_model_len=self.max_model_len)
            self._graphs.capture()
        return self._graphs

    def _decode_step_graph(self, decode: List[_Request], t0: float) -> int:
        """Pure-decode step through the captured graphs (plain temperature sampling)."""
        g = self._graph_runner()
        bs = self.block_size
        for i, r in enumerate(decode):
            L = r.cached + 1
            self.kv.reserve(r.request_id, L)
            g.set_row(i, r.request_id, r.out[-1], L, r.params.temperature, r.seed)
        with nvtx.nvtx_range("decode"):
            toks, lps = g.run(len(decode))
        now = time.perf_counter()
        self.stats["decode_tokens"] += len(decode)
        done = False
        for r, t, lp in zip(decode, toks, lps):
            L = r.cached + 1
            r.cached = L
            self.kv.commit_block(r.request_id, L, r.token_slice(L - bs, L) if L % bs == 0 else [])
            r.out.append(t)
            r.logprobs.append(lp)
            if not r.t_first:
                r.t_first = now
            reason = self._stop_reason(r, t)
            if reason:
                self._finish(r, reason)
                r.cached = -1
                done = True
        if done:
            self.running = [r for r in self.running if r.cached >= 0]
        self.stats["steps"] += 1
        self.stats["busy_s"] += time.perf_counter() - t0
        return len(decode)

    def step(self) -> int:
        t0 = time.perf_counter()
        admitted = self._admit()
        decode = [r for r in self.running if r.cached == r.n_tokens - 1]
        if (not admitted and decode and self._graphs_ok and len(decode) <= self.max_running
                and all(r.params.top_p >= 1.0 and r.params.top_k <= 0 for r in decode)
                and self._graph_runner() is not None):
            return self._decode_step_graph(decode, t0)
        batch = admitted + decode
        if not batch:
            return 0
        items = [WorkItem(r.request_id, r.tokens, r.cached) for r in batch]
        self._publish(items)
        with nvtx.nvtx_range("prefill" if admitted else "decode"):
            logits = self.runner.step(items)
        if logits.device.type == "cuda":
            # the fused samplers (same Philox stream as the captured decode steps); their per-request inputs
            # go up through pinned staging, so the host does not wait for the step's kernels here
            from libra_b200.engine.rollout.runner import _to_device

            dev = logits.device
            temps = _to_device([r.params.temperature for r in batch], torch.float32, dev)
            seeds = _to_device([r.seed for r in batch], torch.long, dev)
            pos = _to_device([r.n_tokens - 1 for r in batch], torch.long, dev)
            toks = torch.empty(len(batch), dtype=torch.long, device=dev)
            lps = torch.empty(len(batch), dtype=torch.float32, device=dev)
            if all(r.params.top_p >= 1.0 and r.params.top_k <= 0 for r in batch):
                ops.sample_tokens(logits.contiguous(), temps, seeds, pos, toks, lps)
            else:
                top_p = _to_device([r.params.top_p for r in batch], torch.float32, dev)
                top_k = _to_device([r.params.top_k for r in batch], torch.long, dev)
                ops.sample_tokens_filtered(logits.contiguous(), temps, top_p, top_k, seeds, pos, toks, lps)
        else:
            temps = torch.tensor([r.params.temperature for r in batch], dtype=torch.float32)
            top_p = torch.tensor([r.params.top_p for r in batch], device=logits.device, dtype=torch.float32)
            top_k = torch.tensor([r.params.top_k for r in batch], device=logits.device, dtype=torch.long)
            gens = [r.generator for r in batch] if any(r.generator is not None for r in batch) else None
            toks, lps = sample(logits, temps, top_p, top_k, gens)
        toks, lps = toks.tolist(), lps.tolist()
        n_new = sum(r.n_tokens - r.cached for r in batch)
        self._eager_io["h2d"] += 28 * n_new + 32 * len(batch)  # tokens, positions, slots, rows, sampler inputs
        self._eager_io["d2h"] += 12 * len(batch)
        now = time.perf_counter()
        self.stats["prefill_tokens"] += sum(len(r.tokens) - r.cached for r in admitted)
        self.stats["decode_tokens"] += len(decode)
        still = []
        for r, t, lp in zip(batch, toks, lps):
            r.cached = len(r.tokens)
            r.out.append(int(t))
            r.logprobs.append(float(lp))
            if not r.t_first:
                r.t_first = now
            reason = self._stop_reason(r, int(t))
            if reason:
                self._finish(r, reason)
            else:
                still.append(r)
        keep = {id(r) for r in still}
        self.running = [r for r in self.running if id(r) in keep] + [r for r in admitted if id(r) in keep]
        self.stats["steps"] += 1
        self.stats["busy_s"] += time.perf_counter() - t0
        return len(batch)

    def _stop_reason(self, r: _Request, tok: int) -> str:
        if tok in r.params.stop_token_ids or (self.eos_token_id is not None and tok == self.eos_token_id):
            return "stop"
        if len(r.out) >= r.params.max_tokens:
            return "length"
        if r.n_tokens >= self.max_model_len:
            return "length"
        return ""

    def _finish(self, r: _Request, reason: str) -> None:
        self._kv_call("free", r.request_id)
        self.stats["finished"] += 1
        res = GenerationResult(r.request_id, r.prompt, list(r.out), list(r.logprobs), reason,
                               {"ttft_s": (r.t_first - r.t_arrive) if r.t_first else 0.0,
                                "latency_s": time.perf_counter() - r.t_arrive, "cached_tokens": 0})
        if r.callback is not None:
            r.callback(res)
        if r.future is not None and r.loop is not None:
            r.loop.call_soon_threadsafe(lambda f=r.future, x=res: f.done() or f.set_result(x))

    # ------------------------------------------------------------------ introspection
    @property
    def io_bytes(self) -> Dict[str, int]:
        """Host<->device bytes moved by this engine's steps so far."""
        g = self._graphs.io_bytes if self._graphs is not None else {"h2d": 0, "d2h": 0}
        return {k: self._eager_io[k] + g[k] for k in ("h2d", "d2h")}

    def load(self) -> Dict[str, float]:
        return {"running": len(self.running), "waiting": len(self.waiting), "kv_usage": self.kv.usage()}
