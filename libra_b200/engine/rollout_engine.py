"""Rollout clients: the object a workflow calls ``generate`` on.

Same call/return contract as the reference (``engine/rollout_engine.py``):
``await generate(prompt, max_new_tokens, temperature, top_p, n, input_tokens,
seed)`` -> ``{"text", "tokens", "logprobs", "finish_reason"}``; here the dict
also carries ``token_ids`` and ``prompt_token_ids`` so trainers never have to
re-tokenise.  ``prompt`` may be a string (tokenised with the client's
tokenizer) or a list of token ids.

* ``LocalRolloutEngine`` - in-process fast path onto an ``LLMEngine`` (no HTTP,
  no serialisation; used when rollout instances live in the trainer's process
  tree on the same box).
* ``HTTPRolloutEngine`` - OpenAI ``/v1/completions`` client (this framework's
  server or any OpenAI-compatible one); ``wait_for_ready`` polls ``/health``.
* ``MultiInstanceRolloutEngine`` - round robin over clients.
* ``MockRolloutEngine`` - fixed answer, for smoke tests without a model.
"""

from __future__ import annotations

import asyncio
import logging
import time
from typing import Any, Dict, List, Optional, Sequence, Union

from libra_b200.engine.rollout.sampler import SamplingParams

log = logging.getLogger(__name__)
Prompt = Union[str, Sequence[int]]


def _ids(tokenizer, prompt: Prompt) -> List[int]:
    if isinstance(prompt, str):
        return list(tokenizer.encode(prompt, add_special_tokens=False))
    return [int(t) for t in prompt]


class LocalRolloutEngine:
    def __init__(self, engine, tokenizer, instance_id: str = ""):
        self.engine = engine
        self.tokenizer = tokenizer
        self.instance_id = instance_id or engine.instance_id

    async def generate(self, prompt: Prompt, max_new_tokens: int = 1024, temperature: float = 1.0,
                       top_p: float = 1.0, n: int = 1, input_tokens: int = 0, seed: Optional[int] = None,
                       top_k: int = -1, stop_token_ids: Optional[List[int]] = None, **_) -> Dict[str, Any]:
        ids = _ids(self.tokenizer, prompt)
        stops = list(stop_token_ids or [])
        eos = getattr(self.tokenizer, "eos_token_id", None)
        if eos is not None and eos not in stops:
            stops.append(int(eos))
        res = await self.engine.generate(ids, SamplingParams(max_tokens=max_new_tokens, temperature=temperature,
                                                             top_p=top_p, top_k=top_k, stop_token_ids=stops,
                                                             seed=seed))
        return {"text": self.tokenizer.decode(res.output_tokens), "tokens": [str(t) for t in res.output_tokens],
                "token_ids": list(res.output_tokens), "prompt_token_ids": ids, "logprobs": list(res.output_logprobs),
                "finish_reason": res.finish_reason, "metrics": res.metrics, "policy_version": self.engine.version}

    async def generate_batch(self, prompts: List[Prompt], **kw) -> List[Dict[str, Any]]:
        out = await asyncio.gather(*(self.generate(p, **kw) for p in prompts), return_exceptions=True)
        return [r for r in out if not isinstance(r, Exception)]

    def wait_for_ready(self, timeout: float = 0.0) -> bool:
        return True

    def close(self) -> None:
        pass


class HTTPRolloutEngine:
    """OpenAI-compatible completions client (aiohttp)."""

    def __init__(self, host: str = "127.0.0.1", port: int = 8000, model_path: str = "", timeout: float = 3600.0,
                 instance_id: str = ""):
        self.base_url = f"http://{host}:{port}"
        self.completions_url = f"{self.base_url}/v1/completions"
        self.model_path = model_path
        self.timeout = timeout
        self.instance_id = instance_id or f"{host}:{port}"
        self._session = None
        self._session_loop = None

    async def _client(self):
        import aiohttp

        loop = asyncio.get_running_loop()
        if self._session is None or self._session.closed or self._session_loop is not loop:
            self._session = aiohttp.ClientSession(timeout=aiohttp.ClientTimeout(total=self.timeout))
            self._session_loop = loop
        return self._session

    async def generate(self, prompt: Prompt, max_new_tokens: int = 1024, temperature: float = 1.0,
                       top_p: float = 1.0, n: int = 1, input_tokens: int = 0, seed: Optional[int] = None,
                       **kw) -> Dict[str, Any]:
        payload = {"model": self.model_path, "prompt": prompt if isinstance(prompt, str) else list(prompt),
                   "max_tokens": max_new_tokens, "temperature": temperature, "top_p": top_p, "n": n, "logprobs": 1}
        if seed is not None:
            payload["seed"] = int(seed)
        for k in ("top_k", "stop_token_ids"):
            if kw.get(k) is not None:
                payload[k] = kw[k]
        session = await self._client()
        async with session.post(self.completions_url, json=payload) as resp:
            if resp.status != 200:
                raise RuntimeError(f"Generation failed: status={resp.status}, {await resp.text()}")
            return self._parse_response(await resp.json())

    @staticmethod
    def _parse_response(response: dict) -> Dict[str, Any]:
        if not isinstance(response, dict):
            raise ValueError(f"Invalid response type: {type(response).__name__}")
        choices = response.get("choices") or []
        if not choices:
            raise ValueError("Empty response")
        c = choices[0]
        lp = c.get("logprobs") or {}
        if not isinstance(lp, dict):
            lp = {}
        return {"text": c.get("text", "") or "", "tokens": lp.get("tokens") or [],
                "token_ids": c.get("token_ids") or [], "prompt_token_ids": c.get("prompt_token_ids") or [],
                "logprobs": lp.get("token_logprobs") or [], "finish_reason": c.get("finish_reason", "length")}

    def import_prefix(self, request: Dict[str, Any], timeout: float = 120.0) -> int:
        """Hand the server KV exported by ``LLMEngine.export_prefix`` (blocking;
        C-MLFQ migration runs on the scheduler's thread).  Returns the prefix
        tokens now cached there."""
        import json
        import urllib.request

        req = urllib.request.Request(f"{self.base_url}/import_kv", data=json.dumps(request).encode(), method="POST",
                                     headers={"Content-Type": "application/json"})
        with urllib.request.urlopen(req, timeout=timeout) as r:
            return int(json.loads(r.read() or b"{}").get("tokens", 0))

    def wait_for_ready(self, timeout: float = 300.0, interval: float = 1.0) -> bool:
        import urllib.request

        deadline = time.monotonic() + timeout
        while time.monotonic() < deadline:
            try:
                with urllib.request.urlopen(f"{self.base_url}/health", timeout=5) as r:
                    if r.status == 200:
                        return True
            except OSError:
                pass
            time.sleep(interval)
        return False

    async def aclose(self) -> None:
        if self._session is not None and not self._session.closed:
            await self._session.close()

    def close(self) -> None:
        s = self._session
        self._session = None
        if s is not None and not s.closed:
            try:
                asyncio.run(s.close())
            except RuntimeError:
                pass


class MultiInstanceRolloutEngine:
    def __init__(self, engines: List[Any]):
        if not engines:
            raise ValueError("MultiInstanceRolloutEngine needs at least one engine")
        self.engines = engines
        self._next = 0

    async def generate(self, prompt: Prompt, **kw) -> Dict[str, Any]:
        eng = self.engines[self._next % len(self.engines)]
        self._next += 1
        return await eng.generate(prompt, **kw)

    def wait_for_ready(self, timeout: float = 300.0) -> bool:
        return all(e.wait_for_ready(timeout) for e in self.engines)


class MockRolloutEngine:
    """Returns a fixed completion (reference ``engine/rollout_engine.py:17-57``)."""

    def __init__(self, response_text: str = "The answer is 42.", tokenizer=None):
        from libra_b200.engine.tokenizer import ByteTokenizer

        self.response_text = response_text
        self.tokenizer = tokenizer or ByteTokenizer()
        self.calls = 0

    async def generate(self, prompt: Prompt, max_new_tokens: int = 1024, **_) -> Dict[str, Any]:
        self.calls += 1
        ids = self.tokenizer.encode(self.response_text)[:max_new_tokens]
        return {"text": self.tokenizer.decode(ids), "tokens": [str(i) for i in ids], "token_ids": ids,
                "prompt_token_ids": _ids(self.tokenizer, prompt), "logprobs": [-0.1] * len(ids),
                "finish_reason": "stop"}

    def wait_for_ready(self, timeout: float = 0.0) -> bool:
        return True


# Reference class name for the HTTP client
VLLMRolloutEngine = HTTPRolloutEngine
