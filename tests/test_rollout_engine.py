"""Rollout engine: paged-KV generation equals naive full recompute (CPU reference ops)."""

import asyncio

import pytest
import torch

from libra_b200.engine.rollout.kv_cache import BlockAllocator, PagedKVCache
from libra_b200.engine.rollout.llm_engine import LLMEngine
from libra_b200.engine.rollout.sampler import SamplingParams, sample
from libra_b200.engine.train_engine import B200TrainEngine
from libra_b200.models.qwen3 import pack_sequences


@pytest.fixture(scope="module")
def tiny():
    eng = B200TrainEngine("tiny", device="cpu", seed=7)
    eng.initialize()
    return eng


def _naive_greedy(model, prompt, n):
    toks = list(prompt)
    for _ in range(n):
        b = pack_sequences([torch.tensor(toks)])
        logits = model.logits(b)
        toks.append(int(logits[-1].float().argmax()))
    return toks[len(prompt):]


def test_greedy_matches_naive(tiny):
    eng = LLMEngine(tiny.cfg, tiny.params, kv_blocks=128, block_size=4, max_batch_tokens=64)
    prompts = [[5, 9, 33, 100, 7], [44, 2, 19], list(range(10, 31))]
    params = SamplingParams(max_tokens=6, temperature=0.0)
    got = eng.generate_sync(prompts, params)
    for p, r in zip(prompts, got):
        assert r.output_tokens == _naive_greedy(tiny.model, p, 6)
        assert r.finish_reason == "length" and len(r.output_logprobs) == 6
        assert all(lp <= 0.0 for lp in r.output_logprobs)


def test_prefix_cache_reuse_and_multiturn(tiny):
    eng = LLMEngine(tiny.cfg, tiny.params, kv_blocks=128, block_size=4)
    params = SamplingParams(max_tokens=4, temperature=0.0)
    first = eng.generate_sync([list(range(40, 61))], params)[0]
    turn2 = list(range(40, 61)) + first.output_tokens + [3, 4, 5]
    cached_before = eng.stats["cached_prefix_tokens"]
    second = eng.generate_sync([turn2], params)[0]
    assert eng.stats["cached_prefix_tokens"] - cached_before >= 20
    assert second.output_tokens == _naive_greedy(tiny.model, turn2, 4)
    eng.update_weights({}, version=3)
    assert eng.version == 3 and not eng.kv.alloc.cached


def test_async_generate_and_seeded_sampling(tiny):
    eng = LLMEngine(tiny.cfg, tiny.params, kv_blocks=256, block_size=8)

    async def run():
        p = SamplingParams(max_tokens=5, temperature=1.0, seed=11)
        a, b = await asyncio.gather(eng.generate([1, 2, 3], p), eng.generate([1, 2, 3], p))
        return a, b

    a, b = asyncio.run(run())
    eng.shutdown()
    assert a.output_tokens == b.output_tokens and len(a.output_tokens) == 5


def test_block_allocator_lru_eviction():
    al = BlockAllocator(2, 4)
    b0 = al.allocate()
    al.register(b0, "h0")
    al.release(b0)
    assert al.lookup("h0") == b0
    al.release(b0)
    b1 = al.allocate()
    b2 = al.allocate()  # evicts the cached block
    assert {b1, b2} == {0, 1} and al.lookup("h0") is None
    with pytest.raises(MemoryError):
        al.allocate()


def test_sampler_top_k_and_greedy():
    logits = torch.tensor([[0.0, 5.0, 1.0, 2.0], [3.0, 0.0, 0.0, 0.0]])
    t, lp = sample(logits, torch.tensor([0.0, 1.0]), torch.tensor([1.0, 1.0]), torch.tensor([-1, 1]))
    assert t.tolist() == [1, 0]
    assert torch.allclose(lp[1], torch.log_softmax(logits[1], -1)[0])
