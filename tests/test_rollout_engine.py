"""Rollout engine: paged-KV generation equals naive full recompute (CPU reference ops)."""

import asyncio
import os

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


def test_kv_prefix_migration_between_engines(tiny):
    """A multi-turn request moved to another instance takes its KV prefix along:
    the target's next turn reuses the migrated blocks (no prefill of the old
    context) and produces the same tokens as on the source."""
    src = LLMEngine(tiny.cfg, tiny.params, kv_blocks=128, block_size=4)
    dst = LLMEngine(tiny.cfg, tiny.params, kv_blocks=128, block_size=4)
    params = SamplingParams(max_tokens=4, temperature=0.0)
    prompt = list(range(40, 61))
    first = src.generate_sync([prompt], params)[0]
    ctx = prompt + first.output_tokens
    moved = src.migrate_prefix_to(dst, ctx)
    assert moved == (len(ctx) // 4) * 4 and moved >= 20
    # the copied blocks hold the source's K/V bit for bit
    blocks_src = src.kv.cached_blocks(ctx)
    blocks_dst = dst.kv.cached_blocks(ctx)
    assert [h for _, h in blocks_src] == [h for _, h in blocks_dst]
    for (bs_, _), (bd, _) in zip(blocks_src, blocks_dst):
        assert torch.equal(src.kv.k[:, bs_], dst.kv.k[:, bd]) and torch.equal(src.kv.v[:, bs_], dst.kv.v[:, bd])
    turn2 = ctx + [3, 4, 5]
    before = dst.stats["cached_prefix_tokens"]
    out_dst = dst.generate_sync([turn2], params)[0]
    assert dst.stats["cached_prefix_tokens"] - before >= 20
    assert out_dst.output_tokens == src.generate_sync([turn2], params)[0].output_tokens
    # a second migration of the same prefix finds it present and copies nothing new
    assert src.migrate_prefix_to(dst, ctx) == moved
    # engines on different weight versions do not exchange KV
    dst.update_weights({}, version=5)
    assert src.migrate_prefix_to(dst, ctx) == 0


def test_hetero_pool_migrates_kv_with_the_request(tiny):
    """C-MLFQ migration of a multi-turn request between two in-process
    instances carries the request's cached context to the target."""
    from types import SimpleNamespace

    from libra_b200.engine.heterogeneous_engine import HeterogeneousRolloutEngine
    from libra_b200.engine.rollout_engine import LocalRolloutEngine
    from libra_b200.engine.tokenizer import ByteTokenizer

    engines = [LocalRolloutEngine(LLMEngine(tiny.cfg, tiny.params, kv_blocks=128, block_size=4),
                                  ByteTokenizer(tiny.cfg.vocab_size)) for _ in range(2)]
    cfgs = [{"instance_id": f"i{i}", "tp_degree": 1} for i in range(2)]

    class _Sched:  # two-bucket stand-in with the C-MLFQ request-route interface
        def __init__(self):
            self.where = {}

        def register_instance(self, *a):
            pass

        def get_request_route(self, rid):
            i = self.where.get(rid)
            return None if i is None else SimpleNamespace(instance_index=i, pending=False, category="short",
                                                          is_fallback=False, reason="", request_id=rid)

        def execute_migration(self, rid, decision):
            self.where[rid] = 1
            return self.get_request_route(rid)

        def finish_request(self, rid, n):
            self.where.pop(rid, None)

    sched = _Sched()
    sched.where["r1"] = 0
    pool = HeterogeneousRolloutEngine(engines, cfgs, sched)
    prompt = list(range(40, 61))
    res = asyncio.run(pool.generate(prompt, max_new_tokens=4, temperature=0.0, request_id="r1"))
    assert res["_schedule_info"]["instance_index"] == 0
    pool.execute_cmlfq_migration("r1", SimpleNamespace(should_migrate=True, target_bucket="long"))
    assert pool.kv_migrations["count"] == 1 and pool.kv_migrations["tokens"] >= 20
    ctx = prompt + res["token_ids"]
    assert engines[1].engine.kv.cached_blocks(ctx)
    for e in engines:
        e.engine.shutdown()


def test_runner_mixed_step_matches_full_forward(tiny):
    """One runner step over a decode row, an extend with a cached prefix and a
    fresh prefill, in that order (the extend queries are not the leading rows
    and their keys come from the paged cache): the last-position logits equal
    a full recompute of each sequence."""
    from libra_b200.engine.rollout.runner import InferenceRunner, WorkItem, build_extend_plan

    cfg = tiny.cfg
    kv = PagedKVCache(cfg.num_hidden_layers, 64, 4, cfg.num_key_value_heads, cfg.head_dim, "cpu")
    run = InferenceRunner(cfg, tiny.params, kv)
    a, b = list(range(3, 14)), list(range(50, 59))
    run.step([WorkItem("a", a, 0), WorkItem("b", b, 0)])  # fill the cache for both
    a2, b2, c = a + [21], b + [7, 8, 9, 10], list(range(80, 87))
    items = [WorkItem("a", a2, len(a)), WorkItem("b", b2, len(b)), WorkItem("c", c, 0)]
    got = run.step(items).float()
    plan = build_extend_plan(items, [0, 1, 5], kv, "cpu")
    assert plan.items == [1, 2] and plan.q_rows is not None and plan.key_slots is not None
    assert plan.cu_q == [0, 4, 11] and plan.cu_k == [0, len(b2), len(b2) + len(c)]
    for row, seq in enumerate((a2, b2, c)):
        want = tiny.model.logits(pack_sequences([torch.tensor(seq)]))[-1].float()
        torch.testing.assert_close(got[row], want, rtol=2e-2, atol=2e-2)


def test_extend_plan_fresh_prefill_reads_no_cache():
    """Fresh prefills only: queries are the leading rows and the keys are the
    step's own K/V (no slot gather)."""
    from libra_b200.engine.rollout.runner import WorkItem, build_extend_plan

    kv = PagedKVCache(1, 16, 4, 1, 8, "cpu")
    items = [WorkItem("x", [1, 2, 3], 0), WorkItem("y", [4, 5, 6, 7, 8], 0)]
    for it in items:
        kv.reserve(it.seq_id, len(it.tokens))
    plan = build_extend_plan(items, [0, 3], kv, "cpu")
    assert plan.q_rows is None and plan.key_slots is None and plan.n_q == 8
    k = torch.arange(8.0).view(8, 1, 1)
    assert torch.equal(plan.keys(kv, 0, k, k)[0], k)
    assert build_extend_plan([WorkItem("x", [1, 2], 1)], [0], kv, "cpu") is None


def test_filtered_keep_mask_rule():
    """top-k keeps the k largest; top-p keeps a token while the mass strictly
    above it is at most p; ties with a threshold are kept; the CPU sampler
    draws inside the kept set."""
    from libra_b200 import ops

    x = torch.tensor([3.0, 2.0, 1.0, 0.0])
    p = torch.softmax(x, -1)  # ~[0.64, 0.24, 0.09, 0.03]
    assert ops.filtered_keep_mask(x, 1.0, 2).tolist() == [True, True, False, False]
    assert ops.filtered_keep_mask(x, 0.5, -1).tolist() == [True, False, False, False]
    assert ops.filtered_keep_mask(x, float(p[0]) + 1e-4, -1).tolist() == [True, True, False, False]
    assert ops.filtered_keep_mask(x, 0.7, 3).tolist() == [True, True, False, False]
    tied = torch.tensor([1.0, 2.0, 2.0, 0.5])
    assert ops.filtered_keep_mask(tied, 1.0, 1).tolist() == [False, True, True, False]
    assert ops.filtered_keep_mask(tied, 0.1, -1).tolist() == [False, True, True, False]
    g = torch.Generator().manual_seed(0)
    logits = torch.randn(3, 50, generator=g)
    tok, lp = torch.empty(3, dtype=torch.long), torch.empty(3)
    ops.sample_tokens_filtered(logits, torch.tensor([1.0, 0.0, 2.0]), torch.tensor([0.6, 0.6, 1.0]),
                               torch.tensor([-1, 3, 4]), torch.tensor([1, 2, 3]), torch.tensor([5, 6, 7]), tok, lp)
    assert int(tok[1]) == int(logits[1].argmax())
    for b, (t, pp, k) in enumerate(((1.0, 0.6, -1), (1.0, 0.6, 3), (2.0, 1.0, 4))):
        x = logits[b] / t
        if b != 1:
            assert bool(ops.filtered_keep_mask(x, pp, k)[int(tok[b])])
        assert abs(float(lp[b]) - float(torch.log_softmax(x, -1)[int(tok[b])])) < 1e-5


@pytest.mark.parametrize("tp", [1, 2, 4])
def test_kv_block_export_import_with_head_slices(tp):
    """Exported blocks land in TP caches as each rank's KV heads (tp=4 shares
    each of 2 heads between two ranks) and register the prefix hash chain."""
    torch.manual_seed(0)
    src = PagedKVCache(2, 16, 4, 2, 8, "cpu", dtype=torch.float32)
    toks = list(range(30, 41))  # 2 full blocks + 3 tokens
    src.reserve("s", len(toks))
    slots = src.slot_mapping("s", 0, len(toks))
    for layer in range(2):
        src.write(layer, slots, torch.randn(len(toks), 2, 8), torch.randn(len(toks), 2, 8))
    src.commit("s", toks)
    blocks = src.cached_blocks(toks)
    assert len(blocks) == 2 and [h for _, h in blocks] == src.block_hashes(toks)
    k, v = src.export_blocks(blocks)
    assert k.shape == (2, 2, 4, 2, 8)
    kv_l = max(1, 2 // tp)
    for r in range(tp):
        kv0 = r * 2 // tp
        dst = PagedKVCache(2, 16, 4, kv_l, 8, "cpu", dtype=torch.float32)
        assert dst.import_block_tensors(toks, k[:, :, :, kv0:kv0 + kv_l], v[:, :, :, kv0:kv0 + kv_l]) == 8
        assert dst.match_prefix("t", toks + [99]) == 8
        got = dst.gather(0, "t", 8)[0]
        want = src.gather(0, "s", 8)[0][:, kv0:kv0 + kv_l]
        assert torch.equal(got, want)


def test_hetero_pool_migrates_kv_into_a_server_instance(tiny):
    """Migration target without an in-process engine (a server client): the
    pool exports the context's KV to a file, the target imports it, and the
    file is removed afterwards."""
    from types import SimpleNamespace

    from libra_b200.engine import heterogeneous_engine as he
    from libra_b200.engine.rollout_engine import LocalRolloutEngine
    from libra_b200.engine.tokenizer import ByteTokenizer

    class _Server:  # the HTTP client's import interface, served by an engine of another "process"
        instance_id = "server"

        def __init__(self):
            self.llm = LLMEngine(tiny.cfg, tiny.params, kv_blocks=128, block_size=4)
            self.paths = []

        def import_prefix(self, payload):
            self.paths.append(payload["path"])
            return self.llm.import_prefix(payload)

    class _Sched:
        where = {"r1": 0}

        def register_instance(self, *a):
            pass

        def get_request_route(self, rid):
            i = self.where.get(rid)
            return None if i is None else SimpleNamespace(instance_index=i, pending=False, category="short",
                                                          is_fallback=False, reason="", request_id=rid)

        def execute_migration(self, rid, decision):
            self.where[rid] = 1
            return self.get_request_route(rid)

    local = LocalRolloutEngine(LLMEngine(tiny.cfg, tiny.params, kv_blocks=128, block_size=4),
                               ByteTokenizer(tiny.cfg.vocab_size))
    server = _Server()
    pool = he.HeterogeneousRolloutEngine([local, server], [{"instance_id": "i0", "tp_degree": 1},
                                                           {"instance_id": "server", "tp_degree": 2}], _Sched())
    prompt = list(range(40, 61))
    res = asyncio.run(pool.generate(prompt, max_new_tokens=4, temperature=0.0, request_id="r1"))
    pool.execute_cmlfq_migration("r1", SimpleNamespace(should_migrate=True))
    ctx = prompt + res["token_ids"]
    assert pool.kv_migrations["count"] == 1 and pool.kv_migrations["tokens"] == (len(ctx) // 4) * 4
    assert server.llm.kv.cached_blocks(ctx) and server.llm.stats["migrated_in_tokens"] > 0
    assert server.paths and not os.path.exists(server.paths[0])
    local.engine.shutdown()
