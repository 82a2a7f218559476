"""Megatron-Core model-space checkpoints across parallel layouts, as gloo
processes on CPU (reference tests/test_megatron_core_checkpointing.py).

* TP=2 x DP=2 with the sharded optimizer saves, loads back exactly, and loads
  into a TP=1 engine whose state, re-sharded, equals the writer's;
* EP=2 saves and loads into an EP=1 engine;
* a fixture written the way Megatron-Core lays the tensors out (one global
  tensor per key, layers stacked, QKV per query group, fc1 [gate; up]) loads
  into a TP=2 engine."""

import os

import pytest
import torch
import torch.distributed as dist

from tests.test_parallel_gloo import _init, _spawn


def _trajs(vocab, seed=0):
    from libra_b200.workflow.synthetic import GRPOWorkload, LengthDist

    wl = GRPOWorkload("ck", vocab_size=vocab, prompts_per_step=2, group_size=2, prompt=LengthDist(12, 0.3, 6, 20),
                      response=LengthDist(8, 0.3, 2, 12))
    return wl.trajectories(seed)


def _full_local_state(eng):
    """Per-parameter fp32 master / moments of this rank's (TP-local) parameters,
    gathered over the data-parallel group when the optimizer is sharded."""
    out = {}
    for attr in ("master", "exp_avg", "exp_avg_sq"):
        flat = eng.optimizer_state_tensors()[attr].float()
        if eng.sharded:
            parts = [torch.empty_like(flat) for _ in range(eng.dp_size)]
            dist.all_gather(parts, flat, group=eng.dp_group)
            flat = torch.cat(parts)
        out[attr] = {n: flat[eng.layout.offsets[n]:eng.layout.offsets[n] + p.numel()].view(p.shape)
                     for n, p in eng.params.items() if eng.layout.offsets[n] < eng.dense_numel}
    return out


def _tp_dp_worker(rank, world, port, ck):
    _init(rank, world, port)
    from libra_b200.engine.checkpointing import DistributedCheckpointManager
    from libra_b200.engine.train_engine import B200TrainEngine
    from libra_b200.parallel.tensor_parallel import shard_full_params

    kw = dict(device="cpu", learning_rate=1e-3, micro_batch_size=2)
    a = B200TrainEngine("tiny", tp_size=2, seed=3, **kw)
    a.initialize()
    assert a.sharded and a.dp_size == 2
    trajs = _trajs(a.cfg.vocab_size)
    a.recompute_logprobs(trajs)
    a.grpo_update(trajs)
    mgr = DistributedCheckpointManager(ck)
    mgr.save(a, 1, export_for_rollout=False)
    if rank == 0:
        import torch.distributed.checkpoint as dcp

        md = dcp.FileSystemReader(os.path.join(ck, "v1", "megatron_dist")).read_metadata().state_dict_metadata
        cfg = a.cfg
        D, L, H = cfg.head_dim, cfg.num_hidden_layers, cfg.hidden_size
        qkv = (cfg.num_attention_heads + 2 * cfg.num_key_value_heads) * D
        assert tuple(md["decoder.layers.self_attention.linear_qkv.weight"].size) == (L, qkv, H)
        assert tuple(md["optimizer.state.exp_avg_sq.decoder.layers.mlp.linear_fc1.weight"].size) == \
            (L, 2 * cfg.intermediate_size, H)
        assert tuple(md["embedding.word_embeddings.weight"].size) == (cfg.vocab_size, H)
        assert os.path.exists(os.path.join(ck, "v1", "megatron_dist", "common.pt"))
    # same layout: exact round trip of weights and optimizer state
    b = B200TrainEngine("tiny", tp_size=2, seed=11, **kw)
    b.initialize()
    mgr.load(b, 1)
    assert torch.equal(a.flat_param, b.flat_param) and b.step_count == a.step_count
    for attr in ("master", "exp_avg", "exp_avg_sq"):
        assert torch.equal(getattr(a, attr), getattr(b, attr)), attr
    # TP=1, one unsharded replica per rank: the same model and optimizer state in full
    solo = [dist.new_group([r]) for r in range(world)][rank]
    c = B200TrainEngine("tiny", dp_group=solo, seed=5, **kw)
    c.initialize()
    mgr.load(c, 1)
    want = _full_local_state(a)
    full = {attr: {n: t for n, t in d.items()} for attr, d in _full_local_state(c).items()}
    for n, p in shard_full_params({n: p.detach() for n, p in c.params.items()}, c.cfg, 2, a.tp_rank).items():
        assert torch.equal(p, a.params[n].detach()), n
    for attr in ("master", "exp_avg", "exp_avg_sq"):
        for n, t in shard_full_params(full[attr], c.cfg, 2, a.tp_rank).items():
            assert torch.equal(t, want[attr][n]), (attr, n)
    open(os.path.join(os.path.dirname(ck), f"ok_{rank}"), "w").close()
    dist.destroy_process_group()


def test_tp2_dp2_checkpoint_loads_at_tp2_and_tp1(tmp_path):
    _spawn(_tp_dp_worker, 4, str(tmp_path / "ck"))
    assert {p.name for p in tmp_path.iterdir() if p.name.startswith("ok_")} == {f"ok_{r}" for r in range(4)}


def _ep_worker(rank, world, port, ck):
    _init(rank, world, port)
    from libra_b200.engine.checkpointing import DistributedCheckpointManager
    from libra_b200.engine.train_engine import B200TrainEngine

    kw = dict(device="cpu", learning_rate=1e-3, micro_batch_size=4)
    a = B200TrainEngine("tiny-moe", ep_size=2, seed=3, **kw)
    a.initialize()
    a.grpo_update(_trajs(2048, seed=rank))
    mgr = DistributedCheckpointManager(ck)
    mgr.save(a, 2, export_for_rollout=False)
    solo = [dist.new_group([r]) for r in range(world)][rank]
    c = B200TrainEngine("tiny-moe", dp_group=solo, seed=9, **kw)
    c.initialize()
    mgr.load(c, 2)
    El = c.cfg.num_experts // 2
    for n, p in a.params.items():
        want = c.params[n][rank * El:(rank + 1) * El] if "experts." in n else c.params[n]
        assert torch.equal(p.detach(), want.detach()), n
        off = a.layout.offsets[n]
        if off >= a.dense_numel:  # expert optimizer state of this rank's experts
            x0 = off - a.dense_numel
            got = c.master[c.layout.offsets[n]:c.layout.offsets[n] + c.params[n].numel()].view(c.params[n].shape)
            assert torch.equal(a.x_master[x0:x0 + p.numel()].view(p.shape), got[rank * El:(rank + 1) * El]), n
    open(os.path.join(os.path.dirname(ck), f"ok_{rank}"), "w").close()
    dist.destroy_process_group()


def test_ep2_checkpoint_loads_at_ep1(tmp_path):
    _spawn(_ep_worker, 2, str(tmp_path / "ck"))
    assert {p.name for p in tmp_path.iterdir() if p.name.startswith("ok_")} == {"ok_0", "ok_1"}


def _write_mcore_fixture(path, cfg, full):
    """One global tensor per key, written the way Megatron-Core lays out a GPT
    model: decoder layers stacked on axis 0, QKV rows per query group, fc1 as
    [gate; up]; plus common.pt / metadata.json."""
    import json

    import torch.distributed.checkpoint as dcp

    D, L = cfg.head_dim, cfg.num_hidden_layers
    nq, nkv = cfg.num_attention_heads, cfg.num_key_value_heads
    per = nq // nkv

    def grouped(w):
        q, k, v = w[:nq * D], w[nq * D:(nq + nkv) * D], w[(nq + nkv) * D:]
        rows = []
        for g in range(nkv):
            rows += [q[g * per * D:(g + 1) * per * D], k[g * D:(g + 1) * D], v[g * D:(g + 1) * D]]
        return torch.cat(rows)

    def stack(name, fn=lambda t: t):
        return torch.stack([fn(full[f"layers.{i}.{name}"]) for i in range(L)])

    sd = {"embedding.word_embeddings.weight": full["embed_tokens"],
          "decoder.final_layernorm.weight": full["norm"],
          "decoder.layers.input_layernorm.weight": stack("input_layernorm"),
          "decoder.layers.self_attention.linear_qkv.weight": stack("qkv_proj", grouped),
          "decoder.layers.self_attention.q_layernorm.weight": stack("q_norm"),
          "decoder.layers.self_attention.k_layernorm.weight": stack("k_norm"),
          "decoder.layers.self_attention.linear_proj.weight": stack("o_proj"),
          "decoder.layers.pre_mlp_layernorm.weight": stack("post_attention_layernorm"),
          "decoder.layers.mlp.linear_fc1.weight": stack("gate_up_proj"),
          "decoder.layers.mlp.linear_fc2.weight": stack("down_proj")}
    if not cfg.tie_word_embeddings:
        sd["output_layer.weight"] = full["lm_head"]
    dcp.save({k: v.contiguous() for k, v in sd.items()}, checkpoint_id=path)
    if dist.get_rank() == 0:
        torch.save({"checkpoint_version": 3.0, "iteration": 4}, os.path.join(path, "common.pt"))
        with open(os.path.join(path, "metadata.json"), "w") as f:
            json.dump({"sharded_backend": "torch_dist", "sharded_backend_version": 1, "common_backend": "torch",
                       "common_backend_version": 1}, f)


def _fixture_worker(rank, world, port, root):
    _init(rank, world, port)
    import json

    from libra_b200.engine.checkpointing import DistributedCheckpointManager
    from libra_b200.engine.train_engine import B200TrainEngine
    from libra_b200.models.qwen3 import ParamLayout, get_config, init_params, param_shapes
    from libra_b200.parallel.tensor_parallel import shard_full_params

    cfg = get_config("tiny")
    lay = ParamLayout(param_shapes(cfg))
    full = lay.views(torch.empty(lay.numel, dtype=torch.bfloat16))
    init_params(cfg, full, seed=21)
    vdir = os.path.join(root, "v4")
    _write_mcore_fixture(os.path.join(vdir, "megatron_dist"), cfg, full)
    if rank == 0:
        with open(os.path.join(vdir, "megatron_checkpoint_manifest.json"), "w") as f:
            json.dump({"version": 4}, f)
    dist.barrier()
    eng = B200TrainEngine("tiny", device="cpu", tp_size=2, seed=1)
    eng.initialize()
    DistributedCheckpointManager(root).load(eng, 4, load_optimizer=False)
    for n, t in shard_full_params(dict(full), cfg, 2, eng.tp_rank).items():
        assert torch.equal(eng.params[n].detach(), t), n
    open(os.path.join(root, f"ok_{rank}"), "w").close()
    dist.destroy_process_group()


def test_mcore_layout_fixture_loads_into_tp2(tmp_path):
    _spawn(_fixture_worker, 2, str(tmp_path))
    assert {p.name for p in tmp_path.iterdir() if p.name.startswith("ok_")} == {"ok_0", "ok_1"}


@pytest.mark.parametrize("tp", [1, 2, 4])
def test_param_chunks_tile_the_global_tensors(tp):
    """Across the TP ranks the chunks of every parameter cover its global tensor
    exactly once (tp=4 shares each of tiny's 2 KV heads between two ranks: those
    chunks coincide and count once)."""
    from libra_b200.engine.mcore_layout import ShardInfo, param_chunks
    from libra_b200.models.qwen3 import get_config, param_shapes

    cfg = get_config("tiny")
    cover = {}
    for r in range(tp):
        for name, shape in param_shapes(cfg, tp, r):
            for c in param_chunks(name, shape, cfg, ShardInfo(tp_size=tp, tp_rank=r)):
                sizes = [1] * c.prepend + list(shape)
                for dim, _, length in c.narrows:
                    sizes[c.prepend + dim] = length
                cover.setdefault(c.key, (c.gshape, set()))[1].add((c.offsets, tuple(sizes)))
    for key, (gshape, chunks) in cover.items():
        mark = torch.zeros(gshape, dtype=torch.int32)
        for off, sizes in chunks:
            mark[tuple(slice(o, o + s) for o, s in zip(off, sizes))] += 1
        assert torch.equal(mark, torch.ones_like(mark)), key
