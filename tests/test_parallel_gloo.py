"""TP / PP / EP equivalence against one rank, as 2 gloo processes on CPU."""

import os
import socket
import sys

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from libra_b200.parallel.mesh import ParallelMesh


def _free_port() -> int:
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _spawn(fn, world, *args):
    port = _free_port()
    mp.start_processes(fn, args=(world, port, *args), nprocs=world, join=True, start_method="spawn")


def _init(rank, world, port):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    import datetime

    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60))


def _model_inputs(cfg_name="tiny"):
    from libra_b200.models.qwen3 import ParamLayout, get_config, init_params, pack_sequences, param_shapes

    cfg = get_config(cfg_name)
    shapes = param_shapes(cfg)
    flat = torch.zeros(ParamLayout(shapes).numel)
    views = ParamLayout(shapes).views(flat)
    init_params(cfg, views, seed=1)
    g = torch.Generator().manual_seed(0)
    seqs = [torch.randint(4, cfg.vocab_size, (n,), generator=g) for n in (9, 14, 5)]
    return cfg, {k: v.clone() for k, v in views.items()}, pack_sequences(seqs)


def _run_model(cfg, params, batch, tp_group=None, tp_size=1, tp_rank=0, sp=False):
    from libra_b200.models.qwen3 import Qwen3Model

    ps = {k: torch.nn.Parameter(v.clone()) for k, v in params.items()}
    m = Qwen3Model(cfg, ps, tp_group=tp_group, tp_size=tp_size, tp_rank=tp_rank, sequence_parallel=sp)
    lp = m.action_logprobs(batch)
    w = torch.linspace(0.5, 1.5, lp.numel())
    (lp * w).sum().backward()
    return lp.detach(), {k: p.grad for k, p in ps.items()}


def _tp_worker(rank, world, port, out_dir):
    _init(rank, world, port)
    from libra_b200.parallel.tensor_parallel import shard_full_params, tp_partial_grad_params

    cfg, full, batch = _model_inputs()
    ref_lp, ref_g = _run_model(cfg, full, batch)
    local = shard_full_params(full, cfg, world, rank)
    lp, grads = _run_model(cfg, local, batch, dist.group.WORLD, world, rank)
    for n in tp_partial_grad_params(list(grads)):
        dist.all_reduce(grads[n])
    torch.testing.assert_close(lp, ref_lp, rtol=1e-4, atol=1e-4)
    ref_local = shard_full_params(ref_g, cfg, world, rank)
    for n, gr in grads.items():
        torch.testing.assert_close(gr, ref_local[n], rtol=1e-3, atol=1e-4, msg=n)
    open(os.path.join(out_dir, f"tp_ok_{rank}"), "w").close()
    dist.destroy_process_group()


def _sp_worker(rank, world, port, out_dir):
    """Tensor + sequence parallelism: residual stream split over tokens, all-gather before the
    column-parallel linears, reduce-scatter after the row-parallel ones."""
    _init(rank, world, port)
    from libra_b200.models.qwen3 import pack_sequences
    from libra_b200.parallel.tensor_parallel import shard_full_params, tp_partial_grad_params

    cfg, full, _ = _model_inputs()
    g = torch.Generator().manual_seed(0)
    seqs = [torch.randint(4, cfg.vocab_size, (n,), generator=g) for n in (9, 14, 6)]  # 29 tokens: padded to 30
    batch = pack_sequences(seqs, pad_multiple=world)
    assert batch.num_tokens == 30 and int(batch.action_rows.max()) < 29
    ref_lp, ref_g = _run_model(cfg, full, pack_sequences(seqs))
    local = shard_full_params(full, cfg, world, rank)
    lp, grads = _run_model(cfg, local, batch, dist.group.WORLD, world, rank, sp=True)
    for n in tp_partial_grad_params(list(grads), sequence_parallel=True):
        dist.all_reduce(grads[n])
    torch.testing.assert_close(lp, ref_lp, rtol=1e-4, atol=1e-4)
    ref_local = shard_full_params(ref_g, cfg, world, rank)
    for n, gr in grads.items():
        torch.testing.assert_close(gr, ref_local[n], rtol=1e-3, atol=1e-4, msg=n)
    open(os.path.join(out_dir, f"sp_ok_{rank}"), "w").close()
    dist.destroy_process_group()


def _pp_worker(rank, world, port, out_dir):
    _init(rank, world, port)
    from libra_b200.models.qwen3 import Qwen3Model
    from libra_b200.parallel.pipeline import P2P, PipelineStage, allreduce_tied_embedding_grad, one_f_one_b

    cfg, full, batch = _model_inputs()
    mbs = [{"batch": batch}, {"batch": batch}, {"batch": batch}]

    def loss_fn(logp, mb):
        return -logp.mean()

    # single-stage reference
    ps_ref = {k: torch.nn.Parameter(v.clone()) for k, v in full.items()}
    ref = PipelineStage(Qwen3Model(cfg, ps_ref), 0, cfg.num_hidden_layers, True, True, loss_fn)
    ref_losses = [float(ref(mb, None).backward() or 0) for mb in mbs]
    ps = {k: torch.nn.Parameter(v.clone()) for k, v in full.items()}
    r = PipelineStage.split_layers(cfg.num_hidden_layers, world)[rank]
    stage = PipelineStage(Qwen3Model(cfg, ps), r.start, r.stop, rank == 0, rank == world - 1, loss_fn)
    p2p = P2P(None, rank - 1 if rank > 0 else None, rank + 1 if rank < world - 1 else None, dtype=torch.float32)
    losses = one_f_one_b(stage, mbs, p2p, world, rank)
    assert cfg.tie_word_embeddings
    allreduce_tied_embedding_grad(ps["embed_tokens"], dist.group.WORLD)
    for name, p in ps.items():
        if p.grad is not None:
            torch.testing.assert_close(p.grad, ps_ref[name].grad, rtol=1e-4, atol=1e-5, msg=name)
    if rank == world - 1:
        assert len(losses) == 3
    open(os.path.join(out_dir, f"pp_ok_{rank}"), "w").close()
    dist.destroy_process_group()


def _ep_worker(rank, world, port, out_dir):
    _init(rank, world, port)
    from libra_b200.models.moe import moe_mlp
    from libra_b200.models.qwen3 import get_config
    from libra_b200.parallel.expert_parallel import ep_moe_mlp

    cfg = get_config("tiny-moe")
    g = torch.Generator().manual_seed(7)
    E, H, F = cfg.num_experts, cfg.hidden_size, cfg.moe_intermediate_size
    h = torch.randn(40, H, generator=g) * 0.5
    res = torch.randn(40, H, generator=g)
    router = torch.randn(E, H, generator=g) * 0.05
    w1 = torch.randn(E, 2 * F, H, generator=g) * 0.05
    w2 = torch.randn(E, H, F, generator=g) * 0.05
    hh = h[rank * 20:(rank + 1) * 20]  # each rank owns different tokens
    ref = moe_mlp(hh, res[rank * 20:(rank + 1) * 20], router, w1, w2, cfg)
    El = E // world
    w1l = w1[rank * El:(rank + 1) * El].clone().requires_grad_(True)
    out = ep_moe_mlp(hh, res[rank * 20:(rank + 1) * 20], router, w1l, w2[rank * El:(rank + 1) * El], cfg,
                     dist.group.WORLD)
    torch.testing.assert_close(out, ref, rtol=1e-4, atol=1e-4)
    out.sum().backward()
    assert w1l.grad is not None and torch.isfinite(w1l.grad).all()
    open(os.path.join(out_dir, f"ep_ok_{rank}"), "w").close()
    dist.destroy_process_group()


@pytest.mark.parametrize("kind,fn", [("tp", _tp_worker), ("sp", _sp_worker), ("pp", _pp_worker),
                                     ("ep", _ep_worker)])
def test_parallel_equivalence(tmp_path, kind, fn):
    _spawn(fn, 2, str(tmp_path))
    assert {p.name for p in tmp_path.iterdir()} == {f"{kind}_ok_0", f"{kind}_ok_1"}


def test_mesh_layout():
    m = ParallelMesh(8, tp=2, pp=2, ep=2, create_groups=False)
    assert m.dp == 2
    assert m.members("tp", 5) == [4, 5]
    assert m.members("dp", 1) == [1, 3] and m.members("pp", 1) == [1, 5]
    assert m.members("ep", 0) == [0, 2] and m.members("mp", 0) == [0, 1, 4, 5]
    c = m.coords(7)
    assert (c.tp, c.dp, c.pp) == (1, 1, 1)
    assert m.is_batch_source(0) and not m.is_batch_source(1) and m.is_pipeline_last(4)
    with pytest.raises(ValueError):
        ParallelMesh(8, tp=3)


def _tp_engine_worker(rank, world, port, out_dir, sp=False):
    _init(rank, world, port)
    from libra_b200.engine.train_engine import B200TrainEngine
    from libra_b200.workflow.synthetic import GRPOWorkload, LengthDist

    eng = B200TrainEngine("tiny", device="cpu", tp_size=2, learning_rate=1e-3, use_distributed_optimizer=False,
                          sequence_parallel=sp)
    eng.initialize()
    assert eng.model.sp == sp
    wl = GRPOWorkload("t", vocab_size=eng.cfg.vocab_size, prompts_per_step=2, group_size=4,
                      prompt=LengthDist(12, 0.3, 4, 24), response=LengthDist(16, 0.3, 2, 32))
    trajs = wl.trajectories(0)
    eng.recompute_logprobs(trajs)
    stats = eng.grpo_update(trajs)
    assert stats["grad_norm"] > 0 and stats["loss"] == stats["loss"]
    # replicated parameters must stay identical on both TP ranks
    for n, p in eng.params.items():
        if p.dim() == 1:
            other = p.detach().clone()
            dist.broadcast(other, src=0)
            torch.testing.assert_close(p.detach(), other, rtol=0, atol=0, msg=n)
    open(os.path.join(out_dir, f"tpe_ok_{rank}"), "w").close()
    dist.destroy_process_group()


@pytest.mark.parametrize("sp", [False, True])
def test_tp_engine_keeps_replicated_params_in_sync(tmp_path, sp):
    _spawn(_tp_engine_worker, 2, str(tmp_path), sp)
    assert {p.name for p in tmp_path.iterdir()} == {"tpe_ok_0", "tpe_ok_1"}


def _ep_engine_worker(rank, world, port, out_dir):
    """EP=2 engine (each rank: its own trajectories, half the experts) against an EP=1 engine that
    sees both ranks' trajectories: same loss, same dense parameters, same experts after one update."""
    _init(rank, world, port)
    from libra_b200.engine.train_engine import B200TrainEngine
    from libra_b200.workflow.synthetic import GRPOWorkload, LengthDist

    wl = GRPOWorkload("ep", vocab_size=2048, prompts_per_step=2, group_size=2, prompt=LengthDist(12, 0.3, 6, 20),
                      response=LengthDist(8, 0.3, 2, 12))
    trajs = [wl.trajectories(0, rank=r) for r in range(world)]
    solo_group = [dist.new_group([r]) for r in range(world)][rank]
    ref = B200TrainEngine("tiny-moe", device="cpu", seed=3, learning_rate=1e-3, micro_batch_size=4,
                          dp_group=solo_group)
    ref.initialize()
    ep = B200TrainEngine("tiny-moe", device="cpu", seed=3, learning_rate=1e-3, micro_batch_size=4, ep_size=2)
    ep.initialize()
    El = ref.cfg.num_experts // world
    for n, p in ep.params.items():
        want = ref.params[n][rank * El:(rank + 1) * El] if "experts." in n else ref.params[n]
        assert torch.equal(p.detach(), want.detach()), n
    s_ref = ref.grpo_update(trajs[0] + trajs[1])
    s_ep = ep.grpo_update(trajs[rank])
    assert abs(s_ref["loss"] - s_ep["loss"]) < 1e-3, (s_ref["loss"], s_ep["loss"])
    assert abs(s_ref["grad_norm"] - s_ep["grad_norm"]) < 1e-2 * max(1.0, s_ref["grad_norm"])
    for n, p in ep.params.items():
        want = ref.params[n][rank * El:(rank + 1) * El] if "experts." in n else ref.params[n]
        torch.testing.assert_close(p.detach().float(), want.detach().float(), rtol=2e-2, atol=2e-3, msg=n)
    open(os.path.join(out_dir, f"epe_ok_{rank}"), "w").close()
    dist.destroy_process_group()


def test_expert_parallel_engine_matches_one_rank(tmp_path):
    _spawn(_ep_engine_worker, 2, str(tmp_path))
    assert {p.name for p in tmp_path.iterdir()} == {"epe_ok_0", "epe_ok_1"}


def _pp_engine_worker(rank, world, port, out_dir, pp):
    """Pipeline-parallel engine (tied embeddings across the first and last
    stage, 1F1B over p2p, DP replicas on identical data) against one rank."""
    _init(rank, world, port)
    import copy

    from libra_b200.engine.train_engine import B200TrainEngine
    from libra_b200.workflow.synthetic import GRPOWorkload, LengthDist

    wl = GRPOWorkload("t", vocab_size=1024, prompts_per_step=2, group_size=4, prompt=LengthDist(12, 0.3, 4, 24),
                      response=LengthDist(16, 0.3, 2, 32))
    trajs = wl.trajectories(0)
    solo = None
    for r in range(world):  # every rank creates every one-rank group, in the same order
        g = dist.new_group([r])
        if r == rank:
            solo = g
    kw = dict(device="cpu", seed=3, learning_rate=1e-3, micro_batch_size=2, max_tokens_per_micro_batch=48)
    ref = B200TrainEngine("tiny", dp_group=solo, **kw)
    ref.initialize()
    eng = B200TrainEngine("tiny", pp_size=pp, **kw)
    eng.initialize()
    assert eng.pp_size == pp and len(eng.params) < len(ref.params)
    for n, p in eng.params.items():
        torch.testing.assert_close(p.detach(), ref.params[n].detach(), rtol=0, atol=0, msg=n)
    t_ref, t_pp = copy.deepcopy(trajs), copy.deepcopy(trajs)
    ref.recompute_logprobs(t_ref)
    eng.recompute_logprobs(t_pp)
    for a, b in zip(t_pp, t_ref):
        torch.testing.assert_close(a["logprobs"], b["logprobs"], rtol=1e-4, atol=1e-5)
    s_ref = ref.grpo_update(t_ref)
    s_pp = eng.grpo_update(t_pp)
    assert abs(s_pp["loss"] - s_ref["loss"]) < 1e-5 and abs(s_pp["grad_norm"] - s_ref["grad_norm"]) < 1e-4 * \
        max(1.0, s_ref["grad_norm"]), (s_pp, s_ref)
    for n, p in eng.params.items():
        torch.testing.assert_close(p.detach().float(), ref.params[n].detach().float(), rtol=1e-2, atol=1e-3, msg=n)
    # distributed checkpoint with per-stage MCore keys + the full-model HF export for rollout
    from libra_b200.engine.checkpointing import DistributedCheckpointManager, load_params_into

    ck = os.path.join(out_dir, "ck")
    DistributedCheckpointManager(ck).save(eng, 1, export_for_rollout=True, include_optimizer=True)
    if rank == 0:
        full = {k: torch.zeros_like(v) for k, v in ref.params.items()}
        load_params_into(full, os.path.join(ck, "v1"), cfg=ref.cfg)
        for n, v in full.items():
            torch.testing.assert_close(v.float(), ref.params[n].detach().float(), rtol=1e-2, atol=1e-3, msg=n)
    back = B200TrainEngine("tiny", pp_size=pp, **dict(kw, seed=11))
    back.initialize()
    DistributedCheckpointManager(ck).load(back, 1)
    for n, p in back.params.items():
        torch.testing.assert_close(p.detach(), eng.params[n].detach(), rtol=0, atol=0, msg=n)
    # the stages' checkpoint loads into one unpipelined replica: same weights and fp32 master weights
    whole = B200TrainEngine("tiny", dp_group=solo, **dict(kw, seed=17))
    whole.initialize()
    DistributedCheckpointManager(ck).load(whole, 1)
    master = eng.optimizer_state_tensors()["master"]
    if eng.sharded:
        parts = [torch.empty_like(master) for _ in range(eng.dp_size)]
        dist.all_gather(parts, master, group=eng.dp_group)
        master = torch.cat(parts)
    for n, p in eng.params.items():
        assert torch.equal(whole.params[n].detach(), p.detach()), n
        o, w = eng.layout.offsets[n], whole.layout.offsets[n]
        assert torch.equal(whole.master[w:w + p.numel()], master[o:o + p.numel()]), n
    # the replica's first stage owns the batch; the other stages receive it from there
    assert eng.is_batch_source() == (eng.pp_rank == 0)
    got = eng.distribute_trajectories(trajs if eng.pp_rank == 0 else None)
    assert len(got) == len(trajs)
    open(os.path.join(out_dir, f"ppe_ok_{rank}"), "w").close()
    dist.destroy_process_group()


@pytest.mark.parametrize("world,pp", [(2, 2), (4, 2)])
def test_pipeline_engine_matches_one_rank(tmp_path, world, pp):
    _spawn(_pp_engine_worker, world, str(tmp_path), pp)
    assert {p.name for p in tmp_path.iterdir() if p.name.startswith("ppe_ok")} == {f"ppe_ok_{r}" for r in range(world)}


@pytest.mark.parametrize("tp", [2, 4])
def test_merge_tp_shards_inverts_sharding(tp):
    """Full parameters -> per-rank TP shards -> merged again is the identity
    (tiny has 2 KV heads, so TP=4 replicates each KV head on two ranks)."""
    from libra_b200.models.qwen3 import get_config
    from libra_b200.parallel.tensor_parallel import merge_tp_shards, shard_full_params

    cfg, full, _ = _model_inputs()
    parts = [shard_full_params(full, cfg, tp, r) for r in range(tp)]
    merged = merge_tp_shards(parts, cfg, tp)
    assert set(merged) == set(full)
    for n, t in full.items():
        assert torch.equal(merged[n], t), n
    moe = get_config("tiny-moe")
    assert moe.is_moe
