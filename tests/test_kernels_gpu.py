"""Numerics of every sm_100a kernel against a plain PyTorch fp32 reference."""

import math

import pytest
import torch

pytestmark = pytest.mark.gpu

DEV = "cuda"


def _bf16(*shape, scale=1.0, seed=0):
    g = torch.Generator(device=DEV).manual_seed(seed)
    return (torch.randn(*shape, generator=g, device=DEV) * scale).to(torch.bfloat16)


def _rel(a, b):
    a, b = a.float(), b.float()
    return ((a - b).norm() / (b.norm() + 1e-12)).item()


# ---------------------------------------------------------------- GEMM
GEMM_SHAPES = [(128, 128, 64), (300, 264, 200), (1000, 520, 136), (4096, 4096, 2560), (129, 2048, 4096),
               (2056, 256, 8), (200, 136, 777)]


@pytest.mark.parametrize("M,N,K", GEMM_SHAPES)
@pytest.mark.parametrize("a_mn,b_mn", [(False, False), (False, True), (True, True), (True, False)])
def test_gemm_layouts(M, N, K, a_mn, b_mn):
    from libra_b200 import ops

    lda = M if a_mn else K
    ldb = N if b_mn else K
    if lda % 8 or ldb % 8:
        pytest.skip("TMA needs every leading dimension to be a multiple of 8 elements")
    A = _bf16(M, K, seed=1)  # logical [M, K]
    B = _bf16(N, K, seed=2)  # logical [N, K]
    a = A.t().contiguous() if a_mn else A
    b = B.t().contiguous() if b_mn else B
    out = ops.gemm(a, b, a_mn=a_mn, b_mn=b_mn)
    torch.cuda.synchronize()
    ops.check_kernel_errors()
    ref = A.float() @ B.float().t()
    assert _rel(out, ref) < 8e-3


@pytest.mark.parametrize("M,N,K", [(512, 384, 256), (333, 1024, 520), (1024, 768, 4096)])
def test_gemm_epilogues(M, N, K):
    from libra_b200 import ops

    A, B = _bf16(M, K, seed=3), _bf16(N, K, seed=4)
    ref = A.float() @ B.float().t()
    f32 = ops.gemm(A, B, epi=ops.EPI_F32)
    assert f32.dtype == torch.float32 and _rel(f32, ref) < 1e-4
    acc = torch.ones(M, N, device=DEV)
    ops.gemm(A, B, out=acc, epi=ops.EPI_ACC_F32)
    assert _rel(acc, ref + 1) < 1e-4
    R = _bf16(M, N, seed=5)
    res = ops.gemm(A, B, epi=ops.EPI_BF16_RESIDUAL, residual=R)
    assert _rel(res, ref + R.float()) < 8e-3
    ops.check_kernel_errors()


def test_linear_autograd_main_grad():
    from libra_b200 import ops

    x = _bf16(777, 512, seed=6).requires_grad_(True)
    w = torch.nn.Parameter(_bf16(1024, 512, scale=0.05, seed=7))
    w.main_grad = torch.zeros(1024, 512, device=DEV)
    y = ops.linear(x, w)
    dy = _bf16(777, 1024, seed=8)
    y.backward(dy)
    xf, wf = x.detach().float().requires_grad_(True), w.detach().float().requires_grad_(True)
    yf = xf @ wf.t()
    yf.backward(dy.float())
    assert _rel(y, yf) < 8e-3
    assert _rel(x.grad, xf.grad) < 8e-3
    assert _rel(w.main_grad, wf.grad) < 1e-3
    assert w.grad is None


# ---------------------------------------------------------------- norms / rope / swiglu
def test_rmsnorm_fwd_bwd():
    from libra_b200 import ops

    x = _bf16(1000, 2560, seed=9).requires_grad_(True)
    w = torch.nn.Parameter((1 + 0.1 * torch.randn(2560, device=DEV)).to(torch.bfloat16))
    y = ops.rmsnorm(x, w, 1e-6)
    dy = _bf16(1000, 2560, seed=10)
    y.backward(dy)
    xf, wf = x.detach().float().requires_grad_(True), w.detach().float().requires_grad_(True)
    yf = xf * torch.rsqrt(xf.pow(2).mean(-1, keepdim=True) + 1e-6) * wf
    yf.backward(dy.float())
    assert _rel(y, yf) < 8e-3
    assert _rel(x.grad, xf.grad) < 1e-2
    assert _rel(w.grad, wf.grad) < 1e-2


@pytest.mark.parametrize("H", [1024, 2048, 2560, 4096, 6144])
def test_rmsnorm_bwd_widths_and_accumulate(H):
    """Every row-width variant of the backward (register-resident up to 4096,
    two-pass beyond), with dx accumulated into an existing gradient."""
    from libra_b200 import ops

    T = 777
    x, dy = _bf16(T, H, seed=21), _bf16(T, H, seed=22)
    w = (1 + 0.1 * torch.randn(H, device=DEV)).to(torch.bfloat16)
    prev = _bf16(T, H, seed=23)
    rstd = torch.rsqrt(x.float().pow(2).mean(-1) + 1e-6).contiguous()
    dw = torch.zeros(H, device=DEV)
    dx = prev.clone()
    ops.ext().rmsnorm_bwd(dy, x, w, rstd, dw, False, dx)
    torch.cuda.synchronize()
    xf, wf = x.float().requires_grad_(True), w.float().requires_grad_(True)
    (xf * torch.rsqrt(xf.pow(2).mean(-1, keepdim=True) + 1e-6) * wf).backward(dy.float())
    assert _rel(dx, xf.grad + prev.float()) < 1e-2
    assert _rel(dw, wf.grad) < 1e-2


def test_qk_norm_rope_fwd_bwd():
    from libra_b200 import ops
    from libra_b200.ops import reference as ref

    T, nq, nkv, D = 300, 8, 2, 128
    qkv = _bf16(T, (nq + 2 * nkv) * D, seed=11).requires_grad_(True)
    qw = torch.nn.Parameter((1 + 0.1 * torch.randn(D, device=DEV)).to(torch.bfloat16))
    kw = torch.nn.Parameter((1 + 0.1 * torch.randn(D, device=DEV)).to(torch.bfloat16))
    pos = torch.randint(0, 4000, (T,), device=DEV, dtype=torch.int32)
    cos, sin = ref.rope_tables(4096, D, 1e6, DEV)
    q, k, v = ops.qk_norm_rope(qkv, qw, kw, pos, cos, sin, nq, nkv, 1e-6)
    gq, gk, gv = _bf16(*q.shape, seed=12), _bf16(*k.shape, seed=13), _bf16(*v.shape, seed=14)
    (q.float() * gq.float()).sum().add((k.float() * gk.float()).sum()).add((v.float() * gv.float()).sum()).backward()

    xf = qkv.detach().float().requires_grad_(True)
    qwf, kwf = qw.detach().float().requires_grad_(True), kw.detach().float().requires_grad_(True)
    x = xf.view(T, nq + 2 * nkv, D)
    qr, kr, vr = x[:, :nq], x[:, nq:nq + nkv], x[:, nq + nkv:]
    norm = lambda t, w: t * torch.rsqrt(t.pow(2).mean(-1, keepdim=True) + 1e-6) * w  # noqa: E731
    qr = ref.apply_rope(norm(qr, qwf), cos, sin, pos)
    kr = ref.apply_rope(norm(kr, kwf), cos, sin, pos)
    ((qr * gq.float()).sum() + (kr * gk.float()).sum() + (vr * gv.float()).sum()).backward()
    assert _rel(q, qr) < 8e-3 and _rel(k, kr) < 8e-3 and _rel(v, vr) < 1e-6
    assert _rel(qkv.grad, xf.grad) < 1e-2
    assert _rel(qw.grad, qwf.grad) < 1e-2 and _rel(kw.grad, kwf.grad) < 1e-2


def test_swiglu_fwd_bwd():
    from libra_b200 import ops

    gu = _bf16(513, 2 * 1024, seed=15).requires_grad_(True)
    h = ops.swiglu(gu)
    dh = _bf16(513, 1024, seed=16)
    h.backward(dh)
    g = gu.detach().float().requires_grad_(True)
    a, b = g.chunk(2, -1)
    hf = torch.nn.functional.silu(a) * b
    hf.backward(dh.float())
    assert _rel(h, hf) < 8e-3
    assert _rel(gu.grad, g.grad) < 1e-2


# ---------------------------------------------------------------- logprob
@pytest.mark.parametrize("R,V", [(64, 151936), (300, 2048), (17, 1000)])
def test_lm_head_logprob(R, V):
    from libra_b200 import ops

    H = 256
    h = _bf16(R, H, seed=17).requires_grad_(True)
    w = torch.nn.Parameter(_bf16(V, H, scale=0.1, seed=18))
    tgt = torch.randint(0, V, (R,), device=DEV)
    ent = torch.empty(R, device=DEV)
    lp = ops.lm_head_logprob(h, w, tgt, 1.0, ent)
    g = torch.randn(R, device=DEV)
    lp.backward(g)
    hf, wf = h.detach().float().requires_grad_(True), w.detach().float().requires_grad_(True)
    logits = (hf @ wf.t()).to(torch.bfloat16).float()  # kernel reduces bf16 logits
    ls = torch.log_softmax(logits, -1)
    lpf = ls.gather(-1, tgt[:, None]).squeeze(-1)
    entf = -(ls.exp() * ls).sum(-1)
    lpf.backward(g)
    assert (lp - lpf).abs().max().item() < 2e-3
    assert (ent - entf).abs().max().item() < 2e-3
    assert _rel(h.grad, hf.grad) < 2e-2
    assert _rel(w.grad, wf.grad) < 2e-2


def test_adamw_matches_reference():
    from libra_b200 import ops

    n = 10_001
    g = torch.Generator(device=DEV).manual_seed(3)
    master = torch.randn(n, device=DEV, generator=g)
    grad = torch.randn(n, device=DEV, generator=g)
    m, v = torch.zeros(n, device=DEV), torch.zeros(n, device=DEV)
    p = master.to(torch.bfloat16)
    rm, rg, rmm, rv, rp = master.cpu(), grad.cpu(), m.cpu(), v.cpu(), p.cpu()
    sq = torch.zeros(1, device=DEV)
    ops.grad_sq_norm(grad, sq)
    assert abs(sq.item() - float(grad.double().pow(2).sum())) / sq.item() < 1e-4
    for step in (1, 2):
        ops.adamw_step(master, grad, m, v, p, lr=1e-3, beta1=0.9, beta2=0.95, eps=1e-8, weight_decay=0.01,
                       step=step, max_grad_norm=1.0, sq_norm=sq)
        ops.adamw_step(rm, rg, rmm, rv, rp, lr=1e-3, beta1=0.9, beta2=0.95, eps=1e-8, weight_decay=0.01,
                       step=step, max_grad_norm=1.0, sq_norm=sq.cpu())
    assert torch.allclose(master.cpu(), rm, atol=1e-5, rtol=1e-5)
    assert torch.allclose(p.float().cpu(), rp.float(), atol=1e-2)


def test_adamw_bf16_moments_match_reference():
    """Precision-aware optimizer state: bf16 moments updated in fp32 by the kernel (plain and
    parameter-gather variants) against the fp32-math CPU reference with the same bf16 storage."""
    from libra_b200 import ops
    from libra_b200.parallel.peer_param_gather import PeerParamGather

    n = 100_003
    g = torch.Generator(device=DEV).manual_seed(4)
    master0 = torch.randn(n, device=DEV, generator=g)
    grad = torch.randn(n, device=DEV, generator=g)
    sq = grad.pow(2).sum().reshape(1)
    hp = dict(lr=1e-3, beta1=0.9, beta2=0.95, eps=1e-8, weight_decay=0.01, max_grad_norm=1.0)
    rm, rmm, rv = master0.cpu(), torch.zeros(n, dtype=torch.bfloat16), torch.zeros(n, dtype=torch.bfloat16)
    rp = torch.zeros(n, dtype=torch.bfloat16)
    master, m = master0.clone(), torch.zeros(n, dtype=torch.bfloat16, device=DEV)
    v, p = torch.zeros_like(m), torch.zeros(n, dtype=torch.bfloat16, device=DEV)
    m2, v2, master2 = m.clone(), v.clone(), master0.clone()
    for step in (1, 2, 3):
        ops.adamw_step(master, grad, m, v, p, step=step, sq_norm=sq, **hp)
        ops.adamw_step(rm, grad.cpu(), rmm, rv, rp, step=step, sq_norm=sq.cpu(), **hp)
    torch.cuda.synchronize()
    ops.check_kernel_errors()
    assert m.dtype == torch.bfloat16
    torch.testing.assert_close(master.cpu(), rm, rtol=1e-5, atol=1e-6)
    torch.testing.assert_close(m.float().cpu(), rmm.float(), rtol=1e-2, atol=1e-6)
    torch.testing.assert_close(v.float().cpu(), rv.float(), rtol=1e-2, atol=1e-8)
    # the fused parameter-gather variant with bf16 moments (one rank): same state, same parameters
    k = n - n % 4
    flat = torch.zeros(k, dtype=torch.bfloat16, device=DEV)
    pg = PeerParamGather(None, flat, 0, k)
    for step in (1, 2, 3):
        pg.step(master2[:k], grad[:k], m2[:k], v2[:k], step=step, sq_norm=sq, **hp)
    torch.cuda.synchronize()
    ops.check_kernel_errors()
    assert torch.equal(master2[:k], master[:k]) and torch.equal(m2[:k], m[:k]) and torch.equal(v2[:k], v[:k])
    assert torch.equal(flat[:k], p[:k])
    pg.close()


# ---------------------------------------------------------------- model
def test_model_matches_fp32_reference():
    """tiny-gpu model: CUDA kernels vs the same weights on the CPU fp32 path."""
    from libra_b200.engine.train_engine import B200TrainEngine
    from libra_b200.workflow.synthetic import GRPOWorkload, LengthDist

    wl = GRPOWorkload("t", vocab_size=2048, prompts_per_step=2, group_size=2, prompt=LengthDist(40, 0.2, 16, 64),
                      response=LengthDist(50, 0.2, 8, 96))
    trajs = wl.trajectories(0)
    gpu = B200TrainEngine("tiny-gpu", device="cuda", seed=1, micro_batch_size=4)
    gpu.initialize()
    cpu = B200TrainEngine("tiny-gpu", device="cpu", seed=1, micro_batch_size=4)
    cpu.initialize()
    cpu.flat_param.copy_(gpu.flat_param.cpu())
    bg = gpu.to_device(gpu.pack(trajs))
    bc = cpu.pack(trajs)
    lg = gpu.model.action_logprobs(bg["batch"])
    lc = cpu.model.action_logprobs(bc["batch"])
    assert (lg.cpu() - lc).abs().max().item() < 5e-2
    lossg, _, _ = gpu.loss(lg, bg["old_logp"], bg["adv"])
    lossc, _, _ = cpu.loss(lc, bc["old_logp"], bc["adv"])
    lossg.backward()
    lossc.backward()
    assert _rel(gpu.flat_grad.cpu(), cpu.flat_grad) < 5e-2


def test_engine_step_reduces_loss():
    from libra_b200.engine.train_engine import B200TrainEngine
    from libra_b200.workflow.synthetic import GRPOWorkload, LengthDist

    wl = GRPOWorkload("t", vocab_size=2048, prompts_per_step=2, group_size=4, prompt=LengthDist(40, 0.2, 16, 64),
                      response=LengthDist(50, 0.2, 8, 96))
    trajs = wl.trajectories(0)
    eng = B200TrainEngine("tiny-gpu", device="cuda", seed=2, micro_batch_size=4, learning_rate=1e-3)
    eng.initialize()
    eng.recompute_logprobs(trajs)
    first = eng.grpo_update(trajs)["loss"]
    for _ in range(4):
        last = eng.grpo_update(trajs)["loss"]
    assert last < first


@pytest.mark.gpu
@pytest.mark.parametrize("M,K,F", [(300, 512, 256), (4096, 2560, 9728), (1, 128, 128)])
def test_linear_swiglu_matches_unfused(M, K, F):
    from libra_b200 import ops

    g = torch.Generator(device="cuda").manual_seed(M + F)
    x = (torch.randn(M, K, device="cuda", generator=g) * 0.5).bfloat16().requires_grad_(True)
    w = (torch.randn(2 * F, K, device="cuda", generator=g) / K ** 0.5).bfloat16().requires_grad_(True)
    a = ops.linear_swiglu(x, w)
    x2, w2 = x.detach().clone().requires_grad_(True), w.detach().clone().requires_grad_(True)
    a2 = ops.swiglu(ops.linear(x2, w2))
    torch.cuda.synchronize()
    ops.check_kernel_errors()
    torch.testing.assert_close(a.float(), a2.float(), rtol=1e-2, atol=1e-2)
    da = torch.randn_like(a)
    a.backward(da)
    a2.backward(da)
    torch.testing.assert_close(x.grad.float(), x2.grad.float(), rtol=1e-2, atol=1e-2)
    torch.testing.assert_close(w.grad.float(), w2.grad.float(), rtol=1e-2, atol=1e-2)
    with torch.no_grad():  # inference path: no gate/up buffer kept
        torch.testing.assert_close(ops.linear_swiglu(x, w).float(), a2.float(), rtol=1e-2, atol=1e-2)
