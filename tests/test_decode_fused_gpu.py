"""Fused decode-step kernels on the GPU against fp32 PyTorch references:
stream-K GEMM, q/k norm + RoPE + KV write, residual + RMSNorm, SwiGLU,
stream-K paged attention, fp32-logit sampling, and the fused captured step
against the unfused one."""

import math

import pytest
import torch

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("M,N,K", [(1, 256, 64), (7, 6144, 2560), (64, 2560, 9728), (64, 19456, 2560),
                                   (128, 2560, 4096), (200, 1024, 704), (64, 151936 // 8, 2560)])
def test_gemm_streamk_matches_fp32(M, N, K):
    from libra_b200 import ops

    torch.manual_seed(M + N + K)
    a = torch.randn(M, K, device="cuda").bfloat16()
    w = (torch.randn(N, K, device="cuda") / math.sqrt(K)).bfloat16()
    acc = torch.zeros(M, N, device="cuda")
    ops.gemm_streamk(a, w, acc)
    ops.gemm_streamk(a, w, acc)  # accumulates: 2 x
    torch.cuda.synchronize()
    ops.check_kernel_errors(a.device)
    ref = 2 * (a.float() @ w.float().t())
    err = (acc - ref).abs().max().item()
    assert err < 2e-3 * max(1.0, ref.abs().max().item()), err


@pytest.mark.parametrize("M,N,K", [(1, 256, 64), (7, 6144, 2560), (33, 2560, 4096), (64, 2560, 9728),
                                   (64, 19456, 2560), (100, 1000, 704), (128, 2560, 4096), (129, 384, 2560),
                                   (256, 6144, 2560), (64, 151936 // 8, 2560)])
@pytest.mark.parametrize("pdl", [False, True])
def test_gemm_decode_matches_fp32(M, N, K, pdl):
    from libra_b200 import ops

    torch.manual_seed(M * 3 + N + K)
    x = torch.randn(M, K, device="cuda").bfloat16()
    w = (torch.randn(N, K, device="cuda") / math.sqrt(K)).bfloat16()
    acc = torch.randn(M, N, device="cuda")
    start = acc.clone()
    ops.gemm_decode(x, w, acc, pdl=pdl)
    ops.gemm_decode(x, w, acc, pdl=pdl)  # accumulates: start + 2 x
    torch.cuda.synchronize()
    ops.check_kernel_errors(x.device)
    ref = start + 2 * (x.float() @ w.float().t())
    err = (acc - ref).abs().max().item()
    assert err < 2e-3 * max(1.0, ref.abs().max().item()), err


def test_qkv_post_matches_reference():
    from libra_b200 import ops
    from libra_b200.ops import reference as ref

    torch.manual_seed(1)
    B, nq, nkv, D, bs = 37, 32, 8, 128, 16
    acc = torch.randn(B, (nq + 2 * nkv) * D, device="cuda")
    acc_copy = acc.clone()
    qw = (1 + 0.1 * torch.randn(D, device="cuda")).bfloat16()
    kw = (1 + 0.1 * torch.randn(D, device="cuda")).bfloat16()
    cos, sin = ref.rope_tables(4096, D, 1e6, torch.device("cuda"))
    pos = torch.randint(0, 4000, (B,), device="cuda", dtype=torch.int32)
    nblocks = 64
    slot = torch.randperm(nblocks * bs, device="cuda")[:B].long()
    kc = torch.zeros(nblocks, bs, nkv, D, device="cuda").bfloat16()
    vc = torch.zeros_like(kc)
    q_out = torch.empty(B, nq, D, device="cuda").bfloat16()
    ops.decode_qkv_post(acc, qw, kw, pos, cos, sin, slot, q_out, kc, vc, 1e-6)
    torch.cuda.synchronize()
    assert acc.abs().max().item() == 0.0  # the accumulator is left zeroed
    q, k, v = ref.qk_norm_rope(acc_copy.bfloat16(), qw, kw, pos, cos, sin, nq, nkv, 1e-6)
    assert (q_out.float() - q.float()).abs().max().item() < 2e-2
    assert (kc.view(-1, nkv, D)[slot].float() - k.float()).abs().max().item() < 2e-2
    assert torch.equal(vc.view(-1, nkv, D)[slot], v.bfloat16())


@pytest.mark.parametrize("B,H", [(1, 2560), (64, 2560), (130, 5120), (3, 8192)])
def test_residual_norm_and_swiglu(B, H):
    from libra_b200 import ops
    from libra_b200.ops import reference as ref

    torch.manual_seed(B)
    x = torch.randn(B, H, device="cuda").bfloat16()
    acc = torch.randn(B + 5, H, device="cuda")
    w = torch.randn(H, device="cuda").bfloat16()
    x_ref = (x.float() + acc[:B]).bfloat16()
    h_ref = ref.rmsnorm(x_ref, w, 1e-6)
    h = torch.empty_like(x)
    tail = acc[B:].clone()
    ops.decode_residual_norm(x, acc[:B], w, h, 1e-6)
    torch.cuda.synchronize()
    assert torch.equal(x, x_ref)
    assert (h.float() - h_ref.float()).abs().max().item() < 3e-2
    assert acc[:B].abs().max().item() == 0.0 and torch.equal(acc[B:], tail)
    F = H // 2
    gu = torch.randn(B, 2 * F, device="cuda")
    gb = gu.bfloat16().float()
    a_ref = torch.nn.functional.silu(gb[:, :F]) * gb[:, F:]
    a = torch.empty(B, F, device="cuda").bfloat16()
    ops.decode_swiglu(gu, a)
    torch.cuda.synchronize()
    assert gu.abs().max().item() == 0.0
    assert (a.float() - a_ref).abs().max().item() < 2e-2 * max(1.0, a_ref.abs().max().item())


def _attn_reference(q, kc, vc, tables, lens, scale):
    B, Hq, D = q.shape
    Hkv, bs = kc.shape[2], kc.shape[1]
    out = torch.empty(B, Hq, D, device=q.device)
    for b, L in enumerate(lens):
        idx = torch.arange(L, device=q.device)
        blocks = tables[b, idx // bs].long()
        k = kc[blocks, idx % bs].float().repeat_interleave(Hq // Hkv, 1)
        v = vc[blocks, idx % bs].float().repeat_interleave(Hq // Hkv, 1)
        s = torch.einsum("hd,lhd->hl", q[b].float(), k) * scale
        out[b] = torch.einsum("hl,lhd->hd", s.softmax(-1), v)
    return out


@pytest.mark.parametrize("Hkv,G,lens", [
    (8, 4, [1, 17, 300, 2049, 16, 32, 5000]),          # Qwen3-4B / 8B heads
    (8, 4, [510] * 64),                                 # a decode batch, every sequence split over CTAs
    (8, 4, [3] * 200),                                  # many short sequences per CTA
    (4, 8, [129, 700, 1]),                              # Qwen3-30B-A3B heads
    (8, 5, [64, 4097]),                                 # Qwen3-14B heads
    (2, 2, [45, 1000, 7]), (1, 1, [33, 2]),
])
def test_decode_attention_matches_reference(Hkv, G, lens):
    from libra_b200 import ops

    torch.manual_seed(len(lens) * 7 + G)
    B, D, bs = len(lens), 128, 16
    Hq = G * Hkv
    nblk = sum(-(-L // bs) for L in lens) + 3
    kc = torch.randn(nblk, bs, Hkv, D, device="cuda").bfloat16()
    vc = torch.randn(nblk, bs, Hkv, D, device="cuda").bfloat16()
    perm = torch.randperm(nblk).tolist()
    width = max(-(-L // bs) for L in lens) + 2
    bt = torch.zeros(B + 3, width, dtype=torch.int32)
    cur = 0
    for i, L in enumerate(lens):
        n = -(-L // bs)
        bt[i, :n] = torch.tensor(perm[cur:cur + n])
        cur += n
    bt = bt.cuda()
    lens_t = torch.tensor(lens + [1, 1, 1], dtype=torch.int32, device="cuda")
    q = torch.randn(B + 3, Hq, D, device="cuda").bfloat16()
    part_o, part_ml, counters = ops.decode_workspace(B + 3, Hq, D, q.device)
    out = torch.empty(B, Hq, D, device="cuda").bfloat16()
    scale = 1.0 / math.sqrt(D)
    ref = _attn_reference(q[:B], kc, vc, bt, lens, scale)
    for _ in range(2):  # the second call checks that the kernel left its counters at zero
        out.zero_()
        ops.decode_attention(q, kc, vc, bt, lens_t, out, part_o, part_ml, counters, scale)
        torch.cuda.synchronize()
        ops.check_kernel_errors(q.device)
        assert counters.abs().max().item() == 0
        err = (out.float() - ref).abs().max().item()
        assert err < 2e-2, err


def test_sample_fp32_logits_zeroes_and_matches_bf16():
    from libra_b200 import ops

    torch.manual_seed(3)
    B, V, W = 5, 151937, 151940  # a vocabulary tail (V % 4 = 1) inside rows padded to 16 bytes
    buf = (3 * torch.randn(B, W, device="cuda")).bfloat16().float()  # exact in bf16: both paths see the same
    logits = buf[:, :V]
    temp = torch.tensor([1.0, 0.0, 0.7, 1.3, 1.0], device="cuda")
    seeds = torch.arange(B, device="cuda", dtype=torch.long) * 11 + 5
    pos = torch.arange(B, device="cuda", dtype=torch.long) + 100
    t1, l1 = torch.empty(B, dtype=torch.long, device="cuda"), torch.empty(B, device="cuda")
    t2, l2 = torch.empty_like(t1), torch.empty_like(l1)
    ops.sample_tokens(buf.bfloat16()[:, :V], temp, seeds, pos, t1, l1)
    ops.sample_tokens(logits, temp, seeds, pos, t2, l2)
    torch.cuda.synchronize()
    assert torch.equal(t1, t2)
    assert (l1 - l2).abs().max().item() < 1e-4
    assert buf[:, :V].abs().max().item() == 0.0  # the fp32 logits are zeroed behind the read
    assert buf[:, V:].abs().max().item() > 0.0   # and nothing past the vocabulary


def test_fused_decode_graphs_match_unfused(monkeypatch):
    from libra_b200.engine.rollout.llm_engine import LLMEngine
    from libra_b200.engine.rollout.sampler import SamplingParams
    from libra_b200.engine.train_engine import B200TrainEngine

    eng = B200TrainEngine("tiny-gpu", device="cuda", seed=5)
    eng.initialize()
    prompts = [list(range(5, 45)), [7, 8, 9], list(range(100, 400)), list(range(3, 20))]
    params = [SamplingParams(max_tokens=n, temperature=0.0) for n in (40, 7, 25, 33)]

    def run(fused: bool):
        monkeypatch.setenv("LIBRA_DECODE_GRAPHS", "1")
        monkeypatch.setenv("LIBRA_DECODE_FUSED", "1" if fused else "0")
        llm = LLMEngine(eng.cfg, eng.params, kv_blocks=512, block_size=16, max_model_len=1024, max_running=64)
        res = {}
        ids = [llm.add_request(p, sp, callback=lambda r: res.__setitem__(r.request_id, r))
               for p, sp in zip(prompts, params)]
        while len(res) < len(ids):
            llm.step()
        return [res[i] for i in ids], llm

    base, _ = run(False)
    fused, llm = run(True)
    assert llm._graphs is not None and llm._graphs.fused and llm._graphs.replays > 0
    agree = total = 0
    for a, b in zip(base, fused):
        # greedy decoding: identical until a near-tie flips one token (fp32 vs bf16 logits)
        for x, y in zip(a.output_tokens, b.output_tokens):
            total += 1
            if x != y:
                break
            agree += 1
        n = min(len(a.output_logprobs), len(b.output_logprobs), 3)
        assert max(abs(x - y) for x, y in zip(a.output_logprobs[:n], b.output_logprobs[:n])) < 5e-2
    assert agree >= 0.9 * total
