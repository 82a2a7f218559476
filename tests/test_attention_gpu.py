"""tcgen05 varlen GQA attention against a plain fp32 PyTorch reference."""

import math

import pytest
import torch

pytestmark = pytest.mark.gpu


def _ref_with_lse(q, k, v, cu, scale):
    T, hq, d = q.shape
    hkv = k.shape[1]
    out = torch.zeros(T, hq, d, dtype=torch.float32, device=q.device)
    lse = torch.zeros(hq, T, dtype=torch.float32, device=q.device)
    b = cu.tolist()
    for s, e in zip(b[:-1], b[1:]):
        if e <= s:
            continue
        qs = q[s:e].float().transpose(0, 1)
        ks = k[s:e].float().transpose(0, 1).repeat_interleave(hq // hkv, 0)
        vs = v[s:e].float().transpose(0, 1).repeat_interleave(hq // hkv, 0)
        att = (qs @ ks.transpose(-1, -2)) * scale
        L = e - s
        att = att.masked_fill(torch.ones(L, L, dtype=torch.bool, device=q.device).triu(1), float("-inf"))
        lse[:, s:e] = torch.logsumexp(att, -1)
        out[s:e] = (att.softmax(-1) @ vs).transpose(0, 1)
    return out, lse


def _inputs(lens, hq=32, hkv=8, d=128, seed=0):
    g = torch.Generator(device="cuda").manual_seed(seed)
    T = sum(lens)
    cu = torch.tensor([0] + list(torch.tensor(lens).cumsum(0).tolist()), dtype=torch.int32, device="cuda")
    q = torch.randn(T, hq, d, device="cuda", generator=g).bfloat16()
    k = torch.randn(T, hkv, d, device="cuda", generator=g).bfloat16()
    v = torch.randn(T, hkv, d, device="cuda", generator=g).bfloat16()
    return q, k, v, cu


@pytest.mark.parametrize("lens", [[128], [1, 7, 130, 255, 256, 513], [1000, 3, 1900], [4096]])
def test_flash_forward_matches_fp32_reference(lens):
    from libra_b200 import ops
    from libra_b200.ops.attention import attn_tiles

    q, k, v, cu = _inputs(lens, seed=len(lens))
    scale = 1.0 / math.sqrt(128)
    tiles = attn_tiles(cu.tolist(), True, "cuda")
    o, lse = ops.ext().flash_fwd(q, k, v, cu, tiles, scale, True, ops.error_flag(q.device))
    torch.cuda.synchronize()
    ops.check_kernel_errors()
    ro, rlse = _ref_with_lse(q, k, v, cu, scale)
    torch.testing.assert_close(o.float(), ro, rtol=2e-2, atol=2e-2)
    torch.testing.assert_close(lse, rlse, rtol=1e-3, atol=2e-3)


def test_flash_autograd_matches_reference_grads():
    from libra_b200 import ops

    lens = [300, 17, 700]
    q, k, v, cu = _inputs(lens, hq=8, hkv=2, seed=5)
    q.requires_grad_(True)
    k.requires_grad_(True)
    v.requires_grad_(True)
    out = ops.varlen_causal_attention(q, k, v, cu, max(lens))
    g = torch.randn_like(out)
    (out.float() * g.float()).sum().backward()
    qr, kr, vr = (t.detach().float().requires_grad_(True) for t in (q, k, v))
    ro, _ = _ref_with_lse(qr, kr, vr, cu, 1.0 / math.sqrt(128))
    (ro * g.float()).sum().backward()
    torch.testing.assert_close(out.float(), ro.detach(), rtol=2e-2, atol=2e-2)
    for a, b in ((q, qr), (k, kr), (v, vr)):
        torch.testing.assert_close(a.grad.float(), b.grad, rtol=5e-2, atol=5e-2)


def test_flash_matches_torch_flash_lse():
    from libra_b200 import ops
    from libra_b200.ops.attention import attn_tiles

    lens = [1024, 512, 77]
    q, k, v, cu = _inputs(lens, seed=9)
    o, lse = ops.ext().flash_fwd(q, k, v, cu, attn_tiles(cu.tolist(), True, "cuda"), 1 / math.sqrt(128), True,
                                 ops.error_flag(q.device))
    to, tlse = torch.ops.aten._flash_attention_forward(q, k, v, cu, cu, max(lens), max(lens), 0.0, True, False)[:2]
    torch.testing.assert_close(o.float(), to.float(), rtol=2e-2, atol=2e-2)
    torch.testing.assert_close(lse, tlse.float(), rtol=1e-3, atol=2e-3)


@pytest.mark.parametrize("lens,hq,hkv", [([128], 4, 1), ([1, 7, 130, 255, 256, 513], 8, 2), ([1000, 3, 1900], 32, 8)])
def test_flash_backward_kernels_match_fp32_reference(lens, hq, hkv):
    from libra_b200 import ops
    from libra_b200.ops.attention import attn_tiles

    q, k, v, cu = _inputs(lens, hq=hq, hkv=hkv, seed=11 + len(lens))
    scale = 1.0 / math.sqrt(128)
    cul = cu.tolist()
    qt, kvt = attn_tiles(cul, True, "cuda"), attn_tiles(cul, True, "cuda", kv=True)
    o, lse = ops.ext().flash_fwd(q, k, v, cu, qt, scale, True, ops.error_flag(q.device))
    g = torch.Generator(device="cuda").manual_seed(3)
    do = torch.randn(q.shape, device="cuda", generator=g).bfloat16()
    dq, dk, dv = ops.ext().flash_bwd(do, q, k, v, o, lse, cu, qt, kvt, scale, True, ops.error_flag(q.device))
    torch.cuda.synchronize()
    ops.check_kernel_errors()
    qr, kr, vr = (t.detach().float().requires_grad_(True) for t in (q, k, v))
    ro, _ = _ref_with_lse(qr, kr, vr, cu, scale)
    (ro * do.float()).sum().backward()
    for name, a, b in (("dq", dq, qr.grad), ("dk", dk, kr.grad), ("dv", dv, vr.grad)):
        err = (a.float() - b).abs().max().item()
        ref = b.abs().max().item()
        assert err <= 2e-2 * max(ref, 1.0), f"{name}: max err {err} (max ref {ref})"


def test_flash_forward_prefix_extend_matches_reference():
    """Queries = the last n tokens of each sequence, keys = the whole sequence."""
    from libra_b200 import ops
    from libra_b200.ops.attention import attn_tiles

    g = torch.Generator(device="cuda").manual_seed(21)
    lens_k, lens_q = [300, 1000, 129, 7], [1, 200, 129, 3]
    hq, hkv, d = 8, 2, 128
    ks = [torch.randn(L, hkv, d, device="cuda", generator=g).bfloat16() for L in lens_k]
    vs = [torch.randn(L, hkv, d, device="cuda", generator=g).bfloat16() for L in lens_k]
    qs = [torch.randn(L, hq, d, device="cuda", generator=g).bfloat16() for L in lens_k]
    cu_q = [0]
    cu_k = [0]
    for a, b in zip(lens_q, lens_k):
        cu_q.append(cu_q[-1] + a)
        cu_k.append(cu_k[-1] + b)
    qx = torch.cat([q[L - n:] for q, L, n in zip(qs, lens_k, lens_q)])
    scale = 1.0 / math.sqrt(d)
    o, _ = ops.ext().flash_fwd(qx, torch.cat(ks), torch.cat(vs), torch.tensor(cu_q, device="cuda", dtype=torch.int32),
                               attn_tiles(cu_q, True, "cuda"), scale, True, ops.error_flag(qx.device),
                               torch.tensor(cu_k, device="cuda", dtype=torch.int32))
    torch.cuda.synchronize()
    ops.check_kernel_errors()
    refs = []
    for q, k, v, L, n in zip(qs, ks, vs, lens_k, lens_q):
        full, _ = _ref_with_lse(q, k, v, torch.tensor([0, L], device="cuda", dtype=torch.int32), scale)
        refs.append(full[L - n:])
    torch.testing.assert_close(o.float(), torch.cat(refs), rtol=2e-2, atol=2e-2)
