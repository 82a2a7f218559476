"""Grouped expert GEMM (tcgen05, group offsets in device memory) against fp32
per-group matmuls: forward, SwiGLU forward, dgrad and accumulated wgrad, with
empty groups and groups of odd sizes padded to 128 rows."""

import pytest
import torch

pytestmark = pytest.mark.gpu


def _layout(counts, align=128):
    offs = [0]
    for c in counts:
        offs.append(offs[-1] + (c + align - 1) // align * align)
    return offs


def _inputs(counts, K, seed):
    g = torch.Generator(device="cuda").manual_seed(seed)
    offs = _layout(counts)
    x = torch.zeros(offs[-1] + 64, K, device="cuda")
    for e, c in enumerate(counts):
        x[offs[e]:offs[e] + c] = torch.randn(c, K, device="cuda", generator=g)
    return x.bfloat16(), torch.tensor(offs, dtype=torch.int32, device="cuda"), offs


@pytest.mark.parametrize("counts,K,N", [([5, 0, 300, 128, 1], 512, 256), ([1000, 77, 0, 0, 513, 64, 9, 200], 2048, 768)])
def test_grouped_linear_forward_backward(counts, K, N):
    from libra_b200 import ops

    G = len(counts)
    x, offs_t, offs = _inputs(counts, K, seed=G)
    w = (torch.randn(G, N, K, device="cuda") * 0.05).bfloat16()
    x.requires_grad_(True)
    w.requires_grad_(True)
    y = ops.grouped_linear(x, w, offs_t)
    dy = torch.zeros_like(y)
    for e, c in enumerate(counts):
        dy[offs[e]:offs[e] + c] = torch.randn(c, N, device="cuda").bfloat16()
    y.backward(dy)
    torch.cuda.synchronize()
    ops.check_kernel_errors()
    for e, c in enumerate(counts):
        a, b = offs[e], offs[e] + c
        ref = x[a:b].float() @ w[e].float().t()
        torch.testing.assert_close(y[a:b].float(), ref, rtol=2e-2, atol=2e-2)
        torch.testing.assert_close(x.grad[a:b].float(), dy[a:b].float() @ w[e].float(), rtol=2e-2, atol=2e-2)
        dw_ref = dy[a:b].float().t() @ x[a:b].float()
        torch.testing.assert_close(w.grad[e].float(), dw_ref, rtol=3e-2, atol=3e-2)
        assert float(y[b:offs[e + 1]].abs().max() if offs[e + 1] > b else 0.0) == 0.0  # padding rows stay zero


def test_grouped_swiglu_and_main_grad_accumulation():
    from libra_b200 import ops

    counts, K, F = [33, 256, 0, 130], 512, 256
    G = len(counts)
    torch.manual_seed(7)  # w and da come from the global generator
    x, offs_t, offs = _inputs(counts, K, seed=7)
    w = (torch.randn(G, 2 * F, K, device="cuda") * 0.05).bfloat16().requires_grad_(True)
    w.main_grad = torch.ones(G, 2 * F, K, device="cuda")  # accumulates on top of what is there
    x.requires_grad_(True)
    a = ops.grouped_swiglu(x, w, offs_t)
    da = torch.randn_like(a)
    a.backward(da)
    torch.cuda.synchronize()
    for e, c in enumerate(counts):
        lo, hi = offs[e], offs[e] + c
        xf = x[lo:hi].float().detach().requires_grad_(True)
        wf = w[e].float().detach().requires_grad_(True)
        gu = (xf @ wf.t()).bfloat16().float()
        ref = torch.nn.functional.silu(gu[:, :F]) * gu[:, F:]
        torch.testing.assert_close(a[lo:hi].float(), ref, rtol=2e-2, atol=2e-2)
        ref.backward(da[lo:hi].float())
        torch.testing.assert_close(x.grad[lo:hi].float(), xf.grad, rtol=3e-2, atol=3e-2)
        # dW sums bf16-rounded activation gradients over up to 256 rows: a few ulps of noise
        torch.testing.assert_close(w.main_grad[e] - 1.0, wf.grad, rtol=3e-2, atol=6e-2)
    assert w.grad is None  # the gradient went into main_grad


def test_moe_block_grouped_matches_loop_on_gpu():
    from libra_b200.models.moe import moe_mlp, moe_mlp_looped
    from libra_b200.models.qwen3 import get_config

    cfg = get_config("tiny-moe")
    g = torch.Generator(device="cuda").manual_seed(1)
    T, H, E, F = 300, cfg.hidden_size, cfg.num_experts, cfg.moe_intermediate_size
    h = (torch.randn(T, H, device="cuda", generator=g) * 0.5).bfloat16()
    res = torch.randn(T, H, device="cuda", generator=g).bfloat16()
    router = torch.randn(E, H, device="cuda", generator=g) * 0.05
    w1 = (torch.randn(E, 2 * F, H, device="cuda", generator=g) * 0.05).bfloat16()
    w2 = (torch.randn(E, H, F, device="cuda", generator=g) * 0.05).bfloat16()
    torch.testing.assert_close(moe_mlp(h, res, router, w1, w2, cfg).float(),
                               moe_mlp_looped(h, res, router, w1, w2, cfg).float(), rtol=2e-2, atol=2e-2)
