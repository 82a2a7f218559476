"""Fused sm_100a operators with autograd.

Every op dispatches on the device of its inputs:

* CUDA tensors run the hand-written kernels in ``libra_b200._C`` (tcgen05 GEMM,
  RMSNorm, q/k-norm+RoPE, SwiGLU, fused logprob, AdamW).  If the extension is
  missing on a machine with a GPU the call raises; there is no silent fallback.
* CPU tensors run the fp32 PyTorch reference in :mod:`libra_b200.ops.reference`
  (used by the gloo multi-process plumbing tests and as the numerics oracle).

Weight gradients follow the "main_grad" convention of Megatron-Core's gradient
accumulation fusion: when a weight carries a ``main_grad`` fp32 tensor (a view
into the engine's flat gradient buffer) the backward pass accumulates into it
directly from the GEMM epilogue and returns ``None`` for the weight.
"""

from __future__ import annotations

import math
import os
from typing import Optional

import torch

from . import reference as ref

_EXT = None
_ERR = {}

EPI_BF16, EPI_F32, EPI_ACC_F32, EPI_BF16_RESIDUAL = 0, 1, 2, 3


def ext():
    """The compiled extension; raises with a build hint when absent."""
    global _EXT
    if _EXT is None:
        try:
            from libra_b200 import _C  # noqa: WPS433
        except ImportError as exc:  # pragma: no cover - exercised only without a build
            raise RuntimeError(
                "libra_b200._C is not built; run `python setup.py build_ext --inplace` "
                "(or __graft_entry__.build()) before using CUDA tensors"
            ) from exc
        _EXT = _C
    return _EXT


def extension_available() -> bool:
    try:
        ext()
        return True
    except RuntimeError:
        return False


ERROR_NAMES = {1: "timeout: TMA tile", 2: "timeout: shared-memory stage", 3: "timeout: TMEM full",
               4: "timeout: TMEM empty", 5: "timeout: peer flag", 6: "bad argument", 7: "timeout: attention Q",
               8: "timeout: attention K/V", 9: "timeout: attention S", 10: "timeout: attention P",
               11: "timeout: attention PV", 12: "timeout: attention O", 13: "timeout: CTA-pair exit"}
TIMEOUT_PEER_FLAG = 5


class KernelError(RuntimeError):
    """A kernel of this library gave up a bounded wait (or rejected an argument) on the device."""

    def __init__(self, code: int, where: str):
        self.code = int(code)
        super().__init__(f"libra_b200 kernel reported error code {code} ({ERROR_NAMES.get(code, 'unknown')}) "
                         f"on {where}")


def error_flag(device: torch.device) -> torch.Tensor:
    """Per-device int32[4] error word handed to every kernel: [0] receives the
    code of the first bounded wait that gave up; [1] > 0 overrides the wait
    budget (milliseconds)."""
    key = (device.type, device.index)
    flag = _ERR.get(key)
    if flag is None:
        flag = torch.zeros(4, dtype=torch.int32, device=device)
        _ERR[key] = flag
    return flag


def set_wait_limit_ms(device: torch.device, ms: int) -> None:
    """Bound every wait of the kernels launched afterwards on ``device`` by ``ms``
    milliseconds (0 restores the compiled-in default of 2 s)."""
    error_flag(device)[1].fill_(int(ms))


def check_kernel_errors(device: Optional[torch.device] = None) -> None:
    """Raise ``KernelError`` if any kernel on ``device`` reported an error (forces a sync)."""
    for (dtype, index), flag in list(_ERR.items()):
        if device is not None and (dtype, index) != (device.type, device.index):
            continue
        code = int(flag[0].item())
        if code:
            flag[0].zero_()
            raise KernelError(code, f"{dtype}:{index}")


# ---------------------------------------------------------------------------
# GEMM
# ---------------------------------------------------------------------------

def gemm(a, b, *, a_mn=False, b_mn=False, out=None, epi=EPI_BF16, residual=None):
    """C (op)= A . B^T on the tcgen05 kernel.

    ``a`` is [M, K] (``a_mn=False``) or [K, M]; ``b`` is [N, K] or [K, N].
    """
    M = a.shape[1] if a_mn else a.shape[0]
    N = b.shape[1] if b_mn else b.shape[0]
    if a.device.type != "cuda":
        A = a.float().t() if a_mn else a.float()
        B = b.float() if b_mn else b.float().t()
        res = A @ B
        if epi == EPI_BF16_RESIDUAL:
            res = res + residual.float()
        if out is None:
            return res.to(torch.float32 if epi in (EPI_F32, EPI_ACC_F32) else torch.bfloat16)
        if epi == EPI_ACC_F32:
            out.add_(res)
        else:
            out.copy_(res)
        return out
    if out is None:
        dtype = torch.float32 if epi in (EPI_F32, EPI_ACC_F32) else torch.bfloat16
        out = torch.empty(M, N, dtype=dtype, device=a.device)
    ext().gemm_bf16(a, b, out, a_mn, b_mn, epi, residual, error_flag(a.device))
    return out


def _accumulate_wgrad(weight, dy2d, x2d):
    """dW = dY^T X, accumulated into weight.main_grad when present."""
    main = getattr(weight, "main_grad", None)
    if main is not None:
        gemm(dy2d, x2d, a_mn=True, b_mn=True, out=main, epi=EPI_ACC_F32)
        return None
    return gemm(dy2d, x2d, a_mn=True, b_mn=True, epi=EPI_F32).to(weight.dtype)


class _Linear(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, weight, residual):
        x2d = x.reshape(-1, x.shape[-1])
        if not x2d.is_contiguous():
            x2d = x2d.contiguous()
        if residual is not None:
            y = gemm(x2d, weight, epi=EPI_BF16_RESIDUAL, residual=residual.reshape(-1, weight.shape[0]))
        else:
            y = gemm(x2d, weight)
        ctx.save_for_backward(x2d, weight)
        ctx.has_residual = residual is not None
        ctx.in_shape = x.shape
        return y.view(*x.shape[:-1], weight.shape[0])

    @staticmethod
    def backward(ctx, dy):
        x2d, weight = ctx.saved_tensors
        dy2d = dy.reshape(-1, weight.shape[0])
        if not dy2d.is_contiguous():
            dy2d = dy2d.contiguous()
        dx = None
        if ctx.needs_input_grad[0]:
            dx = gemm(dy2d, weight, b_mn=True).view(ctx.in_shape)
        dw = _accumulate_wgrad(weight, dy2d, x2d) if ctx.needs_input_grad[1] else None
        dres = dy if ctx.has_residual else None
        return dx, dw, dres


def linear(x, weight, residual=None):
    """y = x W^T (+ residual), bf16 in/out, fp32 accumulation in TMEM."""
    if x.device.type != "cuda":
        y = torch.nn.functional.linear(x.float(), weight.float())
        if residual is not None:
            y = y + residual.float()
        return y.to(x.dtype)
    return _Linear.apply(x, weight, residual)


# ---------------------------------------------------------------------------
# RMSNorm
# ---------------------------------------------------------------------------

def _grad_sink(weight, grad_fp32):
    main = getattr(weight, "main_grad", None)
    if main is not None:
        main.add_(grad_fp32.view_as(main))
        return None
    return grad_fp32.to(weight.dtype)


class _RMSNorm(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, w, eps):
        x2d = x.reshape(-1, x.shape[-1]).contiguous()
        y, rstd = ext().rmsnorm_fwd(x2d, w, eps)
        ctx.save_for_backward(x2d, w, rstd)
        ctx.shape = x.shape
        return y.view(x.shape)

    @staticmethod
    def backward(ctx, dy):
        x2d, w, rstd = ctx.saved_tensors
        main = getattr(w, "main_grad", None)
        dw = main if main is not None else torch.zeros(w.shape, dtype=torch.float32, device=w.device)
        dx = ext().rmsnorm_bwd(dy.reshape(x2d.shape).contiguous(), x2d, w, rstd, dw, main is not None, None)
        return dx.view(ctx.shape), (None if main is not None else dw.to(w.dtype)), None


def rmsnorm(x, w, eps: float = 1e-6):
    if x.device.type != "cuda":
        return ref.rmsnorm(x, w, eps)
    return _RMSNorm.apply(x, w, eps)


# ---------------------------------------------------------------------------
# q/k RMSNorm + RoPE
# ---------------------------------------------------------------------------

class _QKNormRope(torch.autograd.Function):
    @staticmethod
    def forward(ctx, qkv, qw, kw, pos, cos, sin, nq, nkv, eps):
        q, k, v, rstd = ext().qk_norm_rope_fwd(qkv, qw, kw, pos, cos, sin, nq, nkv, eps)
        ctx.save_for_backward(qkv, qw, kw, pos, cos, sin, rstd)
        ctx.nq, ctx.nkv = nq, nkv
        return q, k, v

    @staticmethod
    def backward(ctx, dq, dk, dv):
        qkv, qw, kw, pos, cos, sin, rstd = ctx.saved_tensors
        mq, mk = getattr(qw, "main_grad", None), getattr(kw, "main_grad", None)
        gq = mq if mq is not None else torch.zeros(qw.shape, dtype=torch.float32, device=qw.device)
        gk = mk if mk is not None else torch.zeros(kw.shape, dtype=torch.float32, device=kw.device)
        dqkv = ext().qk_norm_rope_bwd(qkv, qw, kw, pos, cos, sin, rstd, dq.contiguous(), dk.contiguous(),
                                      dv.contiguous(), gq, gk, ctx.nq, ctx.nkv)
        return (dqkv, None if mq is not None else gq.to(qw.dtype), None if mk is not None else gk.to(kw.dtype),
                None, None, None, None, None, None)


def qk_norm_rope(qkv, qw, kw, pos, cos, sin, nq: int, nkv: int, eps: float = 1e-6):
    """Split the fused QKV output into q [T,nq,D], k, v [T,nkv,D] with per-head
    RMSNorm on q/k followed by rotary embedding at positions ``pos``."""
    if qkv.device.type != "cuda":
        return ref.qk_norm_rope(qkv, qw, kw, pos, cos, sin, nq, nkv, eps)
    return _QKNormRope.apply(qkv, qw, kw, pos, cos, sin, nq, nkv, eps)


# ---------------------------------------------------------------------------
# SwiGLU
# ---------------------------------------------------------------------------

class _SwiGLU(torch.autograd.Function):
    @staticmethod
    def forward(ctx, gu):
        ctx.save_for_backward(gu)
        return ext().swiglu_fwd(gu)

    @staticmethod
    def backward(ctx, dh):
        (gu,) = ctx.saved_tensors
        return ext().swiglu_bwd(gu, dh.contiguous())


def swiglu(gu):
    if gu.device.type != "cuda":
        return ref.swiglu(gu)
    return _SwiGLU.apply(gu.contiguous())


class _LinearSwiGLU(torch.autograd.Function):
    """a = silu(x Wg^T) * (x Wu^T) for W = [Wg; Wu] in one tcgen05 GEMM whose
    epilogue applies SwiGLU; the pre-activation gate/up outputs are kept only
    when a backward pass will need them."""

    @staticmethod
    def forward(ctx, x, weight):
        x2d = x.reshape(-1, x.shape[-1])
        if not x2d.is_contiguous():
            x2d = x2d.contiguous()
        M, F = x2d.shape[0], weight.shape[0] // 2
        a = torch.empty(M, F, dtype=x.dtype, device=x.device)
        need_grad = ctx.needs_input_grad[0] or ctx.needs_input_grad[1]
        gu = torch.empty(M, 2 * F, dtype=x.dtype, device=x.device) if need_grad else None
        ext().gemm_swiglu(x2d, weight, a, gu, error_flag(x.device))
        ctx.save_for_backward(x2d, weight, gu)
        ctx.in_shape = x.shape
        return a.view(*x.shape[:-1], F)

    @staticmethod
    def backward(ctx, da):
        x2d, weight, gu = ctx.saved_tensors
        dgu = ext().swiglu_bwd(gu, da.reshape(gu.shape[0], -1).contiguous())
        dx = gemm(dgu, weight, b_mn=True).view(ctx.in_shape) if ctx.needs_input_grad[0] else None
        dw = _accumulate_wgrad(weight, dgu, x2d) if ctx.needs_input_grad[1] else None
        return dx, dw


def linear_swiglu(x, weight):
    """SwiGLU MLP input half: silu(x W_gate^T) * (x W_up^T), W = [W_gate; W_up] ([2F, H])."""
    F2 = weight.shape[0]
    if x.device.type != "cuda" or F2 % 256 != 0:
        return swiglu(linear(x, weight))
    return _LinearSwiGLU.apply(x, weight)


# ---------------------------------------------------------------------------
# grouped (per-expert) linear layers over padded row groups
# ---------------------------------------------------------------------------

EPI_SWIGLU = 4


def _grouped_wgrad(w, dy, x, offs):
    """dW_g (+)= dy[rows of g]^T x[rows of g]; into w.main_grad when present."""
    main = getattr(w, "main_grad", None)
    if main is not None:
        ext().grouped_gemm_wgrad(dy, x, main.view(w.shape), offs, True, error_flag(x.device))
        return None
    out = torch.zeros(w.shape, dtype=torch.float32, device=w.device)
    ext().grouped_gemm_wgrad(dy, x, out, offs, True, error_flag(x.device))
    return out.to(w.dtype)


class _GroupedLinear(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, w, offs, out):
        if out is not None:
            # caller-provided memory (e.g. a peer-visible send slot): alias its storage without making the
            # result an autograd view of that buffer
            y = torch.empty(0, dtype=out.dtype, device=out.device).set_(out.untyped_storage(), out.storage_offset(),
                                                                          out.shape, out.stride())
        else:
            y = torch.zeros(x.shape[0], w.shape[1], dtype=x.dtype, device=x.device)
        ext().grouped_gemm(x, w, y, offs, 0, False, EPI_BF16, None, error_flag(x.device))
        ctx.save_for_backward(x, w, offs)
        return y

    @staticmethod
    def backward(ctx, dy):
        x, w, offs = ctx.saved_tensors
        dy = dy.contiguous()
        dx = None
        if ctx.needs_input_grad[0]:
            dx = torch.zeros_like(x)
            ext().grouped_gemm(dy, w, dx, offs, 0, True, EPI_BF16, None, error_flag(x.device))
        dw = _grouped_wgrad(w, dy, x, offs) if ctx.needs_input_grad[1] else None
        return dx, dw, None, None


class _GroupedSwiGLU(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, w, offs):
        T, F = x.shape[0], w.shape[1] // 2
        a = torch.zeros(T, F, dtype=x.dtype, device=x.device)
        need = ctx.needs_input_grad[0] or ctx.needs_input_grad[1]
        gu = torch.zeros(T, 2 * F, dtype=x.dtype, device=x.device) if need else None
        ext().grouped_gemm(x, w, a, offs, 0, False, EPI_SWIGLU, gu, error_flag(x.device))
        ctx.save_for_backward(x, w, offs, gu)
        return a

    @staticmethod
    def backward(ctx, da):
        x, w, offs, gu = ctx.saved_tensors
        dgu = ext().swiglu_bwd(gu, da.contiguous())
        dx = None
        if ctx.needs_input_grad[0]:
            dx = torch.zeros_like(x)
            ext().grouped_gemm(dgu, w, dx, offs, 0, True, EPI_BF16, None, error_flag(x.device))
        dw = _grouped_wgrad(w, dgu, x, offs) if ctx.needs_input_grad[1] else None
        return dx, dw, None


def _grouped_ref(x, w, offs):
    y = torch.zeros(x.shape[0], w.shape[1], dtype=torch.float32, device=x.device)
    o = offs.tolist()
    for g in range(w.shape[0]):
        if o[g + 1] > o[g]:
            y[o[g]:o[g + 1]] = x[o[g]:o[g + 1]].float() @ w[g].float().t()
    return y


def grouped_linear(x, w, offs, out=None):
    """y[rows of g] = x[rows of g] w[g]^T for the row groups ``offs`` (int32 [G+1] on the device,
    starts multiples of 128, padding rows zero); w [G, N, K].  One launch for every group."""
    if x.device.type != "cuda":
        y = _grouped_ref(x, w, offs).to(x.dtype)
        if out is not None:
            out.copy_(y.detach())
        return y
    return _GroupedLinear.apply(x, w, offs, out)


def grouped_swiglu(x, w, offs):
    """silu(x W_gate,g^T) * (x W_up,g^T) per row group, w [G, 2F, K] ([gate; up] per group)."""
    if x.device.type != "cuda":
        gu = _grouped_ref(x, w, offs)
        F = w.shape[1] // 2
        return (torch.nn.functional.silu(gu[:, :F]) * gu[:, F:]).to(x.dtype)
    return _GroupedSwiGLU.apply(x, w, offs)


# ---------------------------------------------------------------------------
# attention
# ---------------------------------------------------------------------------

def varlen_causal_attention(q, k, v, cu_seqlens, max_seqlen: int, scale=None, tiles=None):
    """Causal GQA attention over packed sequences (q [T,Hq,D], k/v [T,Hkv,D]).

    ``tiles``: the (q tiles, kv tiles) tables of the packed batch, built once
    per batch (``attention.attn_tiles``); computed from ``cu_seqlens`` when absent."""
    if q.device.type != "cuda":
        return ref.varlen_causal_attention(q, k, v, cu_seqlens, scale)
    from .attention import flash_varlen_causal

    qt, kvt = tiles if isinstance(tiles, (tuple, list)) else (tiles, None)
    return flash_varlen_causal(q, k, v, cu_seqlens, max_seqlen, scale, qt, kvt)


# ---------------------------------------------------------------------------
# LM head + token logprob
# ---------------------------------------------------------------------------

LOGPROB_CHUNK_ROWS = int(os.environ.get("LIBRA_LOGPROB_CHUNK_ROWS", "8192"))


class _LMHeadLogprob(torch.autograd.Function):
    """logp[r] = log_softmax(h[r] W^T / T)[target[r]] without an fp32 logits tensor.

    Logits are produced chunk by chunk by the tcgen05 GEMM in bf16, reduced by
    the fused logprob kernel and (when a backward is needed) kept in bf16 so the
    backward rewrites them in place as dlogits and feeds the dgrad/wgrad GEMMs.
    """

    @staticmethod
    def forward(ctx, h, w, targets, temperature, entropy_out):
        C = ext()
        R = h.shape[0]
        logp = torch.empty(R, dtype=torch.float32, device=h.device)
        lse = torch.empty(R, dtype=torch.float32, device=h.device)
        keep = []
        need_grad = ctx.needs_input_grad[0] or ctx.needs_input_grad[1]
        for s in range(0, R, LOGPROB_CHUNK_ROWS):
            e = min(R, s + LOGPROB_CHUNK_ROWS)
            logits = gemm(h[s:e], w)
            lp, ent, stats, _ = C.logprob_fwd(logits, targets[s:e], 0, temperature, entropy_out is not None)
            logp[s:e] = lp
            lse[s:e] = stats[:, 0] + stats[:, 1].log()
            if entropy_out is not None:
                entropy_out[s:e] = ent
            if need_grad:
                keep.append(logits)
        ctx.save_for_backward(h, w, targets, lse)
        ctx.logits = keep
        ctx.temperature = temperature
        return logp

    @staticmethod
    def backward(ctx, g):
        h, w, targets, lse = ctx.saved_tensors
        C = ext()
        g = g.contiguous().float()
        dh = torch.empty_like(h) if ctx.needs_input_grad[0] else None
        main = getattr(w, "main_grad", None)
        dw_local = None
        if ctx.needs_input_grad[1] and main is None:
            dw_local = torch.zeros(w.shape, dtype=torch.float32, device=w.device)
        R = h.shape[0]
        for idx, s in enumerate(range(0, R, LOGPROB_CHUNK_ROWS)):
            e = min(R, s + LOGPROB_CHUNK_ROWS)
            logits = ctx.logits[idx]
            C.logprob_bwd_(logits, targets[s:e], 0, ctx.temperature, lse[s:e], g[s:e])
            if dh is not None:
                gemm(logits, w, b_mn=True, out=dh[s:e])
            if ctx.needs_input_grad[1]:
                gemm(logits, h[s:e], a_mn=True, b_mn=True, out=main if main is not None else dw_local,
                     epi=EPI_ACC_F32)
            ctx.logits[idx] = None
        ctx.logits = []
        dw = None if dw_local is None else dw_local.to(w.dtype)
        return dh, dw, None, None, None


def lm_head_logprob(h, w, targets, temperature: float = 1.0, entropy_out=None):
    """Token logprobs of ``targets`` under the LM head ``w`` for hidden rows ``h``."""
    if h.device.type != "cuda":
        logits = torch.nn.functional.linear(h.float(), w.float())
        lp, ent = ref.token_logprobs(logits, targets, temperature)
        if entropy_out is not None:
            entropy_out.copy_(ent.detach())
        return lp
    h = h.contiguous()
    return _LMHeadLogprob.apply(h, w, targets.contiguous(), float(temperature), entropy_out)


# ---------------------------------------------------------------------------
# rollout: paged decode attention and sampling
# ---------------------------------------------------------------------------

def paged_decode(q, k_cache, v_cache, block_tables, seq_lens, out, part_out, part_ml, split_len: int,
                 scale: float):
    """Decode attention of one new token per sequence over the paged cache.

    ``out`` [B, Hq, D] and the split workspace ``part_out`` [>=B, Hq, S, D] /
    ``part_ml`` [>=B, Hq, S, 2] (fp32) are the caller's; ``S * split_len``
    must cover the longest sequence.  Nothing is allocated, so the call can sit
    inside a captured CUDA graph."""
    if q.device.type != "cuda":
        B, Hq, D = q.shape
        Hkv, bs = k_cache.shape[2], k_cache.shape[1]
        for b in range(B):
            L = int(seq_lens[b])
            idx = torch.arange(L)
            blocks = block_tables[b, idx // bs].long()
            k = k_cache[blocks, idx % bs].float()          # [L, Hkv, D]
            v = v_cache[blocks, idx % bs].float()
            kk = k.repeat_interleave(Hq // Hkv, 1)           # [L, Hq, D]
            vv = v.repeat_interleave(Hq // Hkv, 1)
            s = torch.einsum("hd,lhd->hl", q[b].float(), kk) * scale
            out[b] = torch.einsum("hl,lhd->hd", s.softmax(-1), vv).to(out.dtype)
        return out
    ext().paged_decode_v2(q, k_cache, v_cache, block_tables, seq_lens, out, part_out, part_ml, int(split_len),
                          float(scale))
    return out


def sample_tokens(logits, temperature, seeds, positions, out_tok, out_lp, next_tok=None, pdl: bool = False):
    """Temperature sampling (Gumbel-max over a Philox stream keyed by the
    request seed and counted by position) with the sampled token's logprob.
    ``temperature <= 0`` is greedy.  Writes ``out_tok`` (int64) / ``out_lp``."""
    if logits.device.type != "cuda":
        B = logits.shape[0]
        for b in range(B):
            t = float(temperature[b])
            x = logits[b].float() / (t if t > 0 else 1.0)
            if t > 0:
                g = torch.Generator().manual_seed((int(seeds[b]) * 1000003 + int(positions[b])) & 0x7FFFFFFF)
                tok = int(torch.multinomial(x.softmax(-1), 1, generator=g))
            else:
                tok = int(x.argmax())
            out_tok[b] = tok
            out_lp[b] = x.log_softmax(-1)[tok]
            if next_tok is not None:
                next_tok[b] = tok
        return out_tok, out_lp
    ext().sample_tokens(logits, temperature, seeds, positions, out_tok, out_lp, next_tok, pdl)
    return out_tok, out_lp


def filtered_keep_mask(x: torch.Tensor, top_p: float, top_k: int) -> torch.Tensor:
    """Tokens kept by top-k and top-p on one row of scaled logits ``x`` (fp32):
    the k largest values and the nucleus (a token stays while the probability
    mass strictly above it is at most ``top_p``); values tied with a threshold
    are all kept.  The rule of ``sample_tokens_filtered``."""
    V = x.numel()
    thr = torch.tensor(float("-inf"))
    if 0 < top_k < V:
        thr = torch.maximum(thr, x.topk(top_k).values[-1])
    if top_p < 1.0:
        p = torch.softmax(x, -1)
        sx, order = torch.sort(x, descending=True)
        ps = p[order]
        above = torch.cumsum(ps, 0) - ps
        # ties share the mass above their first occurrence
        first = torch.searchsorted(-sx, -sx, side="left")
        ok = above[first] <= top_p
        thr = torch.maximum(thr, sx[ok].min())
    return x >= thr


def sample_tokens_filtered(logits, temperature, top_p, top_k, seeds, positions, out_tok, out_lp):
    """Temperature sampling restricted to the top-k tokens and the top-p
    nucleus (thresholds by radix select on the device, then Gumbel-max over the
    kept tokens on the Philox stream of ``sample_tokens``), with the token's
    logprob under the unfiltered temperature-scaled distribution.
    ``temperature <= 0`` is greedy; ``top_k <= 0`` and ``top_p >= 1`` disable
    the filters.  Writes ``out_tok`` (int64) / ``out_lp`` (fp32)."""
    if logits.device.type != "cuda":
        for b in range(logits.shape[0]):
            t = float(temperature[b])
            x = logits[b].float() / (t if t > 0 else 1.0)
            if t > 0:
                keep = filtered_keep_mask(x, float(top_p[b]), int(top_k[b]))
                g = torch.Generator().manual_seed((int(seeds[b]) * 1000003 + int(positions[b])) & 0x7FFFFFFF)
                tok = int(torch.multinomial(torch.softmax(x.masked_fill(~keep, float("-inf")), -1), 1, generator=g))
            else:
                tok = int(x.argmax())
            out_tok[b] = tok
            out_lp[b] = x.log_softmax(-1)[tok]
        return out_tok, out_lp
    ext().sample_tokens_filtered(logits, temperature, top_p, top_k, seeds, positions, out_tok, out_lp)
    return out_tok, out_lp


def gemm_streamk(a, w, acc):
    """``acc += a . w^T`` with the stream-K mode of the tcgen05 GEMM: every SM
    takes an equal share of the tiles x K-blocks iterations, so a skinny GEMM
    (a decode step's few rows) streams the weight on all SMs.  ``acc`` is fp32
    [M, N]; the fused decode consumers read it and leave it zeroed."""
    if a.device.type != "cuda":
        acc.add_(a.float() @ w.float().t())
        return acc
    ext().gemm_bf16(a, w, acc, False, False, EPI_ACC_F32, None, error_flag(a.device), True)
    return acc


def gemm_decode(x, w, acc, pdl: bool = False):
    """``acc += x . w^T`` for a decode batch (``x`` [M <= 256, K]): the weight
    is the 128-row operand of the tcgen05 MMA and the batch its N, stream-K
    over all SMs, coalesced fp32 reductions into ``acc`` [M, N].  ``pdl``:
    programmatic dependent launch (the first weight tiles load while the
    previous kernel on the stream finishes)."""
    if x.device.type != "cuda":
        acc.add_(x.float() @ w.float().t())
        return acc
    ext().gemm_decode(x, w, acc, error_flag(x.device), pdl)
    return acc


def _take(acc, rows=None):
    v = (acc if rows is None else acc[:rows]).clone()
    (acc if rows is None else acc[:rows]).zero_()
    return v


def decode_qkv_post(acc, qw, kw, pos, cos, sin, slot, q_out, k_cache, v_cache, eps: float, pdl: bool = False):
    """Fused decode step after the QKV GEMM: round the fp32 accumulator to bf16,
    per-head RMSNorm of q and k, RoPE at ``pos``, q -> ``q_out`` [B, nq, D],
    k and v of the new token straight into cache row ``slot``; zeroes the
    accumulator rows it read."""
    if acc.device.type != "cuda":
        B, nq, D = q_out.shape
        nkv = k_cache.shape[2]
        x = _take(acc, B).to(torch.bfloat16)
        q, k, v = ref.qk_norm_rope(x, qw, kw, pos[:B], cos, sin, nq, nkv, eps)
        q_out.copy_(q)
        k_cache.view(-1, nkv, D)[slot[:B]] = k.to(k_cache.dtype)
        v_cache.view(-1, nkv, D)[slot[:B]] = v.to(v_cache.dtype)
        return q_out
    ext().decode_qkv_post(acc, qw, kw, pos, cos, sin, slot, q_out, k_cache, v_cache, float(eps), pdl)
    return q_out


def decode_residual_norm(x, acc, w, h_out, eps: float, pdl: bool = False):
    """``x = bf16(x + acc)`` in place, ``h_out = RMSNorm(x) * w``; zeroes ``acc[:B]``."""
    if x.device.type != "cuda":
        x.copy_((x.float() + _take(acc, x.shape[0])).to(x.dtype))
        h_out.copy_(ref.rmsnorm(x, w, eps))
        return h_out
    ext().decode_residual_norm(x, acc, w, h_out, float(eps), pdl)
    return h_out


def decode_swiglu(acc, a, pdl: bool = False):
    """``a = silu(bf16(gate)) * bf16(up)`` from the gate/up accumulator [B, 2F]; zeroes it."""
    if a.device.type != "cuda":
        B, F = a.shape
        gu = _take(acc, B).to(torch.bfloat16).float()
        a.copy_((torch.nn.functional.silu(gu[:, :F]) * gu[:, F:]).to(a.dtype))
        return a
    ext().decode_swiglu(acc, a, pdl)
    return a


def decode_attention(q, k_cache, v_cache, block_tables, seq_lens, out, part_o, part_ml, counters, scale: float,
                     pdl: bool = False):
    """Paged decode attention for rows ``0..out.shape[0]-1``: stream-K over the
    sequences' KV blocks (one CTA per SM, every CTA the same share), partial
    results merged in the kernel.  Workspace ``part_o`` [SMs + B, Hq, D] /
    ``part_ml`` [SMs + B, Hq, 2] fp32 and ``counters`` [B] int32 (zero before
    the first call; the kernel leaves them zero) are the caller's, so the call
    allocates nothing and can be captured."""
    if q.device.type != "cuda":
        B = out.shape[0]
        return paged_decode(q[:B], k_cache, v_cache, block_tables, seq_lens, out, None, None, 0, scale)
    ext().decode_attention(q, k_cache, v_cache, block_tables, seq_lens, out, part_o, part_ml, counters,
                           error_flag(q.device), float(scale), pdl)
    return out


def decode_workspace(max_batch: int, num_heads: int, head_dim: int, device):
    """Workspace of ``decode_attention`` for up to ``max_batch`` rows."""
    sms = torch.cuda.get_device_properties(device).multi_processor_count if device.type == "cuda" else 1
    slots = sms + max_batch
    return (torch.zeros(slots, num_heads, head_dim, dtype=torch.float32, device=device),
            torch.zeros(slots, num_heads, 2, dtype=torch.float32, device=device),
            torch.zeros(max_batch, dtype=torch.int32, device=device))


# ---------------------------------------------------------------------------
# optimizer
# ---------------------------------------------------------------------------

def adamw_step(master, grad, exp_avg, exp_avg_sq, param_bf16, *, lr, beta1, beta2, eps, weight_decay, step,
               max_grad_norm=0.0, sq_norm=None, grad_scale=1.0):
    """One AdamW update over flat fp32 buffers, writing the bf16 copy too."""
    if master.device.type != "cuda":
        # fp32 math whatever the moment dtype (bf16 moments are rounded once, on the store)
        g = grad.float() * grad_scale
        if max_grad_norm > 0:
            total = g.norm() if sq_norm is None else sq_norm.float().sqrt() * grad_scale
            g = g * torch.clamp(max_grad_norm / (total + 1e-6), max=1.0)
        m = exp_avg.float().mul_(beta1).add_(g, alpha=1 - beta1)
        v = exp_avg_sq.float().mul_(beta2).addcmul_(g, g, value=1 - beta2)
        bc1, bc2 = 1 - beta1 ** step, 1 - beta2 ** step
        master.sub_(lr * ((m / bc1) / ((v / bc2).sqrt() + eps) + weight_decay * master))
        exp_avg.copy_(m)
        exp_avg_sq.copy_(v)
        param_bf16.copy_(master)
        return
    ext().adamw_step(master, grad, exp_avg, exp_avg_sq, param_bf16, lr, beta1, beta2, eps, weight_decay, step,
                     sq_norm, max_grad_norm, grad_scale)


def grad_sq_norm(grad, out):
    """out += sum(grad^2) (device scalar)."""
    if grad.device.type != "cuda":
        out.add_(grad.float().pow(2).sum())
        return out
    ext().grad_sq_norm(grad, out)
    return out


__all__ = [
    "ext", "extension_available", "check_kernel_errors", "gemm", "linear", "rmsnorm", "qk_norm_rope", "swiglu",
    "varlen_causal_attention", "lm_head_logprob", "adamw_step", "grad_sq_norm", "ref", "linear_swiglu",
    "paged_decode", "sample_tokens", "grouped_linear", "grouped_swiglu",
]
