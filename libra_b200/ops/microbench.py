"""Kernel microbenchmarks: achieved TFLOP/s or GB/s of each sm_100a kernel.

    python -m libra_b200.ops.microbench gemm [--shapes M,N,K;...] [--iters 20]
    python -m libra_b200.ops.microbench decode [--batch 64] [--lens 510x64]
    python -m libra_b200.ops.microbench peer1 [--case gemm_ar|gemm_rs|ag_gemm|grad_rs|adamw_ag|tp_ar_norm]
    python -m libra_b200.ops.microbench all

Timing: CUDA events on the launching stream after warm-up, synchronize on both
sides, inputs larger than L2 for the bandwidth-bound kernels.  The GEMM rows
also time torch.matmul (cuBLAS) on the same operands for comparison.  Prints one
JSON object per line.
"""

from __future__ import annotations

import argparse
import json

import torch

from libra_b200 import ops

# Qwen3-4B training shapes for a 16k-token chunk: (M tokens, N out, K in)
QWEN3_4B_SHAPES = [
    ("qkv_fwd", 16384, 6144, 2560, False, False),
    ("o_fwd", 16384, 2560, 4096, False, False),
    ("gate_up_fwd", 16384, 19456, 2560, False, False),
    ("down_fwd", 16384, 2560, 9728, False, False),
    ("gate_up_dgrad", 16384, 2560, 19456, False, True),
    ("gate_up_wgrad", 19456, 2560, 16384, True, True),
    ("lm_head_fwd", 8192, 151936, 2560, False, False),
    ("square_8192", 8192, 8192, 8192, False, False),
]


def _time(fn, iters: int, warmup: int = 3) -> float:
    for _ in range(warmup):
        fn()
    torch.cuda.synchronize()
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    start.record()
    for _ in range(iters):
        fn()
    end.record()
    torch.cuda.synchronize()
    return start.elapsed_time(end) / iters


def bench_gemm(shapes, iters: int):
    for name, M, N, K, a_mn, b_mn in shapes:
        A = torch.randn(M, K, device="cuda").to(torch.bfloat16)
        B = torch.randn(N, K, device="cuda").to(torch.bfloat16)
        a = A.t().contiguous() if a_mn else A
        b = B.t().contiguous() if b_mn else B
        out = torch.empty(M, N, device="cuda", dtype=torch.bfloat16)
        ms = _time(lambda: ops.gemm(a, b, a_mn=a_mn, b_mn=b_mn, out=out), iters)
        ref_a = a.t() if a_mn else a
        ref_b = b if b_mn else b.t()
        ms_ref = _time(lambda: torch.matmul(ref_a, ref_b, out=out), iters)
        flops = 2.0 * M * N * K
        ops.check_kernel_errors()
        print(json.dumps({"kernel": "gemm_bf16_tcgen05", "case": name, "M": M, "N": N, "K": K, "a_mn": a_mn,
                          "b_mn": b_mn, "ms": ms, "tflops": flops / ms / 1e9, "cublas_ms": ms_ref,
                          "cublas_tflops": flops / ms_ref / 1e9, "ratio_vs_cublas": ms_ref / ms}), flush=True)
        del A, B, a, b, out


def bench_swiglu(iters: int, M: int = 16384, H: int = 2560, F: int = 9728):
    """Gate/up GEMM with the SwiGLU epilogue (with and without the kept gate/up
    output) against the plain GEMM of the same shape, and the SwiGLU backward."""
    err = ops.error_flag(torch.device("cuda"))
    x = torch.randn(M, H, device="cuda").to(torch.bfloat16)
    wgu = (torch.randn(2 * F, H, device="cuda") / H ** 0.5).to(torch.bfloat16)
    a = torch.empty(M, F, device="cuda", dtype=torch.bfloat16)
    gu = torch.empty(M, 2 * F, device="cuda", dtype=torch.bfloat16)
    ms_gu = _time(lambda: ops.ext().gemm_swiglu(x, wgu, a, gu, err), iters)
    ms_nogu = _time(lambda: ops.ext().gemm_swiglu(x, wgu, a, None, err), iters)
    ms_plain = _time(lambda: ops.gemm(x, wgu, out=gu), iters)
    ms_bwd = _time(lambda: ops.ext().swiglu_bwd(gu, a), iters)
    ops.check_kernel_errors()
    flops = 2.0 * M * H * 2 * F
    print(json.dumps({"kernel": "gemm_swiglu", "M": M, "H": H, "F": F, "with_gu_ms": ms_gu, "without_gu_ms": ms_nogu,
                      "plain_gemm_ms": ms_plain, "tflops_with_gu": flops / ms_gu / 1e9,
                      "tflops_plain": flops / ms_plain / 1e9, "swiglu_bwd_ms": ms_bwd,
                      "swiglu_bwd_gbs": 5 * M * F * 2 / ms_bwd / 1e6}), flush=True)


def bench_elementwise(iters: int):
    T, H = 65536, 2560
    x = torch.randn(T, H, device="cuda").to(torch.bfloat16)
    w = torch.ones(H, device="cuda", dtype=torch.bfloat16)
    ms = _time(lambda: ops.ext().rmsnorm_fwd(x, w, 1e-6), iters)
    print(json.dumps({"kernel": "rmsnorm_fwd", "T": T, "H": H, "ms": ms, "gbs": 2 * 2 * T * H / ms / 1e6}), flush=True)
    T2 = 16384
    xb, dy = x[:T2].contiguous(), torch.randn(T2, H, device="cuda").to(torch.bfloat16)
    rstd = torch.rsqrt(xb.float().pow(2).mean(-1) + 1e-6).contiguous()
    dw = torch.zeros(H, device="cuda")
    ms = _time(lambda: ops.ext().rmsnorm_bwd(dy, xb, w, rstd, dw, False, None), iters)
    print(json.dumps({"kernel": "rmsnorm_bwd+colsum", "T": T2, "H": H, "ms": ms,
                      "gbs": 3 * 2 * T2 * H / ms / 1e6}), flush=True)
    nq, nkv, D = 32, 8, 128
    qkv = torch.randn(T2, (nq + 2 * nkv) * D, device="cuda").to(torch.bfloat16)
    qw = torch.ones(D, device="cuda", dtype=torch.bfloat16)
    pos = torch.arange(T2, device="cuda", dtype=torch.int32) % 4096
    from libra_b200.ops import reference as _ref
    cos, sin = [t.float().cuda().contiguous() for t in _ref.rope_tables(4096, D, 1e6)]
    q, k, v, r = ops.ext().qk_norm_rope_fwd(qkv, qw, qw, pos, cos, sin, nq, nkv, 1e-6)
    ms = _time(lambda: ops.ext().qk_norm_rope_fwd(qkv, qw, qw, pos, cos, sin, nq, nkv, 1e-6), iters)
    print(json.dumps({"kernel": "qk_norm_rope_fwd", "T": T2, "ms": ms,
                      "gbs": 2 * 2 * T2 * (nq + 2 * nkv) * D / ms / 1e6}), flush=True)
    dqw, dkw = torch.zeros(D, device="cuda"), torch.zeros(D, device="cuda")
    ms = _time(lambda: ops.ext().qk_norm_rope_bwd(qkv, qw, qw, pos, cos, sin, r, q, k, v, dqw, dkw, nq, nkv), iters)
    print(json.dumps({"kernel": "qk_norm_rope_bwd", "T": T2, "ms": ms,
                      "gbs": 3 * 2 * T2 * (nq + 2 * nkv) * D / ms / 1e6}), flush=True)
    F = 9728
    gu = torch.randn(T // 2, 2 * F, device="cuda").to(torch.bfloat16)
    ms = _time(lambda: ops.ext().swiglu_fwd(gu), iters)
    print(json.dumps({"kernel": "swiglu_fwd", "T": T // 2, "F": F, "ms": ms,
                      "gbs": (T // 2) * 3 * F * 2 / ms / 1e6}), flush=True)
    R, V = 4096, 151936
    logits = torch.randn(R, V, device="cuda").to(torch.bfloat16)
    tgt = torch.randint(0, V, (R,), device="cuda")
    ms = _time(lambda: ops.ext().logprob_fwd(logits, tgt, 0, 1.0, True), iters)
    print(json.dumps({"kernel": "logprob_fwd", "R": R, "V": V, "ms": ms, "gbs": R * V * 2 / ms / 1e6}), flush=True)
    n = 1 << 28
    master = torch.randn(n, device="cuda")
    grad = torch.randn(n, device="cuda")
    m, v = torch.zeros_like(master), torch.zeros_like(master)
    p = master.to(torch.bfloat16)
    ms = _time(lambda: ops.adamw_step(master, grad, m, v, p, lr=1e-6, beta1=0.9, beta2=0.95, eps=1e-8,
                                      weight_decay=0.01, step=1), iters)
    print(json.dumps({"kernel": "adamw", "n": n, "ms": ms, "gbs": n * 30 / ms / 1e6}), flush=True)


def bench_attention(iters: int, lens=None):
    import math

    from libra_b200.ops.attention import attn_tiles

    cases = [lens] if lens else [[4096] * 4, [2048] * 8, [1024] * 16]
    for ls in cases:
        T, hq, hkv, d = sum(ls), 32, 8, 128
        cu = torch.tensor([0] + list(torch.tensor(ls).cumsum(0).tolist()), dtype=torch.int32, device="cuda")
        q = torch.randn(T, hq, d, device="cuda").bfloat16()
        k = torch.randn(T, hkv, d, device="cuda").bfloat16()
        v = torch.randn(T, hkv, d, device="cuda").bfloat16()
        do = torch.randn(T, hq, d, device="cuda").bfloat16()
        qt, kvt = attn_tiles(cu.tolist(), True, "cuda"), attn_tiles(cu.tolist(), True, "cuda", kv=True)
        err = ops.error_flag(q.device)
        sc = 1 / math.sqrt(d)
        o, lse = ops.ext().flash_fwd(q, k, v, cu, qt, sc, True, err)
        fwd_flops = sum(4 * L * L / 2 * d * hq for L in ls)
        ms_f = _time(lambda: ops.ext().flash_fwd(q, k, v, cu, qt, sc, True, err), iters)
        ms_b = _time(lambda: ops.ext().flash_bwd(do, q, k, v, o, lse, cu, qt, kvt, sc, True, err), iters)
        print(json.dumps({"kernel": "flash_attn_tcgen05", "lens": f"{ls[0]}x{len(ls)}", "fwd_ms": ms_f,
                          "fwd_tflops": fwd_flops / ms_f / 1e9, "bwd_ms": ms_b,
                          "bwd_tflops_2.5x": 2.5 * fwd_flops / ms_b / 1e9}), flush=True)
        ops.check_kernel_errors()


# Qwen3-4B decode-step GEMMs: (name, N out, K in); M is the decode batch
QWEN3_4B_DECODE = [("qkv", 6144, 2560), ("o", 2560, 4096), ("gate_up", 19456, 2560), ("down", 2560, 9728),
                   ("lm_head", 151936, 2560)]


def _time_graph(fn, calls: int, replays: int = 5) -> float:
    """Device time per call of ``fn`` captured ``calls`` times in one CUDA graph
    (no host launch cost between the calls)."""
    fn()
    torch.cuda.synchronize()
    g = torch.cuda.CUDAGraph()
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        with torch.cuda.graph(g, stream=s):
            for _ in range(calls):
                fn()
    torch.cuda.current_stream().wait_stream(s)
    g.replay()
    torch.cuda.synchronize()
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    start.record()
    for _ in range(replays):
        g.replay()
    end.record()
    torch.cuda.synchronize()
    return start.elapsed_time(end) / (replays * calls)


def bench_decode(iters: int, batch: int = 64, lens=None):
    """Decode-step kernels, each call captured in a CUDA graph so the device
    time is measured without host launch gaps: the decode GEMM (weight GB/s;
    several weight copies rotate so every call reads HBM, not L2; with and
    without programmatic dependent launch) against torch.matmul on the same
    skinny shape, and the stream-K paged attention (KV GB/s)."""
    M = batch
    for name, N, K in QWEN3_4B_DECODE:
        copies = max(2, -(-400 * 2 ** 20 // (N * K * 2)))  # >= 400 MB of weights in rotation
        ws = [torch.randn(N, K, device="cuda").to(torch.bfloat16) for _ in range(copies)]
        a = torch.randn(M, K, device="cuda").to(torch.bfloat16)
        acc = torch.zeros(M, N, device="cuda")
        out = torch.empty(M, N, device="cuda", dtype=torch.bfloat16)
        i = [0]

        def ours(pdl):
            def f():
                ops.gemm_decode(a, ws[i[0] % copies], acc, pdl=pdl)
                i[0] += 1
            return f

        def ref():
            torch.matmul(a, ws[i[0] % copies].t(), out=out)
            i[0] += 1

        calls = max(copies, iters)
        ms = _time_graph(ours(False), calls)
        ms_pdl = _time_graph(ours(True), calls)
        ms_ref = _time_graph(ref, calls)
        gb = N * K * 2 / 1e9
        ops.check_kernel_errors()
        print(json.dumps({"kernel": "gemm_decode", "case": name, "M": M, "N": N, "K": K, "ms": ms,
                          "weight_gbs": gb / (ms / 1e3), "ms_pdl": ms_pdl, "weight_gbs_pdl": gb / (ms_pdl / 1e3),
                          "torch_ms": ms_ref, "torch_gbs": gb / (ms_ref / 1e3)}), flush=True)
    # attention: Qwen3-4B heads, one layer's cache, several layers' caches in rotation
    lens = lens or [510] * batch
    Hkv, G, D, bs = 8, 4, 128, 16
    Hq = Hkv * G
    B = len(lens)
    nblk = sum(-(-L // bs) for L in lens)
    kv_bytes = 2 * sum(lens) * Hkv * D * 2
    copies = max(2, -(-400 * 2 ** 20 // kv_bytes))
    caches = [(torch.randn(nblk, bs, Hkv, D, device="cuda").to(torch.bfloat16),
               torch.randn(nblk, bs, Hkv, D, device="cuda").to(torch.bfloat16)) for _ in range(copies)]
    width = max(-(-L // bs) for L in lens)
    bt = torch.zeros(B, width, dtype=torch.int32)
    cur = 0
    for r, L in enumerate(lens):
        n = -(-L // bs)
        bt[r, :n] = torch.arange(cur, cur + n)
        cur += n
    bt = bt.cuda()
    lens_t = torch.tensor(lens, dtype=torch.int32, device="cuda")
    q = torch.randn(B, Hq, D, device="cuda").to(torch.bfloat16)
    out = torch.empty(B, Hq, D, device="cuda", dtype=torch.bfloat16)
    ws_o, ws_ml, counters = ops.decode_workspace(B, Hq, D, q.device)
    j = [0]

    def attn():
        kc, vc = caches[j[0] % copies]
        ops.decode_attention(q, kc, vc, bt, lens_t, out, ws_o, ws_ml, counters, 1.0 / D ** 0.5)
        j[0] += 1

    ms = _time_graph(attn, max(copies, iters))
    ops.check_kernel_errors()
    print(json.dumps({"kernel": "decode_attention", "batch": B, "mean_len": sum(lens) / B, "ms": ms,
                      "kv_gbs": kv_bytes / 1e9 / (ms / 1e3)}), flush=True)


def bench_peer_single(iters: int, case: str = "all"):
    """Fused compute+collective kernels in their single-rank mode (the peer
    pointers are this GPU's own buffers; every flag, copy and reduction phase
    runs, only the NVLink hop is local): the kernels as one rank executes them."""
    import math

    from libra_b200.parallel.peer_allreduce import PeerAllReduce
    from libra_b200.parallel.peer_gemm import PeerAllGatherGemm, PeerGemmAllReduce
    from libra_b200.parallel.peer_grad_reduce import PeerGradReduce
    from libra_b200.parallel.peer_param_gather import PeerParamGather

    def emit(name, ms, **kv):
        print(json.dumps({"kernel": name, "ms": round(ms, 4), **kv}), flush=True)

    dev = torch.device("cuda", torch.cuda.current_device())
    if case in ("gemm_ar", "gemm_rs", "all"):
        M, N, K = 16384, 2560, 2048
        a = torch.randn(M, K, device=dev).bfloat16()
        w = (torch.randn(N, K, device=dev) / math.sqrt(K)).bfloat16()
        f = PeerGemmAllReduce(None, M, N, dev)
        # the fused launches come first, so a profiler can take the first launch of the process
        out = {}
        if case in ("gemm_ar", "all"):
            out["gemm_allreduce (1 rank)"] = _time(lambda: f(a, w), iters)
        if case in ("gemm_rs", "all"):
            out["gemm_reduce_scatter (1 rank)"] = _time(lambda: f.reduce_scatter(a, w), iters)
        plain = _time(lambda: ops.gemm(a, w), iters)
        for name, ms in out.items():
            emit(name, ms, shape=[M, N, K], tflops=round(2 * M * N * K / ms / 1e9, 1), plain_gemm_ms=round(plain, 4))
        f.close()
    if case in ("ag_gemm", "all"):
        S, K, N = 8192, 2560, 6144
        a = torch.randn(S, K, device=dev).bfloat16()
        w = (torch.randn(N, K, device=dev) / math.sqrt(K)).bfloat16()
        f = PeerAllGatherGemm(None, S, K, dev)
        ms = _time(lambda: f(a, w), iters)
        plain = _time(lambda: ops.gemm(a, w), iters)
        emit("allgather_gemm (1 rank)", ms, shape=[S, N, K], tflops=round(2 * S * N * K / ms / 1e9, 1),
             plain_gemm_ms=round(plain, 4))
        f.close()
    if case in ("grad_rs", "all"):
        n = 128 << 20
        g = torch.randn(n, device=dev)
        out = torch.empty(n, device=dev)
        sq = torch.zeros(1, device=dev)
        red = PeerGradReduce(None, g, 0, n)
        ms = _time(lambda: red.reduce(out, sq_norm=sq), iters)
        emit("grad_reduce_scatter_peer (1 rank)", ms, bytes=8 * n, gbs=round(8 * n / ms / 1e6, 1))
        red.close()
    if case in ("adamw_ag", "all"):
        n = 128 << 20
        master = torch.randn(n, device=dev)
        grad = torch.randn(n, device=dev)
        m, v = torch.zeros_like(master), torch.zeros_like(master)
        flat = torch.zeros(n, dtype=torch.bfloat16, device=dev)
        pg = PeerParamGather(None, flat, 0, n)
        step = [0]

        def run():
            step[0] += 1
            pg.step(master, grad, m, v, lr=1e-5, beta1=0.9, beta2=0.95, eps=1e-8, weight_decay=0.0, step=step[0])

        ms = _time(run, iters)
        emit("adamw_step_allgather (1 rank)", ms, bytes=(16 + 12 + 2) * n, gbs=round(30 * n / ms / 1e6, 1))
        pg.close()
    if case in ("tp_ar_norm", "all"):
        rows, H = 4096, 2560
        ar = PeerAllReduce(None, rows, H, dev)
        res = torch.randn(rows, H, device=dev).bfloat16()
        wn = torch.ones(H, device=dev).bfloat16()

        def run():
            ar.partial(rows).copy_(res)
            return ar.reduce_add_rmsnorm(res, wn, 1e-6)

        ms = _time(run, iters)
        emit("tp_allreduce_add_rmsnorm (1 rank, incl. partial copy)", ms, rows=rows, hidden=H)
        ar.close()


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("what", choices=["gemm", "elementwise", "attention", "swiglu", "decode", "peer1", "all"])
    ap.add_argument("--case", default="all", help="peer1: gemm_ar, gemm_rs, ag_gemm, grad_rs, adamw_ag, tp_ar_norm")
    ap.add_argument("--batch", type=int, default=64, help="decode: batch rows")
    ap.add_argument("--iters", type=int, default=20)
    ap.add_argument("--shapes", default="", help="name:M,N,K,a_mn,b_mn;...")
    ap.add_argument("--lens", default="", help="attention: sequence lengths, e.g. 2048x4")
    args = ap.parse_args()
    shapes = QWEN3_4B_SHAPES
    if args.shapes:
        shapes = []
        for item in args.shapes.split(";"):
            name, dims = item.split(":")
            M, N, K, a_mn, b_mn = dims.split(",")
            shapes.append((name, int(M), int(N), int(K), a_mn == "1", b_mn == "1"))
    if args.what in ("gemm", "all"):
        bench_gemm(shapes, args.iters)
    if args.what in ("elementwise", "all"):
        bench_elementwise(args.iters)
    if args.what in ("swiglu", "all"):
        bench_swiglu(args.iters)
    if args.what in ("decode", "all"):
        lens = None
        if args.lens:
            n, c = args.lens.split("x")
            lens = [int(n)] * int(c)
        bench_decode(args.iters, args.batch, lens)
    if args.what == "peer1":
        bench_peer_single(args.iters, args.case)
    if args.what in ("attention", "all"):
        lens = None
        if args.lens:
            n, c = args.lens.split("x")
            lens = [int(n)] * int(c)
        bench_attention(args.iters, lens)


if __name__ == "__main__":
    main()
