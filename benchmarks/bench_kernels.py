"""Micro-benchmarks of this package's CUDA kernels (CUDA-event timing).

``python benchmarks/bench_kernels.py attn --mode bwd --t 2048 --s 2560``
times one kernel family on the current GPU after warm-up, with inputs
allocated once, and prints one line per measurement (milliseconds and the
achieved TFLOP/s or GB/s against the algorithmic work). It is also the small,
self-contained case that kernel profiles are captured on.

Families: ``attn`` (bottom-right causal GQA attention; fwd, or fwd+bwd),
``rms`` (RMSNorm fwd/bwd), ``lse`` (log-sum-exp/gather over fp32 logits),
``gdn`` (gated delta rule fwd/bwd), ``conv`` (causal conv1d + SiLU fwd/bwd),
``swiglu``, ``rope`` (QK-norm + RoPE), ``dlogits``, ``adamw``, ``fold``
(GRPO statistic folds), ``gemm`` (tcgen05 GEMM vs the library at decoder
shapes), ``lmhead`` (fused tcgen05 LM-head logprob fwd+bwd vs the unfused
cuBLAS-logits path), ``baselines`` (attention vs FlashAttention-2, the reference's
GPU path without FA4, and the gated delta rule timed alone) and
``gemm_host`` (host cost of a library GEMM call).
"""

from __future__ import annotations

import os
import sys

sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))

import argparse
import math

import torch

from thundersync_b200.ops._ext import native


def _time(fn, iters: int, warmup: int = 3) -> float:
    for _ in range(warmup):
        fn()
    torch.cuda.synchronize()
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    a.record()
    for _ in range(iters):
        fn()
    b.record()
    torch.cuda.synchronize()
    return a.elapsed_time(b) / iters


def bench_attn(args) -> None:
    t, s, hq, hkv, d = args.t, args.s, args.hq, args.hkv, args.d
    g = torch.Generator(device="cuda").manual_seed(0)
    q = torch.randn(t, hq, d, device="cuda", dtype=torch.bfloat16, generator=g)
    k = torch.randn(s, hkv, d, device="cuda", dtype=torch.bfloat16, generator=g)
    v = torch.randn(s, hkv, d, device="cuda", dtype=torch.bfloat16, generator=g)
    scale = 1 / math.sqrt(d)
    flops = 4 * hq * d * (t * (s - t) + t * (t + 1) / 2)  # two GEMMs over the visible (q, k) pairs
    ext = native()
    o, lse = ext.attn_fwd_tc(q, k, v, scale)
    ms = _time(lambda: ext.attn_fwd_tc(q, k, v, scale), args.iters)
    print(f"attn fwd T={t} S={s} Hq={hq} Hkv={hkv} D={d}: {ms:.3f} ms  {flops / ms / 1e9:.1f} TFLOP/s")
    if args.mode == "bwd":
        do = torch.randn(o.shape, device="cuda", dtype=torch.bfloat16, generator=g)
        ms = _time(lambda: ext.attn_bwd_tc(do, q, k, v, o, lse, scale), args.iters)
        print(f"attn bwd: {ms:.3f} ms  {2.5 * flops / ms / 1e9:.1f} TFLOP/s (5 GEMM-equivalents)")
        if args.kernels:  # device time of each kernel of one backward
            from torch.profiler import ProfilerActivity, profile

            with profile(activities=[ProfilerActivity.CUDA]) as prof:
                ext.attn_bwd_tc(do, q, k, v, o, lse, scale)
                torch.cuda.synchronize()
            print(prof.key_averages().table(sort_by="cuda_time_total", row_limit=8, max_name_column_width=60))
    print("kernel status", int(ext.tc_status(q).item()))


def bench_rms(args) -> None:
    x = torch.randn(args.rows, args.cols, device="cuda", dtype=torch.bfloat16)
    w = torch.rand(args.cols, device="cuda", dtype=torch.bfloat16)
    ext = native()
    y, r = ext.rms_norm_fwd(x, w, 1e-6, False)
    ms = _time(lambda: ext.rms_norm_fwd(x, w, 1e-6, False), args.iters)
    gb = 2 * x.numel() * 2 / 1e9
    print(f"rms fwd {args.rows}x{args.cols}: {ms:.3f} ms  {gb / ms * 1e3:.0f} GB/s")
    dy = torch.randn_like(x)
    ms = _time(lambda: ext.rms_norm_bwd(dy, x, w, r, False), args.iters)
    print(f"rms bwd (one pass, dx + weight partials): {ms:.3f} ms  {1.5 * gb / ms * 1e3:.0f} GB/s")
    res = torch.randn_like(x)
    ms = _time(lambda: ext.rms_norm_bwd(dy, x, w, r, False, res), args.iters)
    print(f"rms bwd + residual gradient: {ms:.3f} ms  {2 * gb / ms * 1e3:.0f} GB/s")
    # the allocation-free entry point runs the three-kernel form (dx; column partials; ordered sum)
    import ctypes

    from thundersync_b200.ops._ext import so_path

    fn = ctypes.CDLL(so_path()).ts_rms_norm_bwd_noalloc
    fn.argtypes = [ctypes.c_void_p] * 6 + [ctypes.c_int, ctypes.c_int, ctypes.c_int, ctypes.c_void_p]
    fn.restype = ctypes.c_int
    dx = torch.empty_like(x)
    dw = torch.empty(args.cols, device="cuda", dtype=torch.float32)
    st = torch.cuda.current_stream().cuda_stream
    if args.cols <= 4096 and args.rows <= 128 * 1024:
        ms = _time(lambda: fn(dy.data_ptr(), x.data_ptr(), w.data_ptr(), r.data_ptr(), dx.data_ptr(),
                              dw.data_ptr(), args.rows, args.cols, 0, st), args.iters)
        print(f"rms bwd (three kernels): {ms:.3f} ms  {1.5 * gb / ms * 1e3:.0f} GB/s")


def bench_baselines(args) -> None:
    """The reference's GPU baselines on this box, next to this package's kernels: attention against
    FlashAttention-2 (the reference's path when FA4 is absent; bottom-right causal, GQA). The gated delta rule
    is timed alone: FLA's chunked Triton kernel, the reference's hybrid-layer path, faulted on this box."""
    from thundersync_b200.ops.attention import chunked_attention
    from thundersync_b200.ops.gdn import gated_delta_rule

    torch.manual_seed(0)
    for t, s, hq, hkv, d in ((args.t, args.s, args.hq, args.hkv, 128), (args.t, args.s, 16, 2, 256)):
        q = torch.randn(t, hq, d, device="cuda", dtype=torch.bfloat16, requires_grad=True)
        k = torch.randn(s, hkv, d, device="cuda", dtype=torch.bfloat16, requires_grad=True)
        v = torch.randn(s, hkv, d, device="cuda", dtype=torch.bfloat16, requires_grad=True)
        do = torch.randn(t, hq, d, device="cuda", dtype=torch.bfloat16)
        pairs = t * (s - t) + t * (t + 1) / 2
        flops = 4.0 * pairs * hq * d
        with torch.no_grad():
            f_ours = _time(lambda: chunked_attention(q, [k], [v]), args.iters)
        b_ours = _time(lambda: torch.autograd.grad(chunked_attention(q, [k], [v]), (q, k, v), do), args.iters)
        line = (f"attention T={t} S={s} {hq}/{hkv} heads d={d}: ours fwd {f_ours:.3f} ms "
                f"({flops / f_ours / 1e9:.0f} TFLOP/s), fwd+bwd {b_ours:.3f} ms ({3.5 * flops / b_ours / 1e9:.0f})")
        try:
            from flash_attn import flash_attn_func

            q4, k4, v4, do4 = q[None], k[None], v[None], do[None]
            with torch.no_grad():
                f_fa = _time(lambda: flash_attn_func(q4, k4, v4, causal=True), args.iters)
            b_fa = _time(lambda: torch.autograd.grad(flash_attn_func(q4, k4, v4, causal=True), (q4, k4, v4), do4),
                         args.iters)
            line += (f"; FlashAttention-2 fwd {f_fa:.3f} ms ({flops / f_fa / 1e9:.0f}), "
                     f"fwd+bwd {b_fa:.3f} ms ({3.5 * flops / b_fa / 1e9:.0f})")
        except Exception as exc:  # noqa: BLE001 - report, do not fail the other lines
            line += f"; FlashAttention-2 unavailable ({type(exc).__name__}: {exc})"[:160]
        print(line)
    t, h, dk = args.t, args.h, 128
    q = torch.randn(t, h, dk, device="cuda", dtype=torch.bfloat16, requires_grad=True)
    k = torch.randn(t, h, dk, device="cuda", dtype=torch.bfloat16, requires_grad=True)
    v = torch.randn(t, h, dk, device="cuda", dtype=torch.bfloat16, requires_grad=True)
    g = (-torch.rand(t, h, device="cuda") * 0.3).requires_grad_(True)
    beta = torch.rand(t, h, device="cuda").requires_grad_(True)
    s0 = torch.zeros(h, dk, dk, device="cuda", requires_grad=True)
    do = torch.randn(t, h, dk, device="cuda", dtype=torch.bfloat16)
    with torch.no_grad():
        f_ours = _time(lambda: gated_delta_rule(q, k, v, g, beta, s0), args.iters)
    b_ours = _time(lambda: torch.autograd.grad(gated_delta_rule(q, k, v, g, beta, s0)[0], (q, k, v, g, beta, s0), do),
                   args.iters)
    # FLA's chunked Triton kernel is not run: on this box it raised "misaligned address" (a device fault)
    print(f"gated delta rule T={t} H={h} dk=dv={dk}: ours fwd {f_ours:.3f} ms, fwd+bwd {b_ours:.3f} ms")


def bench_lse(args) -> None:
    logits = torch.randn(args.rows, args.cols, device="cuda", dtype=torch.float32)
    tgt = torch.randint(0, args.cols, (args.rows,), device="cuda")
    ext = native()
    ms = _time(lambda: ext.lse_gather(logits, tgt, False), args.iters)
    print(f"lse {args.rows}x{args.cols}: {ms:.3f} ms  {logits.numel() * 4 / ms / 1e6:.0f} GB/s")


def bench_gdn(args) -> None:
    t, h = args.t, args.h
    q = torch.randn(t, h, 128, device="cuda", dtype=torch.bfloat16)
    k = torch.randn(t, h, 128, device="cuda", dtype=torch.bfloat16)
    v = torch.randn(t, h, 128, device="cuda", dtype=torch.bfloat16)
    gg = -torch.rand(t, h, device="cuda") * 0.1
    beta = torch.rand(t, h, device="cuda")
    s0 = torch.zeros(h, 128, 128, device="cuda")
    ext = native()
    o, fin, *saved = ext.gdn_chunk_fwd(q, k, v, gg, beta, s0)
    ms = _time(lambda: ext.gdn_chunk_fwd(q, k, v, gg, beta, s0), args.iters)
    print(f"gdn chunked fwd T={t} H={h}: {ms:.3f} ms  {t / ms * 1e3:.0f} tokens/s")
    do = torch.randn_like(o)
    dfin = torch.zeros_like(fin)
    ms = _time(lambda: ext.gdn_chunk_bwd(do, dfin, q, k, v, gg, beta, *saved), args.iters)
    print(f"gdn chunked bwd: {ms:.3f} ms")
    o, fin, ck = ext.gdn_fwd(q, k, v, gg, beta, s0)
    ms = _time(lambda: ext.gdn_fwd(q, k, v, gg, beta, s0), args.iters)
    print(f"gdn token-recurrent fwd: {ms:.3f} ms")
    ms = _time(lambda: ext.gdn_bwd(do, dfin, q, k, v, gg, beta, ck), args.iters)
    print(f"gdn token-recurrent bwd: {ms:.3f} ms")


def bench_conv(args) -> None:
    x = torch.randn(args.rows, args.cols, device="cuda", dtype=torch.bfloat16)
    w = torch.randn(args.cols, 4, device="cuda", dtype=torch.bfloat16)
    tail = torch.zeros(3, args.cols, device="cuda", dtype=torch.bfloat16)
    ext = native()
    y, nt = ext.conv1d_silu_fwd(x, w, tail)
    ms = _time(lambda: ext.conv1d_silu_fwd(x, w, tail), args.iters)
    print(f"conv fwd {args.rows}x{args.cols}: {ms:.3f} ms  {2 * x.numel() * 2 / ms / 1e6:.0f} GB/s")
    dy = torch.randn_like(y)
    ms = _time(lambda: ext.conv1d_silu_bwd(dy, torch.zeros_like(nt), x, w, tail), args.iters)
    print(f"conv bwd: {ms:.3f} ms")


def bench_swiglu(args) -> None:
    gu = torch.randn(args.rows, 2 * args.cols, device="cuda", dtype=torch.bfloat16)
    ext = native()
    a = ext.swiglu_fwd(gu)
    ms = _time(lambda: ext.swiglu_fwd(gu), args.iters)
    print(f"swiglu fwd {args.rows}x{args.cols}: {ms:.3f} ms  {3 * a.numel() * 2 / ms / 1e6:.0f} GB/s")
    ms = _time(lambda: ext.swiglu_bwd(a, gu), args.iters)
    print(f"swiglu bwd: {ms:.3f} ms  {5 * a.numel() * 2 / ms / 1e6:.0f} GB/s")


def bench_rope(args) -> None:
    hq, hkv, d = args.hq, args.hkv, args.d
    qkv = torch.randn(args.rows, (hq + 2 * hkv) * d, device="cuda", dtype=torch.bfloat16)
    qw = torch.rand(d, device="cuda", dtype=torch.bfloat16)
    kw = torch.rand(d, device="cuda", dtype=torch.bfloat16)
    pos = torch.arange(args.rows, device="cuda")
    inv = 1.0 / (1e6 ** (torch.arange(0, d, 2, device="cuda").float() / d))
    from thundersync_b200.ops.rope import rope_tables

    ext = native()
    ct, st = rope_tables(inv)
    q, k, v = ext.qk_norm_rope_fwd(qkv, qw, kw, pos, inv, hq, hkv, d, 1e-6, False, ct, st)
    ms = _time(lambda: ext.qk_norm_rope_fwd(qkv, qw, kw, pos, inv, hq, hkv, d, 1e-6, False, ct, st), args.iters)
    print(f"qk_norm_rope fwd {args.rows} rows: {ms:.3f} ms  {2 * qkv.numel() * 2 / ms / 1e6:.0f} GB/s")
    ms = _time(lambda: ext.qk_norm_rope_bwd(q, k, v, qkv, qw, kw, pos, inv, hq, hkv, d, 1e-6, False, ct, st),
               args.iters)
    print(f"qk_norm_rope bwd: {ms:.3f} ms  {3 * qkv.numel() * 2 / ms / 1e6:.0f} GB/s")


def bench_dlogits(args) -> None:
    logits = torch.randn(args.rows, args.cols, device="cuda", dtype=torch.float32)
    tgt = torch.randint(0, args.cols, (args.rows,), device="cuda")
    ext = native()
    lp, lse, _ = ext.lse_gather(logits, tgt, False)
    g = torch.randn(args.rows, device="cuda")
    ms = _time(lambda: ext.logprob_dlogits(logits, tgt, lse, g, None, None, True), args.iters)
    print(f"dlogits {args.rows}x{args.cols}: {ms:.3f} ms  {logits.numel() * 6 / ms / 1e6:.0f} GB/s")


def bench_adamw(args) -> None:
    n = args.rows * args.cols
    master = torch.randn(n, device="cuda")
    param = master.to(torch.bfloat16)
    grad = torch.randn(n, device="cuda")
    m = torch.zeros(n, device="cuda")
    v = torch.zeros(n, device="cuda")
    ext = native()
    ms = _time(lambda: ext.adamw_flat(master, param, grad, m, v, 1e-5, 0.9, 0.999, 1e-8, 0.0, 1, None, 1.0, True),
               args.iters)
    print(f"adamw {n} elems: {ms:.3f} ms  {n * 18 / ms / 1e6:.0f} GB/s")


def bench_fold(args) -> None:
    n = args.rows * args.cols
    g1 = torch.zeros(n, device="cuda")
    g2 = torch.zeros(n, device="cuda")
    src = torch.randn(n, device="cuda")
    ext = native()
    ms = _time(lambda: ext.fold_stats(g1, g2, src, 1.0), args.iters)
    print(f"fold {n} elems: {ms:.3f} ms  {n * 20 / ms / 1e6:.0f} GB/s")
    ms = _time(lambda: ext.axpby(g1, g2, src, 0.5, -0.25), args.iters)
    print(f"axpby {n} elems: {ms:.3f} ms  {n * 16 / ms / 1e6:.0f} GB/s")


def bench_gemm(args) -> None:
    """tcgen05 GEMM variants vs the library GEMM on the decoder's projection shapes: CTA pairs with the automatic
    256x256 / 256x512 tile choice, 256x256 only, 256x512 only, and the single-CTA 128x256 kernel. Variants run
    one after another: compare within a line (``gemm_ab`` interleaves them)."""
    ext = native()
    variants = [("CTA pair, automatic 256x256 / 256x512 choice", 1, 1), ("CTA pair, 256x256 tiles", 1, 0),
                ("CTA pair, 256x512 tiles", 1, 2), ("single CTA, 128x256 tiles", 0, 0)]
    for name, pair, wide in variants:
        prev, prev_w = ext.gemm_tc_pair(pair), ext.gemm_tc_wide(wide)
        print(f"-- tcgen05 kernel: {name}")
        try:
            _bench_gemm_shapes(args)
        finally:
            ext.gemm_tc_pair(prev)
            ext.gemm_tc_wide(prev_w)


def bench_gemm_ab(args) -> None:
    """Interleaved A/B of tcgen05 GEMM launch variants at the projection shapes: for each shape the variants
    (kernel selection settings) alternate, ``--rounds`` rounds of ``--iters`` launches each, and the median
    per variant is reported next to the library GEMM timed in the same rounds. Clock changes under the power
    cap then shift every variant of a shape alike, which a variant-by-variant sweep does not guarantee."""
    from thundersync_b200.ops.gemm import gemm, gemm_accumulate

    ext = native()
    variants = {"by output mode (default)": dict(pair=2, wide=0, epi=1),
                "pair 256x256, 4 epilogue warps": dict(pair=1, wide=0, epi=0),
                "pair 256x256, 8 epilogue warps for bf16": dict(pair=1, wide=0, epi=1),
                "single CTA 128x256": dict(pair=0, wide=0, epi=1)}
    m = args.rows
    cases = []
    for name, n, k in [("qkv fwd", 4096, 2048), ("o fwd", 2048, 2048), ("gate/up fwd", 12288, 2048),
                       ("down fwd", 2048, 6144)]:
        x = torch.randn(m, k, device="cuda", dtype=torch.bfloat16)
        w = torch.randn(n, k, device="cuda", dtype=torch.bfloat16)
        cases.append((f"{name} {m}x{n}x{k}", 2.0 * m * n * k, (lambda x=x, w=w: gemm(x, w)),
                      (lambda x=x, w=w: torch.nn.functional.linear(x, w))))
    for name, n, k in (("dW qkv", 4096, 2048), ("dW gate/up", 12288, 2048)):
        dy = torch.randn(m, n, device="cuda", dtype=torch.bfloat16)
        x = torch.randn(m, k, device="cuda", dtype=torch.bfloat16)
        acc = torch.zeros(n, k, device="cuda")
        cases.append((f"{name} {n}x{k}x{m} fp32+=", 2.0 * m * n * k,
                      (lambda a=acc, dy=dy, x=x: gemm_accumulate(a, dy, x, a_t=True, b_t=False)),
                      (lambda a=acc, dy=dy, x=x: torch.addmm(a, dy.t(), x, out_dtype=torch.float32, out=a))))
    for name, n, k in (("dx qkv", 2048, 4096), ("dx down", 6144, 2048)):
        dy = torch.randn(m, k, device="cuda", dtype=torch.bfloat16)
        w = torch.randn(k, n, device="cuda", dtype=torch.bfloat16)  # the weight [out, in]: dx = dy · W
        cases.append((f"{name} {m}x{n}x{k}", 2.0 * m * n * k, (lambda dy=dy, w=w: gemm(dy, w, b_t=False)),
                      (lambda dy=dy, w=w: torch.matmul(dy, w))))
    prev = (ext.gemm_tc_pair(-1), ext.gemm_tc_wide(-1), ext.gemm_tc_epi8(-1))
    try:
        for label, flops, ours, lib in cases:
            times = {v: [] for v in variants}
            times["library"] = []
            for _ in range(args.rounds):
                for v, cfg in variants.items():
                    ext.gemm_tc_pair(cfg["pair"])
                    ext.gemm_tc_wide(cfg["wide"])
                    ext.gemm_tc_epi8(cfg["epi"])
                    times[v].append(_time(ours, args.iters))
                times["library"].append(_time(lib, args.iters))
            med = {v: sorted(t)[len(t) // 2] for v, t in times.items()}
            cells = ", ".join(f"{v}: {flops / med[v] / 1e9:.0f}" for v in times)
            print(f"{label}: TFLOP/s {cells}")
    finally:
        ext.gemm_tc_pair(prev[0])
        ext.gemm_tc_wide(prev[1])
        ext.gemm_tc_epi8(prev[2])


def bench_gemm_one(args) -> None:
    """One projection GEMM, x [rows, cols] · Wᵀ with W [n, cols] (bf16 out), with the default kernel selection;
    the small case an ncu capture of a single launch runs on."""
    from thundersync_b200.ops.gemm import gemm

    x = torch.randn(args.rows, args.cols, device="cuda", dtype=torch.bfloat16)
    w = torch.randn(args.n, args.cols, device="cuda", dtype=torch.bfloat16)
    ms = _time(lambda: gemm(x, w), args.iters)
    print(f"gemm {args.rows}x{args.n}x{args.cols}: {ms:.4f} ms  {2.0 * args.rows * args.n * args.cols / ms / 1e9:.1f} "
          "TFLOP/s")


def bench_packed(args) -> None:
    """Packed attention vs per-segment attention on a close-rebuild pack: ``--segs`` trajectories of one group
    (lengths spread over [--t / 4, --t]) that share a 512-token prompt chunk, 16 q / 8 kv heads, d = 128.
    Times forward + backward of `packed_attention` (one launch each way, the shared prompt stored once) against
    one `chunked_attention` call per segment (the prompt concatenated into each segment's chain)."""
    import random

    from thundersync_b200.ops.attention import chunked_attention
    from thundersync_b200.ops.packed_attention import packed_attention

    hq, hkv, d = 16, 8, 128
    rng = random.Random(0)
    lens = [rng.randint(args.t // 4, args.t) for _ in range(args.segs)]
    t = sum(lens)
    dev = "cuda"
    prompt_k = torch.randn(512, hkv, d, device=dev, dtype=torch.bfloat16, requires_grad=True)
    prompt_v = torch.randn(512, hkv, d, device=dev, dtype=torch.bfloat16, requires_grad=True)
    q = torch.randn(t, hq, d, device=dev, dtype=torch.bfloat16, requires_grad=True)
    k = torch.randn(t, hkv, d, device=dev, dtype=torch.bfloat16, requires_grad=True)
    v = torch.randn(t, hkv, d, device=dev, dtype=torch.bfloat16, requires_grad=True)
    meta, s0 = [], 0
    for n in lens:
        meta.append((s0, s0 + n, 1, ()))
        s0 += n
    pk, pv = [prompt_k] * len(lens), [prompt_v] * len(lens)
    g = torch.randn(t, hq, d, device=dev, dtype=torch.bfloat16)

    def packed():
        o = packed_attention(q, k, v, meta, pk, pv)
        torch.autograd.backward(o, g)

    def per_segment():
        outs = [chunked_attention(q[a:b], [prompt_k, k[a:b]], [prompt_v, v[a:b]]) for a, b, _, _ in meta]
        torch.autograd.backward(torch.cat(outs, 0), g)

    pairs = sum(n * 512 + n * (n + 1) / 2 for n in lens)
    flops = 3.5 * 4 * hq * d * pairs  # forward (2 GEMMs) + backward (5): 7 GEMM-equivalents of 2*pairs*hq*d
    for name, fn in (("packed (one launch each way)", packed), ("per segment", per_segment)):
        ms = _time(fn, args.iters)
        print(f"{name:30s} {len(lens)} segments, {t} queries: {ms:.3f} ms fwd+bwd  {flops / ms / 1e9:.1f} TFLOP/s")


def _bench_gemm_shapes(args) -> None:
    from thundersync_b200.ops.gemm import gemm, gemm_accumulate

    m = args.rows
    shapes = [("qkv fwd", 4096, 2048), ("o fwd", 2048, 2048), ("gate/up fwd", 12288, 2048), ("down fwd", 2048, 6144),
              ("lm head chunk", 151936, 2048)]
    for name, n, k in shapes:
        x = torch.randn(m, k, device="cuda", dtype=torch.bfloat16)
        w = torch.randn(n, k, device="cuda", dtype=torch.bfloat16)
        flops = 2.0 * m * n * k
        t_ours = _time(lambda: gemm(x, w), args.iters)
        t_lib = _time(lambda: torch.nn.functional.linear(x, w), args.iters)
        print(f"{name:14s} {m}x{n}x{k}: tcgen05 {flops / t_ours / 1e9:7.1f} TFLOP/s, library {flops / t_lib / 1e9:7.1f}")
    for name, n, k in (("dW qkv", 4096, 2048), ("dW gate/up", 12288, 2048)):
        dy = torch.randn(m, n, device="cuda", dtype=torch.bfloat16)
        x = torch.randn(m, k, device="cuda", dtype=torch.bfloat16)
        acc = torch.zeros(n, k, device="cuda")
        flops = 2.0 * m * n * k
        t_ours = _time(lambda: gemm_accumulate(acc, dy, x, a_t=True, b_t=False), args.iters)
        t_lib = _time(lambda: torch.addmm(acc, dy.t(), x, out_dtype=torch.float32, out=acc), args.iters)
        print(f"{name:14s} {n}x{k}x{m} (fp32 +=): tcgen05 {flops / t_ours / 1e9:7.1f} TFLOP/s, "
              f"library {flops / t_lib / 1e9:7.1f}")
    for name, n, k in (("dx qkv", 2048, 4096), ("dx down", 6144, 2048)):
        dy = torch.randn(m, k, device="cuda", dtype=torch.bfloat16)
        w = torch.randn(k, n, device="cuda", dtype=torch.bfloat16)
        flops = 2.0 * m * n * k
        t_ours = _time(lambda: gemm(dy, w, b_t=False), args.iters)
        t_lib = _time(lambda: dy.matmul(w), args.iters)
        print(f"{name:14s} {m}x{n}x{k}: tcgen05 {flops / t_ours / 1e9:7.1f} TFLOP/s, library {flops / t_lib / 1e9:7.1f}")


def bench_lmhead(args) -> None:
    """LM-head logprob forward and forward+backward: fused tcgen05 epilogues vs cuBLAS logits + row kernels."""
    from thundersync_b200.ops import logprob as L

    n, dmod, vocab = args.rows, args.cols, 151936
    h = (torch.randn(n, dmod, device="cuda") / dmod ** 0.5).to(torch.bfloat16).requires_grad_(True)
    w = (torch.randn(vocab, dmod, device="cuda") / dmod ** 0.25).to(torch.bfloat16).requires_grad_(True)
    tgt = torch.randint(0, vocab, (n,), device="cuda")
    g = torch.randn(n, device="cuda")
    flops = 2.0 * n * dmod * vocab
    for fused in (True, False):
        L.FUSED_TC = fused
        with torch.no_grad():
            t_f = _time(lambda: L.lm_head_logprob(h, w, tgt), args.iters)
        t_fb = _time(lambda: torch.autograd.grad(L.lm_head_logprob(h, w, tgt), (h, w), g), args.iters)
        name = "fused tcgen05" if fused else "cuBLAS+rows"
        print(f"lmhead {name:14s} {n}x{dmod}x{vocab}: fwd {t_f:.3f} ms ({flops / t_f / 1e9:.0f} TFLOP/s), "
              f"fwd+bwd {t_fb:.3f} ms ({4 * flops / t_fb / 1e9:.0f} TFLOP/s of 4 GEMMs)")
    L.FUSED_TC = True


def bench_lora(args) -> None:
    """LoRA projection (Qwen3-8B q_proj: 4096 -> 4096, rank 64) fwd and fwd+bwd: this package's unmerged op
    vs the merged-weight form (one base GEMM forward, the reference's fused mode) and the bare base GEMM."""
    from thundersync_b200.accel.fused_lora import FusedLoRALinear
    from thundersync_b200.ops.lora import _LoRALinear

    t, din, dout, r, s = args.rows, 4096, 4096, 64, 2.0
    x = (torch.randn(t, din, device="cuda") * 0.5).to(torch.bfloat16).requires_grad_(True)
    w = (torch.randn(dout, din, device="cuda") / din ** 0.5).to(torch.bfloat16)
    a = (torch.randn(r, din, device="cuda") / din ** 0.5).requires_grad_(True)
    b = (torch.randn(dout, r, device="cuda") * 0.01).requires_grad_(True)
    dy = torch.randn(t, dout, device="cuda", dtype=torch.bfloat16)
    flops = 2.0 * t * din * dout
    from thundersync_b200.ops import lora as L

    cases = (("unmerged, one tcgen05 GEMM", True, lambda: _LoRALinear.apply(x, w, a, b, s)),
             ("unmerged, library GEMMs", False, lambda: _LoRALinear.apply(x, w, a, b, s)),
             ("merged weight", True, lambda: FusedLoRALinear.apply(x, w, a, b, s)),
             ("base GEMM alone", True, lambda: x @ w.t()))
    for name, fused, fn in cases:
        L.FUSED_TC = fused
        with torch.no_grad():
            f = _time(fn, args.iters)
        fb = _time(lambda: torch.autograd.grad(fn(), (x, a, b), dy, allow_unused=True), args.iters)
        print(f"lora {name:28s} T={t}: fwd {f:.3f} ms ({flops / f / 1e9:.0f} TFLOP/s of the base GEMM), "
              f"fwd+bwd(dx, dA, dB) {fb:.3f} ms")
    L.FUSED_TC = True
    if args.trace:  # per-kernel device times of one unmerged forward+backward
        from torch.profiler import ProfilerActivity, profile

        fn = cases[0][2]
        torch.autograd.grad(fn(), (x, a, b), dy)
        torch.cuda.synchronize()
        with profile(activities=[ProfilerActivity.CUDA]) as prof:
            torch.autograd.grad(fn(), (x, a, b), dy)
            torch.cuda.synchronize()
        print(prof.key_averages().table(sort_by="cuda_time_total", row_limit=15, max_name_column_width=70))


def bench_layer_host(args) -> None:
    """Host time vs device time of one pack through all decoder layers (Qwen3-1.7B shapes), forward + backward
    into a gradient sink, for several pack lengths: where host time exceeds device time the GPU waits."""
    import time

    from thundersync_b200.engine.layers import Executor, Segment
    from thundersync_b200.engine.streaming import arena_for
    from thundersync_b200.models.qwen3 import PRESETS, Qwen3ForCausalLM
    from thundersync_b200.ops.sink import GradSink, grad_sink

    torch.manual_seed(0)
    with torch.device("cuda"):
        model = Qwen3ForCausalLM(PRESETS["qwen3-1.7b"])
    model.to(torch.bfloat16)
    arena = arena_for(model)
    ex = Executor(model, arena)
    buf = torch.zeros(arena.numel, device="cuda")
    prompt = 512
    ids_p = torch.randint(0, 1000, (prompt,), device="cuda")
    with torch.no_grad():
        _, st = ex.run(ids_p, torch.arange(prompt, device="cuda"), [Segment(0, prompt, [])])
    past = [([k], [v]) for (k, v) in st[0]]
    for n in (256, 1024, 2176, 4096):
        pad = (-n) % 128
        ids = torch.randint(0, 1000, (n + pad,), device="cuda")
        pos = torch.cat((torch.arange(prompt, prompt + n, device="cuda"), torch.zeros(pad, dtype=torch.long,
                                                                                        device="cuda")))

        def once():
            h, _ = ex.run(ids, pos, [Segment(0, n, past)])
            with grad_sink(GradSink(arena, buf)):
                h[:n].float().square().mean().backward()

        for _ in range(2):
            once()
        torch.cuda.synchronize()
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record()
        t0 = time.perf_counter()
        for _ in range(args.iters):
            once()
        t1 = time.perf_counter()
        b.record()
        torch.cuda.synchronize()
        print(f"pack of {n} tokens (+{pad} padding) over a {prompt}-token prompt: host issue {1e3 * (t1 - t0) / args.iters:.2f} ms, "
              f"device {a.elapsed_time(b) / args.iters:.2f} ms per forward+backward")


def bench_gemm_host(args) -> None:
    """Host (CPU) cost of one library GEMM call: repeated shape vs a new row count every call."""
    import time

    w = torch.randn(6144, 2048, device="cuda", dtype=torch.bfloat16)
    xs = [torch.randn(1000 + 7 * i, 2048, device="cuda", dtype=torch.bfloat16) for i in range(200)]
    acc = torch.zeros(6144, 2048, device="cuda", dtype=torch.float32)
    for name, seq in (("same", [xs[0]] * 200), ("varying", xs)):
        for fn_name, fn in (("linear", lambda x: torch.nn.functional.linear(x, w)),
                            ("addmm_fp32", lambda x: torch.addmm(acc, w.new_empty(6144, x.shape[0]).normal_() if False
                                                                 else torch.empty(6144, x.shape[0], device="cuda",
                                                                                  dtype=torch.bfloat16), x,
                                                                 out_dtype=torch.float32, out=acc))):
            fn(seq[0])
            torch.cuda.synchronize()
            t0 = time.perf_counter()
            for x in seq:
                fn(x)
            t1 = time.perf_counter()
            torch.cuda.synchronize()
            t2 = time.perf_counter()
            print(f"{fn_name:10s} {name:8s}: host {1e6 * (t1 - t0) / len(seq):7.1f} us/call, "
                  f"device+host {1e6 * (t2 - t0) / len(seq):7.1f} us/call")
    # host issue cost of single small launches (a 256-row pack): library GEMM vs this package's kernels
    ext = native()
    x = torch.randn(256, 2048, device="cuda", dtype=torch.bfloat16)
    wq = torch.randn(4096, 2048, device="cuda", dtype=torch.bfloat16)
    y = torch.empty(256, 4096, device="cuda", dtype=torch.bfloat16)
    ln = torch.ones(2048, device="cuda", dtype=torch.bfloat16)
    q = torch.randn(256, 16, 128, device="cuda", dtype=torch.bfloat16)
    kv = torch.randn(768, 8, 128, device="cuda", dtype=torch.bfloat16)
    acc = torch.zeros(4096, 2048, device="cuda")
    dy = torch.randn(256, 4096, device="cuda", dtype=torch.bfloat16)
    side = torch.cuda.Stream()

    def deposit_side():
        side.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(side):
            torch.addmm(acc, dy.t(), x, out_dtype=torch.float32, out=acc)
        torch.cuda.current_stream().wait_stream(side)

    cases = (("F.linear 256x4096x2048", lambda: torch.nn.functional.linear(x, wq)),
             ("torch.mm out_dtype fp32", lambda: torch.mm(x, wq.t(), out_dtype=torch.float32)),
             ("tcgen05 gemm_tc", lambda: ext.gemm_tc(y, x, wq, False, True, 0, 1.0)),
             ("addmm fp32 sink deposit", lambda: torch.addmm(acc, dy.t(), x, out_dtype=torch.float32, out=acc)),
             ("deposit on a side stream", deposit_side),
             ("rms_norm_fwd", lambda: ext.rms_norm_fwd(x, ln, 1e-6, False)),
             ("attn_fwd_tc 256 over 768", lambda: ext.attn_fwd_tc(q, kv, kv, 0.088)),
             ("torch.empty", lambda: torch.empty(256, 4096, device="cuda", dtype=torch.bfloat16)))
    for name, fn in cases:
        for _ in range(20):
            fn()
        torch.cuda.synchronize()
        t0 = time.perf_counter()
        for _ in range(200):
            fn()
        t1 = time.perf_counter()
        torch.cuda.synchronize()
        t2 = time.perf_counter()
        print(f"{name:28s}: host {1e6 * (t1 - t0) / 200:7.1f} us/call, device+host {1e6 * (t2 - t0) / 200:7.1f} us/call")


def main(argv=None) -> None:
    ap = argparse.ArgumentParser(description=__doc__.splitlines()[0])
    ap.add_argument("family", choices=["attn", "rms", "lse", "gdn", "conv", "gemm_host", "swiglu", "rope", "dlogits",
                                       "adamw", "fold", "gemm", "gemm_ab", "gemm_one", "packed", "lmhead", "baselines", "lora", "layer_host"])
    ap.add_argument("--mode", choices=["fwd", "bwd"], default="bwd")
    ap.add_argument("--t", type=int, default=2048)
    ap.add_argument("--s", type=int, default=2560)
    ap.add_argument("--hq", type=int, default=16)
    ap.add_argument("--hkv", type=int, default=8)
    ap.add_argument("--d", type=int, default=128)
    ap.add_argument("--h", type=int, default=16)
    ap.add_argument("--rows", type=int, default=16384)
    ap.add_argument("--cols", type=int, default=2048)
    ap.add_argument("--n", type=int, default=4096, help="gemm_one: output columns")
    ap.add_argument("--segs", type=int, default=8, help="packed: segments per pack")
    ap.add_argument("--iters", type=int, default=10)
    ap.add_argument("--rounds", type=int, default=5, help="gemm_ab: interleaved rounds per variant")
    ap.add_argument("--trace", action="store_true", help="lora: per-kernel device times of one forward+backward")
    ap.add_argument("--kernels", action="store_true", help="attn: per-kernel device times of one backward")
    args = ap.parse_args(argv)
    {"attn": bench_attn, "rms": bench_rms, "lse": bench_lse, "gdn": bench_gdn, "conv": bench_conv,
     "gemm_host": bench_gemm_host, "swiglu": bench_swiglu, "rope": bench_rope, "dlogits": bench_dlogits,
     "adamw": bench_adamw, "fold": bench_fold, "gemm": bench_gemm, "gemm_ab": bench_gemm_ab, "gemm_one": bench_gemm_one, "packed": bench_packed,
     "lmhead": bench_lmhead, "baselines": bench_baselines, "lora": bench_lora,
     "layer_host": bench_layer_host}[args.family](args)


if __name__ == "__main__":
    main()
