"""Single-kernel cases for profiling and tuning: one frozen-base linear of a chosen shape, or one
attention of the DiT step's shape, run a few times through the C ABI, so that a profiler
(ncu -k regex:gemm_tc -c 1) sees a handful of launches of one kernel on a few hundred MB.

    python sa3.cpp_b200/kernel_cases.py gemm --m 4352 --n 1536 --k 1536 [--dx] [--qtype q8_0]
        [--pair 0|1|2] [--tile-n 0|128|192|256] [--adapter] [--smem-dequant] [--reps 3] [--time]

--dx runs the input-gradient GEMM dx[m][k] = dy[m][n] . W[n][k] of a linear with in = k,
out = n (the weight is used transposed); the default is the forward y = x W^T + 0.
--adapter adds a rank-16 LoRA adapter (the forward then also runs u = x A^T).
--smem-dequant reads a quantized base as its codes, dequantized in shared memory.

    python sa3.cpp_b200/kernel_cases.py attention [--b 4 --h 24 --s 1088 --window -1] [--fwd-only]
--time prints the CUDA-event time per launch (not to be used under a profiler)."""
import argparse
import os
import sys

sys.path.insert(0, os.path.dirname(os.path.abspath(__file__)))


def gemm_case(a):
    import numpy as np
    import torch
    import sa3k
    import gguf_blocks
    torch.cuda.set_device(0)
    ctx = sa3k.Context(0)
    ctx.set_option(sa3k.OPT_GEMM_PAIR, a.pair)
    ctx.set_option(sa3k.OPT_GEMM_TILE_N, a.tile_n)
    ctx.set_option(sa3k.OPT_SMEM_DEQUANT, 1 if a.smem_dequant else 0)
    g = torch.Generator().manual_seed(0)
    W = torch.randn(a.n, a.k, generator=g) * 0.02                 # [out = n][in = k]
    if a.qtype == "f32":
        w = ctx.upload(W.numpy().view(np.uint8).reshape(a.n, -1), "f32", a.k, a.n)
    else:
        w = ctx.upload(gguf_blocks.encode(W.numpy(), a.qtype), a.qtype, a.k, a.n)
    dev = torch.device("cuda", 0)
    x = torch.randn(a.m, a.k, device=dev)
    y = torch.empty(a.m, a.n, device=dev)
    ad = None
    if a.adapter:
        A = torch.randn(16, a.k, device=dev) * 0.02
        Bm = torch.randn(a.n, 16, device=dev) * 0.02
        ad = ctx.adapter(A, Bm, 1.0)
    if a.dx:
        dy = torch.randn(a.m, a.n, device=dev)
        dx = torch.empty(a.m, a.k, device=dev)
        gA = torch.zeros(16, a.k, device=dev) if ad else None
        gB = torch.zeros(a.n, 16, device=dev) if ad else None
        run = lambda: ctx.linear_bwd(w, x, y, dy, dx, ad=ad, dA=gA, dB=gB)
        flops = 2.0 * a.m * a.n * a.k
    else:
        run = lambda: ctx.linear_fwd(w, x, y, ad=ad)
        flops = 2.0 * a.m * a.n * a.k
    for _ in range(a.warmup):
        run()
    ctx.sync()
    if a.time:
        ctx.profile_enable(timing=1)
    for _ in range(a.reps):
        run()
    ctx.sync()
    if a.time:
        pr = ctx.profile_read()
        name = "linear.dx" if a.dx else "linear.fwd"
        n, ms = pr[name]
        print(f"{'dx' if a.dx else 'fwd'} {a.m}x{a.n}x{a.k} {a.qtype} pair{a.pair} bn{a.tile_n}: "
              f"{ms / n * 1e3:.1f} us/launch, {flops * n / (ms / 1e3) / 1e12:.1f} TFLOP/s")
        for other, (n2, ms2) in sorted(pr.items()):
            if other != name:
                print(f"    {other}: {n2 // a.reps} launch(es) per call, {ms2 / a.reps * 1e3:.1f} us per call")
    w.free()
    ctx.close()


def attention_case(a):
    """Self-attention of the DiT step: B x H heads of Sq = Sk tokens, head_dim 64, q / k / v /
    o as [B][S][H * 64] bf16 (the layout of the fused projection), forward and backward."""
    import torch
    import sa3k
    torch.cuda.set_device(0)
    ctx = sa3k.Context(0)
    g = torch.Generator(device="cuda").manual_seed(0)
    B, H, S = a.b, a.h, a.s
    bf = lambda: torch.randn(B, S, H * 64, generator=g, device="cuda").to(torch.bfloat16)
    q, k, v, dO = bf(), bf(), bf(), bf()
    o = torch.empty_like(q)
    dq, dk, dv = (torch.empty(B, S, H * 64, device="cuda") for _ in range(3))
    lse = torch.empty(B * H * S, device="cuda")
    st = (S * H * 64, 64, H * 64)
    T4 = sa3k.t4
    fwd = lambda: ctx.attention_fwd(B, H, S, S, 0.125, a.window, T4(q, *st), T4(k, *st), T4(v, *st), T4(o, *st), lse)
    bwd = lambda: ctx.attention_bwd(B, H, S, S, 0.125, a.window, T4(q, *st), T4(k, *st), T4(v, *st), T4(o, *st),
                                    T4(dO, *st), lse, T4(dq, *st), T4(dk, *st), T4(dv, *st))
    for _ in range(a.warmup):
        fwd()
        bwd()
    ctx.sync()
    if a.time:
        ctx.profile_enable(timing=1)
    for _ in range(a.reps):
        fwd()
        if not a.fwd_only:
            bwd()
    ctx.sync()
    if a.time:
        for name, (n, ms) in sorted(ctx.profile_read().items()):
            print(f"attention B{B} H{H} S{S} window {a.window}: {name} {ms / n * 1e3:.1f} us/launch")
    ctx.close()


def main():
    ap = argparse.ArgumentParser()
    sub = ap.add_subparsers(dest="case", required=True)
    gp = sub.add_parser("gemm")
    gp.add_argument("--m", type=int, default=4352)
    gp.add_argument("--n", type=int, default=1536)
    gp.add_argument("--k", type=int, default=1536)
    gp.add_argument("--dx", action="store_true")
    gp.add_argument("--qtype", default="f32", choices=["f32", "q8_0", "q4_k"])
    gp.add_argument("--pair", type=int, default=1)
    gp.add_argument("--tile-n", type=int, default=0)
    gp.add_argument("--adapter", action="store_true")
    gp.add_argument("--smem-dequant", action="store_true")
    gp.add_argument("--warmup", type=int, default=2)
    gp.add_argument("--reps", type=int, default=3)
    gp.add_argument("--time", action="store_true")
    at = sub.add_parser("attention")
    at.add_argument("--b", type=int, default=4)
    at.add_argument("--h", type=int, default=24)
    at.add_argument("--s", type=int, default=1088)
    at.add_argument("--window", type=int, default=-1)
    at.add_argument("--fwd-only", action="store_true")
    at.add_argument("--warmup", type=int, default=2)
    at.add_argument("--reps", type=int, default=3)
    at.add_argument("--time", action="store_true")
    a = ap.parse_args()
    if a.case == "gemm":
        gemm_case(a)
    else:
        attention_case(a)


if __name__ == "__main__":
    main()
