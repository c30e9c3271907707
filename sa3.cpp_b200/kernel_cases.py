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

    python sa3.cpp_b200/kernel_cases.py mat --type bora [--m 1024 --n 1536 --k 1536 --rank 16]
        [--qtype q8_0] [--reps 3] [--time]

mat runs the forward and backward of a linear with a materialized adapter (W_eff built from the
base and the low-rank update every call); --time prints each launch class with its algorithmic
bytes or FLOPs per call.
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
    o as [B][S][H * 64] f16 (the layout of the fused projection), forward and backward."""
    import torch
    import sa3k
    torch.cuda.set_device(0)
    ctx = sa3k.Context(0)
    g = torch.Generator(device="cuda").manual_seed(0)
    B, H, S = a.b, a.h, a.s
    bf = lambda: torch.randn(B, S, H * 64, generator=g, device="cuda").to(torch.float16)
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


def mat_case(a):
    import torch
    import sa3k
    import gguf_blocks
    torch.cuda.set_device(0)
    ctx = sa3k.Context(0)
    g = torch.Generator().manual_seed(0)
    n, k, m, r = a.n, a.k, a.m, a.rank
    W = torch.randn(n, k, generator=g) * 0.02
    w = ctx.upload(gguf_blocks.encode(W.numpy(), a.qtype), a.qtype, k, n)
    dev = torch.device("cuda", 0)
    t = lambda *shape: torch.randn(*shape, device=dev) * 0.02
    xs = a.type.endswith("-xs")
    fam = a.type[:-3] if xs else a.type
    p = dict(U=t(n, r), V=t(k, r), M=t(r, r)) if xs else dict(A=t(r, k), B=t(n, r))
    grads = dict(dM=torch.empty(r, r, device=dev)) if xs else dict(dA=torch.empty(r, k, device=dev),
                                                                     dB=torch.empty(n, r, device=dev))
    if fam == "dora-rows":
        p["m"], grads["dm"] = torch.ones(n, device=dev), torch.empty(n, device=dev)
    elif fam == "dora-cols":
        p["m"], grads["dm"] = torch.ones(k, device=dev), torch.empty(k, device=dev)
    elif fam == "bora":
        p["m_r"], p["m_c"] = torch.ones(n, device=dev), torch.ones(k, device=dev)
        grads["dm_r"], grads["dm_c"] = torch.empty(n, device=dev), torch.empty(k, device=dev)
    ad = ctx.mat_adapter(a.type, r, 1.0, **p)
    x, dy = torch.randn(m, k, device=dev), torch.randn(m, n, device=dev)
    y, dx = torch.empty(m, n, device=dev), torch.empty(m, k, device=dev)
    run = lambda: ctx.linear_mat_fwd_bwd(w, ad, x, dy, y=y, dx=dx, **grads)
    for _ in range(a.warmup):
        run()
    ctx.sync()
    if a.time:
        ctx.profile_enable(timing=1)
    for _ in range(a.reps):
        run()
    ctx.sync()
    if a.time:
        E = n * k
        code = {"q8_0": 1.0 + 4.0 / 32, "q4_k": 0.5 + 8.0 / 32}[a.qtype]
        work = {"mat.build": (E * (code + 4), "B"), "mat.cols": (E * 4, "B"), "mat.weff": (E * 6, "B"),
                "mat.transpose": (m * n * 4, "B"), "mat.cols_bwd": (E * 8, "B"), "mat.rows_bwd": (E * 10, "B"),
                "mat.dA": (2.0 * E * r, "F"), "mat.dB": (2.0 * E * r, "F"), "mat.fwd": (2.0 * m * n * k, "F"),
                "mat.dx": (2.0 * m * n * k, "F"), "mat.dW": (2.0 * m * n * k, "F")}
        total = 0.0
        print(f"mat {a.type} {a.qtype} tokens {m}, in {k}, out {n}, rank {r}")
        for name, (cnt, ms) in sorted(ctx.profile_read().items()):
            us = ms / a.reps * 1e3
            total += us
            amt, kind = work.get(name, (0, ""))
            rate = (f"{amt * cnt / a.reps / (us * 1e-6) / 1e9:8.0f} GB/s (algorithmic)" if kind == "B" else
                    f"{amt * cnt / a.reps / (us * 1e-6) / 1e12:8.0f} TFLOP/s" if kind == "F" else "")
            print(f"    {name:14s} {cnt // a.reps} launch(es) {us:8.1f} us  {rate}")
        print(f"    total {total:.1f} us per call")
    w.free()
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
    mp = sub.add_parser("mat")
    mp.add_argument("--type", default="bora")
    mp.add_argument("--m", type=int, default=1024)
    mp.add_argument("--n", type=int, default=1536)
    mp.add_argument("--k", type=int, default=1536)
    mp.add_argument("--rank", type=int, default=16)
    mp.add_argument("--qtype", default="q8_0", choices=["q8_0", "q4_k"])
    mp.add_argument("--warmup", type=int, default=2)
    mp.add_argument("--reps", type=int, default=3)
    mp.add_argument("--time", action="store_true")
    a = ap.parse_args()
    if a.case == "gemm":
        gemm_case(a)
    elif a.case == "mat":
        mat_case(a)
    else:
        attention_case(a)


if __name__ == "__main__":
    main()
