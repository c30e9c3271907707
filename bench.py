"""Benchmark of the sa3.cpp adapter-training hot path on B200.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl sa3k|reference]

One step = one training step of the BASELINE workload on every rank: forward + backward of the
frozen-base adapted linear over one sample, the NCCL gradient all-reduce across ranks
(data parallel, one sample per rank), then the averaged + clipped AdamW update of the adapter
(the reference's train_apply_accumulated_adamw, src/train_loop.h:173-211).

Workload: DoRA rank 16 / alpha 16 on the MLP up-projection
1536 -> 6144 with a Q4_K base (N(0, 0.02)), 2048 tokens per sample, X and dY ~ N(0, 1), seeded
synthetic data (no dataset is involved).  The unit is samples/s summed over all ranks.

Reported beside the device-timed value:
  roofline      the two quant-GEMM kernels (forward Y and backward dX), algorithmic FLOPs / their
                summed CUDA-event time in a timed pass, against the measured bf16 peak
  e2e           the same step through the C ABI with the inputs copied from pinned host memory and
                the output read back every step
  cpu_baseline  the CPU restatement (oracle, float32 numpy/BLAS on all host threads)
  clocks        nvidia-smi samples taken during the timed region
Rank 0 prints one JSON line.
"""
import argparse
import json
import os
import statistics
import subprocess
import sys
import time

import numpy as np

REPO = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.join(REPO, "sa3.cpp_b200"))

METRIC = "DoRA train samples/s at 1/2/4/8 B200; quant-GEMM fwd+bwd % of roofline"
S, IN, OUT, RANK, ALPHA, QTYPE = 2048, 1536, 6144, 16, 16.0, "q4_k"
WORKLOAD = ("config2: DoRA r16/a16 on a Q4_K 1536->6144 linear, 2048 tokens/sample; "
            "fwd + bwd (Y, dX, dA, dB, dm) + NCCL grad all-reduce + clipped AdamW per step")


def load_peaks():
    p = os.path.join(REPO, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        d = json.load(open(p))
        return d["bf16_tflops"], d["hbm_gbs"], "measured"
    return 1590.0, 6650.0, "fallback"


def synth(seed):
    """Seeded synthetic weights and sample for one rank (float32 numpy)."""
    rng = np.random.default_rng(seed)
    W = rng.normal(0, 0.02, (OUT, IN)).astype(np.float32)
    A = rng.normal(0, 1 / np.sqrt(IN), (RANK, IN)).astype(np.float32)
    B = rng.normal(0, 0.01, (OUT, RANK)).astype(np.float32)
    bias = rng.normal(0, 0.02, OUT).astype(np.float32)
    x = rng.normal(0, 1, (S, IN)).astype(np.float32)
    dy = rng.normal(0, 1, (S, OUT)).astype(np.float32)
    return W, A, B, bias, x, dy


class Clocks:
    """nvidia-smi sampling during the timed region."""

    def __init__(self, index):
        self.index = index
        self.proc = None
        self.path = os.path.join(REPO, "gpurun_out", f"clocks_{index}.csv")

    def __enter__(self):
        os.makedirs(os.path.dirname(self.path), exist_ok=True)
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", "-i", str(self.index), "--query-gpu=clocks.sm,clocks.max.sm,power.draw,"
                 "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
                 "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap",
                 "--format=csv,noheader,nounits", "-lms", "100"],
                stdout=open(self.path, "w"), stderr=subprocess.DEVNULL)
        except OSError:
            self.proc = None
        time.sleep(0.3)
        return self

    def __exit__(self, *a):
        if self.proc:
            self.proc.terminate()
            self.proc.wait()

    def summary(self):
        try:
            rows = [r.split(",") for r in open(self.path).read().strip().splitlines()]
        except OSError:
            return None
        rows = [[c.strip() for c in r] for r in rows if len(r) >= 7]
        if not rows:
            return None
        sm = [float(r[0]) for r in rows if r[0].replace(".", "").isdigit()]
        mx = max(float(r[1]) for r in rows)
        load = [v for v in sm if v > 0.5 * mx] or sm
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({names[i] for r in rows for i in range(4) if r[3 + i].lower() == "active"})
        return {"sm_mhz": statistics.median(load) if load else None, "sm_max_mhz": mx,
                "reasons": reasons, "samples": len(rows)}


def _oracle():
    """The CPU oracle (test infrastructure): only the cpu_baseline / reference legs use it."""
    path = os.path.join(REPO, "oracle")
    if path not in sys.path:
        sys.path.insert(0, path)
    import oracle
    return oracle


def cpu_reference_step(W, A, B, bias, x, dy, m, bns, p, mom, vel, step):
    """One step of the CPU restatement: float32 forward + backward + AdamW (oracle)."""
    oracle = _oracle()
    y, cache = oracle.dit_lin_fwd(x, W, A, B, ALPHA / RANK, m, bns, bias, dtype=np.float32)
    g = oracle.dit_lin_bwd(dy, cache)
    grad = np.concatenate([g["dA"].ravel(), g["dB"].ravel(), g["dm"].ravel()]).astype(np.float32)
    oracle.average_and_clip([grad], 1, 1.0)
    oracle.adamw_f32(p, grad, mom, vel, 1e-4, 0.9, 0.999, 1e-8, 0.01, step)
    return y


def cpu_baseline(seed, budget_s=15.0, max_reps=5):
    """Time the CPU restatement on the full sample, repeated within a bounded budget."""
    oracle = _oracle()
    W, A, B, bias, x, dy = synth(seed)
    Wd = oracle.dequantize(oracle.quantize(W, QTYPE), QTYPE, OUT, IN)
    bns, nrm = oracle.row_norms(Wd)
    m = nrm.copy()
    n = A.size + B.size + m.size
    p = np.concatenate([A.ravel(), B.ravel(), m]).astype(np.float32)
    mom = np.zeros(n, np.float32)
    vel = np.zeros(n, np.float32)
    cpu_reference_step(Wd, A, B, bias, x, dy, m, bns, p, mom, vel, 1)   # warm-up
    times = []
    t_start = time.perf_counter()
    for rep in range(max_reps):
        t0 = time.perf_counter()
        cpu_reference_step(Wd, A, B, bias, x, dy, m, bns, p, mom, vel, rep + 2)
        times.append(time.perf_counter() - t0)
        if time.perf_counter() - t_start > budget_s:
            break
    t = statistics.median(times)
    return {"value": 1.0 / t, "unit": "samples/s", "cores": os.cpu_count(), "kind": "port",
            "sample": f"full 2048-token sample, {len(times)} timed reps (median), float32 numpy/BLAS "
                      f"restatement of dit_lin fwd+bwd + AdamW (ggml, which holds the reference's CPU "
                      f"kernels, is not available)"}


def run_reference(args):
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return 0
    oracle = _oracle()
    W, A, B, bias, x, dy = synth(1000)
    Wd = oracle.dequantize(oracle.quantize(W, QTYPE), QTYPE, OUT, IN)
    bns, nrm = oracle.row_norms(Wd)
    m = nrm.copy()
    n = A.size + B.size + m.size
    p = np.concatenate([A.ravel(), B.ravel(), m]).astype(np.float32)
    mom = np.zeros(n, np.float32)
    vel = np.zeros(n, np.float32)
    for i in range(args.warmup):
        cpu_reference_step(Wd, A, B, bias, x, dy, m, bns, p, mom, vel, i + 1)
    t0 = time.perf_counter()
    for i in range(args.steps):
        cpu_reference_step(Wd, A, B, bias, x, dy, m, bns, p, mom, vel, args.warmup + i + 1)
    dt = time.perf_counter() - t0
    value = args.steps / dt
    line = {"impl": "reference", "metric": METRIC, "value": value, "unit": "samples/s", "n_gpus": args.gpus,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": 1000 * dt / args.steps,
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32",
            "data": "synthetic", "config": {"workload": WORKLOAD, "global_batch": 1, "seq_len": S,
                                            "parallelism": "cpu"},
            "cpu_baseline": {"value": value, "unit": "samples/s", "cores": os.cpu_count(), "kind": "port",
                             "sample": "full 2048-token sample per step, float32 numpy/BLAS restatement "
                                       "(ggml, which holds the reference's CPU kernels, is absent)"},
            "e2e": {"value": value, "unit": "samples/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)
    return 0


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=50)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", default="sa3k", choices=["sa3k", "reference"])
    ap.add_argument("--no-cpu-baseline", action="store_true")
    args = ap.parse_args()
    args.warmup = max(args.warmup, 3)
    if args.impl == "reference":
        return run_reference(args)

    import torch
    import torch.distributed as dist
    import sa3k
    import gguf_blocks

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    if world > 1:
        from datetime import timedelta
        dist.init_process_group("nccl", timeout=timedelta(seconds=120), device_id=torch.device("cuda", local))
    dev = torch.device("cuda", local)

    ctx = sa3k.Context(local)
    W, A, B, bias, x_h, dy_h = synth(1000 + rank)
    w = ctx.upload(gguf_blocks.encode(W, QTYPE), QTYPE, IN, OUT)
    bns = torch.empty(OUT, device=dev)
    nrm = torch.empty(OUT, device=dev)
    ctx.row_norms(w, 1e-12, bns, nrm)                       # DoRA constants + magnitude init
    # flat adapter state: [A | B | m]
    n_a, n_b = RANK * IN, OUT * RANK
    n = n_a + n_b + OUT
    p = torch.empty(n, device=dev)
    p[:n_a].copy_(torch.from_numpy(A.ravel()))
    p[n_a:n_a + n_b].copy_(torch.from_numpy(B.ravel()))
    p[n_a + n_b:].copy_(nrm)
    if world > 1:
        dist.broadcast(p, 0)                                 # identical adapters on every rank
    grad = torch.zeros(n, device=dev)
    mom = torch.zeros(n, device=dev)
    vel = torch.zeros(n, device=dev)
    pA, pB, pm = p[:n_a].view(RANK, IN), p[n_a:n_a + n_b].view(OUT, RANK), p[n_a + n_b:]
    gA, gB, gm = grad[:n_a].view(RANK, IN), grad[n_a:n_a + n_b].view(OUT, RANK), grad[n_a + n_b:]
    ad = ctx.adapter(pA, pB, ALPHA / RANK, pm, bns)
    bias_d = torch.from_numpy(bias).to(dev)
    x = torch.from_numpy(x_h).to(dev)
    dy = torch.from_numpy(dy_h).to(dev)
    y = torch.empty(S, OUT, device=dev)
    dx = torch.empty(S, IN, device=dev)
    hp = sa3k.AdamWParams(1e-4, 0.9, 0.999, 1e-8, 0.01, 1.0)
    flush = torch.empty(256 * 1024 * 1024 // 4, device=dev)          # 256 MB > 126 MB L2
    state = {"step": 0}

    def fwd_bwd():
        ctx.linear_fwd_bwd(w, x, dy, y, dx, ad=ad, bias=bias_d, dA=gA, dB=gB, dm=gm)
        if world > 1:
            dist.all_reduce(grad)

    def adam():
        # eager: the bias corrections are computed on the host per step (the reference's powf)
        state["step"] += 1
        ctx.average_clip_adamw(p, grad, mom, vel, world, hp, state["step"])

    def step():
        fwd_bwd()
        adam()

    def capture(timing):
        """CUDA graph of the forward + backward (+ all-reduce) of one step."""
        ctx.profile_enable(timing=timing)
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g):
            ctx.set_stream(torch.cuda.current_stream().cuda_stream)
            fwd_bwd()
        ctx.set_stream(torch.cuda.current_stream().cuda_stream)
        return g

    def timed(fn, k, per_step=None):
        """Per-step CUDA events with an L2 flush between steps; returns summed ms (max over ranks)."""
        evs = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(k)]
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize()
        for e0, e1 in evs:
            flush.zero_()
            e0.record()
            fn()
            e1.record()
            if per_step:
                per_step()
        torch.cuda.synchronize()
        if world > 1:
            dist.barrier()
        total = sum(e0.elapsed_time(e1) for e0, e1 in evs)
        t = torch.tensor([total], device=dev, dtype=torch.float64)
        if world > 1:
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    for _ in range(args.warmup):
        step()                                   # eager warm-up: sizes scratch, sets attributes
    ctx.sync()

    # ---- pass 1: the headline device-timed value; the step replays a CUDA graph
    graph = capture(0)
    launches_graph = sum(v[0] for v in ctx.profile_read().values())

    def graph_step():
        graph.replay()
        adam()

    for _ in range(3):
        graph_step()
    ctx.profile_enable(timing=0)
    with Clocks(local) as clk:
        total_ms = timed(graph_step, args.steps)
    launches = launches_graph * args.steps + sum(v[0] for v in ctx.profile_read().values())
    value = world * args.steps / (total_ms / 1000.0)

    # ---- pass 2: per-kernel CUDA events captured in the graph -> roofline of the GEMMs
    peak_tf, peak_hbm, peak_kind = load_peaks()
    gemm_flops = 2.0 * S * IN * OUT                         # per launch (fwd and dX alike)

    def gemm_roofline(smem_dequant):
        ctx.set_option(sa3k.OPT_SMEM_DEQUANT, 1 if smem_dequant else 0)
        g = capture(2)
        acc = {}
        for _ in range(args.steps):
            flush.zero_()
            g.replay()
            for k, (n_l, ms) in ctx.profile_read().items():
                a = acc.setdefault(k, [0, 0.0])
                a[0] += n_l
                a[1] += ms
        ctx.profile_enable(timing=0)
        ctx.set_option(sa3k.OPT_SMEM_DEQUANT, 0)
        del g
        n_g = acc["linear.fwd"][0] + acc["linear.dx"][0]
        ms_g = acc["linear.fwd"][1] + acc["linear.dx"][1]
        return acc, n_g, ms_g, gemm_flops * n_g / (ms_g / 1000.0) / 1e12

    prof, n_gemm, ms_gemm, achieved = gemm_roofline(False)
    prof_q, n_q, ms_q, achieved_q = gemm_roofline(True)
    traffic = None
    tf = os.path.join(REPO, "profiles", "traffic.json")
    if os.path.exists(tf):
        traffic = json.load(open(tf)).get("config2_quant_gemm_bytes_per_launch")

    # ---- pass 3: e2e through the C ABI with host buffers (pinned) copied every step
    x_pin = torch.from_numpy(x_h).pin_memory()
    dy_pin = torch.from_numpy(dy_h).pin_memory()
    y_pin = torch.empty(S, OUT, pin_memory=True)

    def e2e_step():
        x.copy_(x_pin, non_blocking=True)
        dy.copy_(dy_pin, non_blocking=True)
        graph_step()
        y_pin.copy_(y, non_blocking=True)

    e2e_ms = timed(e2e_step, args.steps)
    e2e_val = world * args.steps / (e2e_ms / 1000.0)
    ctx.sync()
    del graph

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        cpu = cpu_baseline(2000)

    if rank == 0:
        line = {
            "metric": METRIC, "value": value, "unit": "samples/s", "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": total_ms / args.steps, "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": "bf16", "data": "synthetic",
            "config": {"workload": WORKLOAD, "global_batch": world, "seq_len": S, "parallelism": f"dp{world}",
                       "l2": "256 MB flush between timed steps"},
            "roofline": {"bound": "tensor", "achieved": achieved, "peak": peak_tf, "unit": "TFLOP/s",
                         "frac": achieved / peak_tf, "traffic": traffic,
                         "kernel": "linear.fwd + linear.dx: tcgen05 GEMM on the bf16 copy of the Q4_K "
                                   "base (dequantized once, bit-exact, at upload)",
                         "peak_kind": f"{peak_kind} bf16 burst", "launches": n_gemm,
                         "kernel_ms_per_step": ms_gemm / args.steps},
            "quant_gemm_smem_dequant": {
                "bound": "tensor", "achieved": achieved_q, "peak": peak_tf, "unit": "TFLOP/s",
                "frac": achieved_q / peak_tf,
                "kernel": "linear.fwd + linear.dx with TMA-loaded Q4_K codes dequantized in shared memory",
                "kernel_ms_per_step": ms_q / args.steps,
                "kernels": {k: {"launches": v[0], "ms": round(v[1], 4)} for k, v in sorted(prof_q.items())}},
            "cpu_baseline": cpu,
            "e2e": {"value": e2e_val, "unit": "samples/s",
                    "h2d_bytes_per_step": x_h.nbytes + dy_h.nbytes, "d2h_bytes_per_step": S * OUT * 4},
            "gpu_launches": launches,
            "clocks": clk.summary(),
            "kernels": {k: {"launches": v[0], "ms": round(v[1], 4)} for k, v in sorted(prof.items())},
            "graph": "fwd+bwd (+all-reduce) replayed from a CUDA graph; AdamW launched eagerly per step",
        }
        print(json.dumps(line), flush=True)
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()
    return 0


if __name__ == "__main__":
    sys.exit(main())
