"""Contexts on two devices of one process: every large-shared-memory kernel (the GEMM engine on one
CTA and on CTA pairs, the grouped rank-16 GEMMs inside a linear backward, both attention kernel
families) must launch on the second device too, and give the same result as on the first.  The
dynamic shared-memory attribute those kernels need is per device.  Skipped with fewer than 2 GPUs."""
import math

import numpy as np
import pytest

import oracle

pytestmark = pytest.mark.gpu


def _run(dev, raw, IN, OUT, x, dy, A, Bm, q, k, v, dO, attn_tc):
    import torch
    import sa3k
    c = sa3k.Context(dev)
    c.set_option(sa3k.OPT_ATTN_TC, attn_tc)
    with torch.cuda.device(dev):
        w = c.upload(raw, "q8_0", IN, OUT)
        d = lambda a: torch.from_numpy(np.ascontiguousarray(a)).to(f"cuda:{dev}")
        tA, tB = d(A), d(Bm)
        ad = c.adapter(tA, tB, 1.0)
        S = x.shape[0]
        y = torch.empty(S, OUT, device=f"cuda:{dev}")
        dx = torch.empty(S, IN, device=f"cuda:{dev}")
        dA = torch.empty_like(tA)
        dB = torch.empty_like(tB)
        c.linear_fwd_bwd(w, d(x), d(dy), y, dx, ad=ad, dA=dA, dB=dB)
        Bt, H, Sq, _ = q.shape
        qs = (H * Sq * 64, Sq * 64, 64)
        qd, kd, vd, dod = (t.to(f"cuda:{dev}") for t in (q, k, v, dO))
        od = torch.empty_like(qd)
        lse = torch.empty(Bt * H * Sq, device=f"cuda:{dev}")
        T4 = sa3k.t4
        c.attention_fwd(Bt, H, Sq, Sq, 0.125, -1, T4(qd, *qs), T4(kd, *qs), T4(vd, *qs), T4(od, *qs), lse)
        f32 = lambda t: torch.zeros(t.shape, dtype=torch.float32, device=f"cuda:{dev}")
        dq, dk, dv = f32(qd), f32(kd), f32(vd)
        c.attention_bwd(Bt, H, Sq, Sq, 0.125, -1, T4(qd, *qs), T4(kd, *qs), T4(vd, *qs), T4(od, *qs), T4(dod, *qs),
                        lse, T4(dq, *qs), T4(dk, *qs), T4(dv, *qs))
        c.sync()
        out = [t.float().cpu().numpy() for t in (y, dx, dA, dB, od, dq, dk, dv)]
    c.close()
    return out


@pytest.mark.parametrize("attn_tc", [1, 0])
def test_contexts_on_two_devices(attn_tc):
    import torch
    if not torch.cuda.is_available() or torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    import build as sa3k_build
    sa3k_build.build()
    rng = np.random.default_rng(3)
    S, IN, OUT, R = 1024, 1536, 1536, 16
    raw = oracle.quantize(rng.normal(0, 0.02, (OUT, IN)).astype(np.float32), "q8_0")
    x = rng.standard_normal((S, IN)).astype(np.float32)
    dy = rng.standard_normal((S, OUT)).astype(np.float32)
    A = rng.normal(0, 1 / math.sqrt(IN), (R, IN)).astype(np.float32)
    Bm = rng.normal(0, 0.01, (OUT, R)).astype(np.float32)
    g = torch.Generator().manual_seed(4)
    q, k, v, dO = (torch.randn(2, 3, 300, 64, generator=g).to(torch.float16) for _ in range(4))
    r0 = _run(0, raw, IN, OUT, x, dy, A, Bm, q, k, v, dO, attn_tc)
    r1 = _run(1, raw, IN, OUT, x, dy, A, Bm, q, k, v, dO, attn_tc)
    for name, a, b in zip(("y", "dx", "dA", "dB", "o", "dq", "dk", "dv"), r0, r1):
        # same kernels, same order of summation, except the f32 atomics of split-K gradients
        rel = np.linalg.norm(a - b) / max(np.linalg.norm(a), 1e-30)
        assert rel < 1e-5, (name, rel)
