"""GPU parity of attention (nn::sdpa, src/nn.h:135-144, dense / banded / cross) and of the qk
RMSNorm + partial NeoX RoPE head preparation (src/dit.h:195, 209-217; src/nn.h:53-59), forward and
backward, through the C ABI, against float64 torch autograd over the oracle's restatement.

Inputs are rounded to f16 (IEEE half) first (the kernels' operand type), so the comparison isolates the
kernels' own error; tolerance rel-L2 <= 1e-2 (16-bit operands, f32 accumulation)."""
import math

import numpy as np
import pytest

import oracle

pytestmark = pytest.mark.gpu
TOL = 1e-2


@pytest.fixture(autouse=True, params=["tcgen05", "mma_sync"])
def attn_path(request, ctx):
    """Every test runs on both attention kernel families (SA3K_OPT_ATTN_TC)."""
    import sa3k
    ctx.set_option(sa3k.OPT_ATTN_TC, 1 if request.param == "tcgen05" else 0)
    yield request.param
    ctx.set_option(sa3k.OPT_ATTN_TC, 1)


def rel_l2(a, b):
    a = np.asarray(a, np.float64)
    b = np.asarray(b, np.float64)
    return float(np.linalg.norm(a - b) / max(np.linalg.norm(b), 1e-30))


def _ref_attention(q, k, v, dO, scale, window):
    """q/k/v/dO as [B, H, S, 64] float64 torch tensors -> o, dq, dk, dv."""
    import torch
    q = q.clone().requires_grad_(True)
    k = k.clone().requires_grad_(True)
    v = v.clone().requires_grad_(True)
    o = oracle.sdpa(q, k, v, scale, window)
    o.backward(dO)
    return o.detach(), q.grad, k.grad, v.grad


@pytest.mark.parametrize("B,H,Sq,Sk,window,token_major", [
    (2, 3, 200, 200, -1, False),       # dense self-attention, ragged length
    (1, 2, 700, 700, 100, False),      # banded, |i - j| <= 100
    (2, 2, 300, 128, -1, True),        # cross-attention shape (queries != keys), token-major
    (2, 4, 1088, 1088, -1, True),      # the DiT's S = 1024 + 64 memory tokens, token-major
])
def test_attention_fwd_bwd(ctx, B, H, Sq, Sk, window, token_major):
    import torch
    import sa3k
    g = torch.Generator().manual_seed(B * 1000 + Sq)
    bf = lambda *s: torch.randn(*s, generator=g).to(torch.float16)
    q, k, v, dO = bf(B, H, Sq, 64), bf(B, H, Sk, 64), bf(B, H, Sk, 64), bf(B, H, Sq, 64)
    scale = 1.0 / math.sqrt(64)
    ro, rdq, rdk, rdv = _ref_attention(q.double(), k.double(), v.double(), dO.double(), scale,
                                       None if window < 0 else window)

    def dev(t):   # device copy in the requested layout + its strides
        if token_major:
            tm = t.permute(0, 2, 1, 3).contiguous().cuda()          # [B][S][H][64]
            S = t.shape[2]
            return tm, (S * H * 64, 64, H * 64)
        return t.contiguous().cuda(), (t.shape[1] * t.shape[2] * 64, t.shape[2] * 64, 64)

    (qd, qs), (kd, ks), (vd, vs), (dod, ds) = dev(q), dev(k), dev(v), dev(dO)
    od = torch.empty_like(qd)
    lse = torch.empty(B * H * Sq, device="cuda")
    T4 = sa3k.t4
    ctx.attention_fwd(B, H, Sq, Sk, scale, window, T4(qd, *qs), T4(kd, *ks), T4(vd, *vs), T4(od, *qs), lse)
    f32 = lambda t: torch.zeros(t.shape, dtype=torch.float32, device="cuda")
    dq, dk, dv = f32(qd), f32(kd), f32(vd)
    ctx.attention_bwd(B, H, Sq, Sk, scale, window, T4(qd, *qs), T4(kd, *ks), T4(vd, *vs), T4(od, *qs),
                      T4(dod, *ds), lse, T4(dq, *qs), T4(dk, *ks), T4(dv, *vs))
    ctx.sync()

    def back(t):
        t = t.float().cpu()
        return t.permute(0, 2, 1, 3) if token_major else t

    res = {"o": rel_l2(back(od), ro), "dq": rel_l2(back(dq), rdq), "dk": rel_l2(back(dk), rdk),
           "dv": rel_l2(back(dv), rdv)}
    assert all(x < TOL for x in res.values()), res


def test_attention_dq_only_for_frozen_context(ctx):
    import torch
    import sa3k
    B, H, Sq, Sk = 1, 2, 130, 128
    g = torch.Generator().manual_seed(5)
    q, k, v, dO = (torch.randn(B, H, s, 64, generator=g).to(torch.float16) for s in (Sq, Sk, Sk, Sq))
    _, rdq, _, _ = _ref_attention(q.double(), k.double(), v.double(), dO.double(), 0.125, None)
    qs, ks = (H * Sq * 64, Sq * 64, 64), (H * Sk * 64, Sk * 64, 64)
    qd, kd, vd, dod = q.cuda(), k.cuda(), v.cuda(), dO.cuda()
    od = torch.empty_like(qd)
    lse = torch.empty(B * H * Sq, device="cuda")
    dq = torch.zeros(B, H, Sq, 64, device="cuda")
    T4 = sa3k.t4
    ctx.attention_fwd(B, H, Sq, Sk, 0.125, -1, T4(qd, *qs), T4(kd, *ks), T4(vd, *ks), T4(od, *qs), lse)
    ctx.attention_bwd(B, H, Sq, Sk, 0.125, -1, T4(qd, *qs), T4(kd, *ks), T4(vd, *ks), T4(od, *qs), T4(dod, *qs), lse,
                      T4(dq, *qs))
    ctx.sync()
    assert rel_l2(dq.cpu(), rdq) < TOL


@pytest.mark.parametrize("rot", [32, 64])
def test_head_prep_norm_rope_fwd_bwd(ctx, rot):
    """qk RMSNorm (eps 1e-6) + partial NeoX RoPE on the q and k slices of a fused qkv output,
    v copied, forward and backward, with positions restarting per sample."""
    import torch
    import sa3k
    B, S, H = 2, 70, 3
    T, dim = B * S, H * 64
    ncols = 3 * dim
    g = torch.Generator().manual_seed(rot)
    y = torch.randn(T, ncols, generator=g, dtype=torch.float64)
    gq = 1 + 0.1 * torch.randn(64, generator=g, dtype=torch.float64)
    gk = 1 + 0.1 * torch.randn(64, generator=g, dtype=torch.float64)
    up = torch.randn(T, ncols, generator=g, dtype=torch.float64)
    # reference: per sample positions 0..S-1
    yr = y.clone().requires_grad_(True)
    pos = torch.arange(S).repeat(B)
    outs = []
    for i, gamma in ((0, gq), (1, gk)):
        h = yr[:, i * dim:(i + 1) * dim].reshape(T, H, 64)
        h = oracle.rms_norm(h, gamma, 1e-6)
        h = torch.cat([oracle.rope_neox(h[b * S:(b + 1) * S], pos[:S], rot, 10000.0) for b in range(B)], 0)
        outs.append(h.reshape(T, dim))
    outs.append(yr[:, 2 * dim:])
    ref = torch.cat(outs, 1)
    ref.backward(up)

    yd = y.float().cuda()
    out = torch.empty(T, ncols, dtype=torch.float16, device="cuda")
    rq = torch.empty(T, H, device="cuda")
    rk = torch.empty(T, H, device="cuda")
    gqd, gkd = gq.float().cuda(), gk.float().cuda()
    sl = [sa3k.HeadSliceC(0, gqd.data_ptr(), 1, rq.data_ptr()), sa3k.HeadSliceC(dim, gkd.data_ptr(), 1, rk.data_ptr()),
          sa3k.HeadSliceC(2 * dim, None, 0, None)]
    ctx.head_prep_fwd(yd, T, ncols, H, sl, S, 1e-6, rot, 10000.0, out)
    gup = up.float().cuda()
    dy = torch.empty(T, ncols, device="cuda")
    for j, s in enumerate(sl):
        ctx.head_prep_bwd(gup[:, j * dim:], ncols, yd, T, ncols, H, s, S, rot, 10000.0, dy)
    ctx.sync()
    assert rel_l2(out.float().cpu(), ref.detach()) < TOL
    assert rel_l2(dy.cpu(), yr.grad) < 1e-4


def test_config3_banded_rope_attention(ctx):
    """batch 2, 24 heads, head_dim 64, 2048 frames, window +-256, NeoX RoPE on
    q and k (rot 32, base 1e4), f16 N(0,1) inputs.  The full problem runs on the GPU; two heads
    are checked against float64 autograd (the oracle cost grows with S^2)."""
    import torch
    import sa3k
    B, H, S, W = 2, 24, 2048, 256
    dim = H * 64
    g = torch.Generator().manual_seed(3)
    qkv = torch.randn(B * S, 3 * dim, generator=g).to(torch.float16).float()
    dO = torch.randn(B, S, dim, generator=g).to(torch.float16)
    yd = qkv.cuda()
    prep = torch.empty(B * S, 3 * dim, dtype=torch.float16, device="cuda")
    sl = [sa3k.HeadSliceC(0, None, 1, None), sa3k.HeadSliceC(dim, None, 1, None), sa3k.HeadSliceC(2 * dim, None, 0, None)]
    ctx.head_prep_fwd(yd, B * S, 3 * dim, H, sl, S, 1e-6, 32, 10000.0, prep)
    T4 = sa3k.t4
    st = (S * 3 * dim, 64, 3 * dim)
    so = (S * dim, 64, dim)
    q, k, v = prep, prep[:, dim:], prep[:, 2 * dim:]
    o = torch.empty(B * S, dim, dtype=torch.float16, device="cuda")
    lse = torch.empty(B * H * S, device="cuda")
    ctx.attention_fwd(B, H, S, S, 0.125, W, T4(q, *st), T4(k, *st), T4(v, *st), T4(o, *so), lse)
    d3 = torch.zeros(B * S, 3 * dim, device="cuda")
    dod = dO.reshape(B * S, dim).cuda()
    ctx.attention_bwd(B, H, S, S, 0.125, W, T4(q, *st), T4(k, *st), T4(v, *st), T4(o, *so), T4(dod, *so), lse,
                      T4(d3, *st), T4(d3[:, dim:], *st), T4(d3[:, 2 * dim:], *st))
    dqkv = torch.empty_like(d3)
    for j, s in enumerate(sl):
        ctx.head_prep_bwd(d3[:, j * dim:], 3 * dim, yd, B * S, 3 * dim, H, s, S, 32, 10000.0, dqkv)
    ctx.sync()
    # float64 reference for heads 0 and 17 of both samples
    heads = [0, 17]
    x = qkv.double().reshape(B, S, 3, H, 64)[:, :, :, heads]              # [B, S, 3, h, 64]
    x = x.clone().requires_grad_(True)
    pos = torch.arange(S)
    qh = torch.stack([oracle.rope_neox(x[b, :, 0], pos, 32, 10000.0) for b in range(B)])   # [B, S, h, 64]
    kh = torch.stack([oracle.rope_neox(x[b, :, 1], pos, 32, 10000.0) for b in range(B)])
    vh = x[:, :, 2]
    tr = lambda t: t.permute(0, 2, 1, 3)
    # the kernel consumes the f16-rounded roped q / k; round the reference the same way
    # (straight-through: the rounded value forward, the identity backward)
    qr = tr(qh).detach().to(torch.float16).double() + (tr(qh) - tr(qh).detach())
    kr = tr(kh).detach().to(torch.float16).double() + (tr(kh) - tr(kh).detach())
    ref_o = oracle.sdpa(qr, kr, tr(vh), 0.125, W)
    dOr = dO.double().reshape(B, S, H, 64)[:, :, heads].permute(0, 2, 1, 3)
    ref_o.backward(dOr)
    got_o = o.float().cpu().reshape(B, S, H, 64)[:, :, heads].permute(0, 2, 1, 3)
    got_d = dqkv.cpu().reshape(B, S, 3, H, 64)[:, :, :, heads]
    assert rel_l2(got_o, ref_o.detach()) < TOL
    assert rel_l2(got_d, x.grad) < TOL


def test_config3_cross_attention_through_kv_projection(ctx):
    """BASELINE config 3's cross-attention: 2 x 2048 queries (24 heads x 64) attend to 128
    conditioning tokens of width 768 through frozen K / V projections (one Q8_0 [2 x 1536][768]
    weight, the DiT's cross.kv layout) run on the library's own GEMM; the backward goes through the
    attention to dK / dV and on through the projection to d(conditioning).  Every head is checked
    against float64 autograd of the same chain on the dequantized weight."""
    import torch
    import sa3k
    import gguf_blocks
    B, H, S, C, CD = 2, 24, 2048, 128, 768
    D = H * 64
    rng = np.random.default_rng(31)
    W = rng.normal(0, 0.02, (2 * D, CD)).astype(np.float32)
    raw = gguf_blocks.encode(W, "q8_0")
    Wd = oracle.dequantize(raw, "q8_0", 2 * D, CD)
    cond = rng.standard_normal((B * C, CD)).astype(np.float32)
    g = torch.Generator().manual_seed(32)
    q = torch.randn(B * S, D, generator=g).to(torch.float16)
    dO = torch.randn(B * S, D, generator=g).to(torch.float16)
    w = ctx.upload(raw, "q8_0", CD, 2 * D)
    condd = torch.from_numpy(cond).cuda()
    kv = torch.empty(B * C, 2 * D, device="cuda")
    ctx.linear_fwd(w, condd, kv)
    kvh = torch.empty(B * C, 2 * D, dtype=torch.float16, device="cuda")
    sl = [sa3k.HeadSliceC(0, None, 0, None), sa3k.HeadSliceC(D, None, 0, None)]
    ctx.head_prep_fwd(kv, B * C, 2 * D, H, sl, C, 1e-6, 0, 10000.0, kvh)
    T4 = sa3k.t4
    sq, skv = (S * D, 64, D), (C * 2 * D, 64, 2 * D)
    qd, dod = q.cuda(), dO.cuda()
    o = torch.empty(B * S, D, dtype=torch.float16, device="cuda")
    lse = torch.empty(B * H * S, device="cuda")
    ctx.attention_fwd(B, H, S, C, 0.125, -1, T4(qd, *sq), T4(kvh, *skv), T4(kvh[:, D:], *skv), T4(o, *sq), lse)
    dq = torch.zeros(B * S, D, device="cuda")
    dkv = torch.zeros(B * C, 2 * D, device="cuda")
    ctx.attention_bwd(B, H, S, C, 0.125, -1, T4(qd, *sq), T4(kvh, *skv), T4(kvh[:, D:], *skv), T4(o, *sq),
                      T4(dod, *sq), lse, T4(dq, *sq), T4(dkv, *skv), T4(dkv[:, D:], *skv))
    dcond = torch.empty(B * C, CD, device="cuda")
    ctx.linear_bwd(w, condd, kv, dkv, dcond)
    ctx.sync()

    Wt = torch.tensor(Wd, dtype=torch.float64)
    ct = torch.tensor(cond, dtype=torch.float64).requires_grad_(True)
    kvr = ct @ Wt.t()
    qr = q.double().reshape(B, S, H, 64).permute(0, 2, 1, 3).requires_grad_(True)
    kr = kvr[:, :D].reshape(B, C, H, 64).permute(0, 2, 1, 3)
    vr = kvr[:, D:].reshape(B, C, H, 64).permute(0, 2, 1, 3)
    ref_o = oracle.sdpa(qr, kr, vr, 0.125)
    kvr.retain_grad()
    ref_o.backward(dO.double().reshape(B, S, H, 64).permute(0, 2, 1, 3))
    back = lambda t: t.permute(0, 2, 1, 3).reshape(B * S, D)
    res = {"kv": rel_l2(kv.cpu(), kvr.detach()), "o": rel_l2(o.float().cpu(), back(ref_o.detach())),
           "dq": rel_l2(dq.cpu(), back(qr.grad)), "dkv": rel_l2(dkv.cpu(), kvr.grad),
           "dcond": rel_l2(dcond.cpu(), ct.grad)}
    assert all(v < TOL for v in res.values()), res
