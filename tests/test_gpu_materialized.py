"""GPU parity of the materialized adapter families (src/train_lora.h:275-329; the trainer's path
for dora-cols, bora and the -xs families, src/train_dit.h:90-164) through the C ABI, against the
float64 oracle on the same dequantized base.  The effective weight is f32 end to end (rel-L2
1e-5); outputs and gradients pass through bf16 GEMM operands (W_eff, x, dy), so they take the
bf16 bar, rel-L2 <= 1e-2."""
import numpy as np
import pytest

import oracle

pytestmark = pytest.mark.gpu
TOL = 1e-2
TYPES = ["lora", "dora-rows", "dora-cols", "bora", "lora-xs", "dora-rows-xs", "dora-cols-xs", "bora-xs"]


def rel_l2(a, b):
    a = np.asarray(a, np.float64)
    b = np.asarray(b, np.float64)
    return float(np.linalg.norm(a - b) / max(np.linalg.norm(b), 1e-30))


def _dev(a):
    import torch
    return torch.from_numpy(np.ascontiguousarray(a, np.float32)).cuda()


def _case(adapter_type, qtype, S, inn, out, r, seed):
    """Parameters as a trained adapter has them: A ~ U(+-1/sqrt(in)), B and M non-zero, magnitudes
    near the base's row / column norms (their init, src/train_lora.h:262-269)."""
    rng = np.random.default_rng(seed)
    W = rng.normal(0, 0.02, (out, inn)).astype(np.float32)
    raw = oracle.quantize(W, qtype)
    Wd = oracle.dequantize(raw, qtype, out, inn)
    fam, xs = oracle.split_adapter_type(adapter_type)
    p = {}
    if xs:
        p["U"] = np.linalg.qr(rng.normal(size=(out, r)))[0].astype(np.float32)
        p["V"] = np.linalg.qr(rng.normal(size=(inn, r)))[0].astype(np.float32)
        p["M"] = rng.normal(0, 0.05, (r, r)).astype(np.float32)
    else:
        b = 1 / np.sqrt(inn)
        p["A"] = rng.uniform(-b, b, (r, inn)).astype(np.float32)
        p["B"] = rng.normal(0, 0.02, (out, r)).astype(np.float32)
    rn = np.sqrt((Wd.astype(np.float64) ** 2).sum(1))
    cn = np.sqrt((Wd.astype(np.float64) ** 2).sum(0))
    if fam == "dora-rows":
        p["m"] = (rn * rng.uniform(0.9, 1.1, out)).astype(np.float32)
    elif fam == "dora-cols":
        p["m"] = (cn * rng.uniform(0.9, 1.1, inn)).astype(np.float32)
    elif fam == "bora":
        p["m_r"] = (rn * rng.uniform(0.9, 1.1, out)).astype(np.float32)
        p["m_c"] = (cn * rng.uniform(0.9, 1.1, inn)).astype(np.float32)
    x = rng.normal(0, 1, (S, inn)).astype(np.float32)
    dy = rng.normal(0, 1, (S, out)).astype(np.float32)
    bias = rng.normal(0, 0.1, out).astype(np.float32)
    return dict(raw=raw, Wd=Wd, p=p, x=x, dy=dy, bias=bias)


def _adapter(ctx, adapter_type, r, s, dp):
    return ctx.mat_adapter(adapter_type, r, s, **dp)


@pytest.mark.parametrize("adapter_type", TYPES)
def test_effective_weight_matches_oracle(ctx, adapter_type):
    import torch
    c = _case(adapter_type, "q8_0", 1, 512, 384, 8, 3)
    s = 2.0
    w = ctx.upload(c["raw"], "q8_0", 512, 384)
    dp = {k: _dev(v) for k, v in c["p"].items()}
    weff = torch.empty(384, 512, device="cuda")
    ctx.mat_effective_weight(w, _adapter(ctx, adapter_type, 8, s, dp), weff)
    ctx.sync()
    ref, _ = oracle.mat_effective_weight(c["Wd"], c["p"], adapter_type, s)
    assert rel_l2(weff.cpu().numpy(), ref) < 1e-5
    w.free()


@pytest.mark.parametrize("adapter_type", TYPES)
@pytest.mark.parametrize("qtype,S,inn,out,r", [("q8_0", 200, 512, 384, 16), ("q4_k", 77, 768, 320, 3)])
def test_mat_linear_fwd_bwd_matches_oracle(ctx, adapter_type, qtype, S, inn, out, r):
    import torch
    c = _case(adapter_type, qtype, S, inn, out, r, 11)
    s = 16.0 / r
    w = ctx.upload(c["raw"], qtype, inn, out)
    dp = {k: _dev(v) for k, v in c["p"].items()}
    ad = _adapter(ctx, adapter_type, r, s, dp)
    fam, xs = oracle.split_adapter_type(adapter_type)
    y = torch.empty(S, out, device="cuda")
    dx = torch.empty(S, inn, device="cuda")
    g = {}
    if xs:
        g["dM"] = torch.full((r, r), np.nan, device="cuda")
    else:
        g["dA"] = torch.full((r, inn), np.nan, device="cuda")
        g["dB"] = torch.full((out, r), np.nan, device="cuda")
    if fam == "dora-rows":
        g["dm"] = torch.full((out,), np.nan, device="cuda")
    elif fam == "dora-cols":
        g["dm"] = torch.full((inn,), np.nan, device="cuda")
    elif fam == "bora":
        g["dm_r"] = torch.full((out,), np.nan, device="cuda")
        g["dm_c"] = torch.full((inn,), np.nan, device="cuda")
    ctx.linear_mat_fwd_bwd(w, ad, _dev(c["x"]), _dev(c["dy"]), y=y, dx=dx, bias=_dev(c["bias"]), **g)
    ctx.sync()
    ref_y, cache = oracle.mat_lin_fwd(c["x"], c["Wd"], c["p"], adapter_type, s, c["bias"])
    ref = oracle.mat_lin_bwd(c["dy"], cache)
    res = {"y": rel_l2(y.cpu().numpy(), ref_y), "dx": rel_l2(dx.cpu().numpy(), ref["dx"])}
    for k, t in g.items():
        res[k] = rel_l2(t.cpu().numpy(), ref[k])
    assert set(g) | {"dx"} == set(ref)
    assert all(v < TOL for v in res.values()), res
    # the forward-only entry point gives the same y
    y2 = torch.empty(S, out, device="cuda")
    ctx.linear_mat_fwd(w, ad, _dev(c["x"]), y2, bias=_dev(c["bias"]))
    ctx.sync()
    assert torch.equal(y, y2)
    w.free()


@pytest.mark.parametrize("adapter_type", ["lora", "dora-rows"])
def test_materialized_agrees_with_functional(ctx, adapter_type):
    """For the two families the trainer applies functionally, the materialized path and the
    functional linear (sa3k_linear_fwd_bwd) compute the same step (tests/dit_lin_functional_test.cpp
    holds the reference to the same relation)."""
    import torch
    S, inn, out, r = 256, 1024, 512, 16
    c = _case(adapter_type, "q8_0", S, inn, out, r, 21)
    s = 1.0
    w = ctx.upload(c["raw"], "q8_0", inn, out)
    dp = {k: _dev(v) for k, v in c["p"].items()}
    dora = adapter_type == "dora-rows"
    ys, dxs, dAs, dBs = [], [], [], []
    for mode in ("functional", "materialized"):
        y = torch.empty(S, out, device="cuda")
        dx = torch.empty(S, inn, device="cuda")
        dA = torch.empty(r, inn, device="cuda")
        dB = torch.empty(out, r, device="cuda")
        dm = torch.empty(out, device="cuda") if dora else None
        if mode == "functional":
            bns, _ = oracle.row_norms(c["Wd"])
            keep = _dev(bns)
            ad = ctx.adapter(dp["A"], dp["B"], s, dp.get("m"), keep if dora else None)
            ctx.linear_fwd_bwd(w, _dev(c["x"]), _dev(c["dy"]), y, dx, ad=ad, dA=dA, dB=dB, dm=dm)
        else:
            ad = _adapter(ctx, adapter_type, r, s, dp)
            ctx.linear_mat_fwd_bwd(w, ad, _dev(c["x"]), _dev(c["dy"]), y=y, dx=dx, dA=dA, dB=dB, dm=dm)
        ctx.sync()
        ys.append(y.cpu().numpy()); dxs.append(dx.cpu().numpy()); dAs.append(dA.cpu().numpy()); dBs.append(dB.cpu().numpy())
    for a, b in ((ys[0], ys[1]), (dxs[0], dxs[1]), (dAs[0], dAs[1]), (dBs[0], dBs[1])):
        assert rel_l2(b, a) < TOL
    w.free()


def test_mat_rejects_bad_adapters(ctx):
    import torch
    import sa3k
    c = _case("bora", "q8_0", 4, 256, 128, 4, 5)
    w = ctx.upload(c["raw"], "q8_0", 256, 128)
    dp = {k: _dev(v) for k, v in c["p"].items()}
    y = torch.empty(4, 128, device="cuda")
    x = _dev(c["x"])
    with pytest.raises(sa3k.Sa3kError):
        ctx.linear_mat_fwd(w, _adapter(ctx, "bora-xl", 4, 1.0, dp), x, y)
    with pytest.raises(sa3k.Sa3kError):    # bora needs m_r and m_c
        ctx.linear_mat_fwd(w, _adapter(ctx, "bora", 4, 1.0, {"A": dp["A"], "B": dp["B"], "m_r": dp["m_r"]}), x, y)
    with pytest.raises(sa3k.Sa3kError):    # rank above 16
        ctx.linear_mat_fwd(w, _adapter(ctx, "lora", 17, 1.0, {"A": dp["A"], "B": dp["B"]}), x, y)
    with pytest.raises(sa3k.Sa3kError):    # -xs needs U, V and M
        ctx.linear_mat_fwd(w, _adapter(ctx, "lora-xs", 4, 1.0, {"A": dp["A"], "B": dp["B"]}), x, y)
    w.free()
