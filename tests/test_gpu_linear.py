"""GPU parity of the frozen-base linear (dit_lin, src/dit.h:92-149) through the C ABI.

Dequantization is checked bit for bit against the C oracle (which is pinned to gguf-py);
forward outputs and every gradient are checked against the float64 oracle on the same
dequantized weights with the north star's 16-bit-operand tolerance, rel-L2 <= 1e-2.
"""
import numpy as np
import pytest

import oracle

pytestmark = pytest.mark.gpu
TOL = 1e-2      # rel-L2, 16-bit tensor-core operands with f32 accumulation


def rel_l2(a, b):
    a = np.asarray(a, np.float64)
    b = np.asarray(b, np.float64)
    return float(np.linalg.norm(a - b) / max(np.linalg.norm(b), 1e-30))


def _dev(a):
    import torch
    return torch.from_numpy(np.ascontiguousarray(a, np.float32)).cuda()


def _case(qtype, S, inn, out, rank, seed, b_std=0.05):
    rng = np.random.default_rng(seed)
    W = rng.normal(0, 0.02, (out, inn)).astype(np.float32)
    raw = oracle.quantize(W, qtype)
    Wd = oracle.dequantize(raw, qtype, out, inn)
    A = rng.normal(0, 1 / np.sqrt(inn), (rank, inn)).astype(np.float32)
    B = rng.normal(0, b_std, (out, rank)).astype(np.float32)
    bns, nrm = oracle.row_norms(Wd)
    m = (nrm * rng.uniform(0.9, 1.2, out)).astype(np.float32)
    x = rng.normal(0, 1, (S, inn)).astype(np.float32)
    dy = rng.normal(0, 1, (S, out)).astype(np.float32)
    bias = rng.normal(0, 0.1, out).astype(np.float32)
    return dict(raw=raw, Wd=Wd, A=A, B=B, bns=bns, m=m, x=x, dy=dy, bias=bias)


@pytest.mark.parametrize("qtype,inn,out", [("q8_0", 1536, 384), ("q4_k", 512, 640),
                                           ("f16", 320, 192), ("f32", 192, 256)])
def test_dequant_bit_exact(ctx, qtype, inn, out):
    import torch
    c = _case(qtype, 4, inn, out, 2, 1)
    w = ctx.upload(c["raw"], qtype, inn, out)
    dst = torch.empty(out, inn, dtype=torch.float32, device="cuda")
    ctx.dequant(w, dst)
    ctx.sync()
    got = dst.cpu().numpy()
    assert np.array_equal(got.view(np.uint32), c["Wd"].view(np.uint32))


def test_dequant_golden_q4_k_random_blocks(ctx):
    import os
    import torch
    g = np.load(os.path.join(os.path.dirname(__file__), "golden", "q4_k.npz"))
    raw = g["raw_rand"]
    out, inn = raw.shape[0], raw.shape[1] // 144 * 256
    w = ctx.upload(raw, "q4_k", inn, out)
    dst = torch.empty(out, inn, dtype=torch.float32, device="cuda")
    ctx.dequant(w, dst)
    ctx.sync()
    assert np.array_equal(dst.cpu().numpy().view(np.uint32), g["deq_rand"].view(np.uint32))


@pytest.mark.parametrize("qtype", ["q8_0", "q4_k"])
def test_row_norms(ctx, qtype):
    import torch
    c = _case(qtype, 4, 512, 384, 2, 2)
    w = ctx.upload(c["raw"], qtype, 512, 384)
    nsq = torch.empty(384, device="cuda")
    nrm = torch.empty(384, device="cuda")
    ctx.row_norms(w, 1e-12, nsq, nrm)
    ctx.sync()
    ref_nsq, ref_nrm = oracle.row_norms(c["Wd"])
    np.testing.assert_allclose(nsq.cpu().numpy(), ref_nsq, rtol=1e-6)
    np.testing.assert_allclose(nrm.cpu().numpy(), ref_nrm, rtol=1e-6)


@pytest.fixture(params=["f16_cache", "smem_dequant"])
def operand_path(request, ctx):
    """Run a test through both operand paths of the quantized GEMMs (identical numerics)."""
    import sa3k
    if request.param == "smem_dequant":
        ctx.set_option(sa3k.OPT_SMEM_DEQUANT, 1)
    yield request.param
    ctx.set_option(sa3k.OPT_SMEM_DEQUANT, 0)


def _run(ctx, qtype, mode, S, inn, out, rank, seed=3, api="fwd_bwd"):
    import torch
    c = _case(qtype, S, inn, out, rank, seed)
    s = 16.0 / rank if rank == 16 else 2.0
    w = ctx.upload(c["raw"], qtype, inn, out)
    x, dy, bias = _dev(c["x"]), _dev(c["dy"]), _dev(c["bias"])
    A, B, m, bns = _dev(c["A"]), _dev(c["B"]), _dev(c["m"]), _dev(c["bns"])
    ad = None
    if mode != "plain":
        ad = ctx.adapter(A, B, s, m if mode == "dora" else None, bns if mode == "dora" else None)
    y = torch.empty(S, out, device="cuda")
    dx = torch.empty(S, inn, device="cuda")
    dA = torch.empty(rank, inn, device="cuda")
    dB = torch.empty(out, rank, device="cuda")
    dm = torch.empty(out, device="cuda")
    kw = dict(ad=ad, bias=bias, dA=dA if ad else None, dB=dB if ad else None, dm=dm if mode == "dora" else None)
    if api == "fwd_bwd":
        ctx.linear_fwd_bwd(w, x, dy, y, dx, **kw)
    else:
        ctx.linear_fwd(w, x, y, ad=ad, bias=bias)
        ctx.linear_bwd(w, x, y, dy, dx, **kw)
    ctx.sync()
    ref_y, cache = oracle.dit_lin_fwd(c["x"], c["Wd"], c["A"] if ad else None, c["B"] if ad else None, s,
                                      c["m"] if mode == "dora" else None, c["bns"] if mode == "dora" else None,
                                      c["bias"])
    ref = oracle.dit_lin_bwd(c["dy"], cache)
    res = {"y": rel_l2(y.cpu().numpy(), ref_y), "dx": rel_l2(dx.cpu().numpy(), ref["dx"])}
    if ad:
        res["dA"] = rel_l2(dA.cpu().numpy(), ref["dA"])
        res["dB"] = rel_l2(dB.cpu().numpy(), ref["dB"])
    if mode == "dora":
        res["dm"] = rel_l2(dm.cpu().numpy(), ref["dm"])
    return res


@pytest.mark.parametrize("qtype", ["q8_0", "q4_k", "f16", "f32"])
@pytest.mark.parametrize("mode", ["plain", "lora", "dora"])
def test_linear_fwd_bwd_small(ctx, operand_path, qtype, mode):
    res = _run(ctx, qtype, mode, S=200, inn=512, out=384, rank=16)
    assert all(v < TOL for v in res.values()), res


@pytest.mark.parametrize("rank", [2, 16])
def test_linear_separate_fwd_then_bwd(ctx, operand_path, rank):
    res = _run(ctx, "q8_0", "dora", S=130, inn=256, out=512, rank=rank, api="separate")
    assert all(v < TOL for v in res.values()), res


def test_linear_config1_q8_0_lora(ctx, operand_path):
    # 1536 x 1536 Q8_0, 1024 tokens, LoRA r 16 / alpha 16
    res = _run(ctx, "q8_0", "lora", S=1024, inn=1536, out=1536, rank=16, seed=11)
    assert all(v < TOL for v in res.values()), res


def test_linear_config2_q4_k_dora(ctx, operand_path):
    # 1536 -> 6144 Q4_K, 2048 tokens, DoRA r 16 / alpha 16
    res = _run(ctx, "q4_k", "dora", S=2048, inn=1536, out=6144, rank=16, seed=12)
    assert all(v < TOL for v in res.values()), res


def _outputs(ctx, c, qtype, S, inn, out, rank):
    import torch
    w = ctx.upload(c["raw"], qtype, inn, out)
    A, B, m, bns = _dev(c["A"]), _dev(c["B"]), _dev(c["m"]), _dev(c["bns"])
    ad = ctx.adapter(A, B, 1.0, m, bns)
    y = torch.empty(S, out, device="cuda")
    dx = torch.empty(S, inn, device="cuda")
    dA = torch.empty(rank, inn, device="cuda")
    dB = torch.empty(out, rank, device="cuda")
    dm = torch.empty(out, device="cuda")
    ctx.linear_fwd_bwd(w, _dev(c["x"]), _dev(c["dy"]), y, dx, ad=ad, bias=_dev(c["bias"]), dA=dA, dB=dB, dm=dm)
    ctx.sync()
    return {k: v.cpu().numpy() for k, v in dict(y=y, dx=dx, dA=dA, dB=dB, dm=dm).items()}


@pytest.mark.parametrize("S,inn,out", [(1000, 2560, 3072), (4352, 1536, 4608)])
def test_cta_pair_gemms_match_single_cta(ctx, S, inn, out):
    """The forward and dX GEMMs of these shapes run on CTA pairs (cta_group::2, 256-row tiles) by
    default; with pairs switched off they run one CTA per 128-row tile.  Both accumulate every
    output element over K in the same order (except the tiles of a last, partial round, which may
    run as K parts added into the output), so y and dx agree to f32 rounding (and the adapter
    gradients, fed by them, to the rounding of their atomic column sums)."""
    import sa3k
    c = _case("q8_0", S, inn, out, 16, 31)
    got = {}
    for pair in (1, 0):
        ctx.set_option(sa3k.OPT_GEMM_PAIR, pair)
        got[pair] = _outputs(ctx, c, "q8_0", S, inn, out, 16)
    ctx.set_option(sa3k.OPT_GEMM_PAIR, 1)
    for k in ("y", "dx"):
        assert np.isfinite(got[1][k]).all(), k
        assert rel_l2(got[1][k], got[0][k]) < 1e-5, k     # K parts of tail tiles reassociate the f32 sums
    for k in ("dA", "dB", "dm"):
        assert rel_l2(got[1][k], got[0][k]) < 1e-5, k
    if S * inn * out <= 1e10:     # oracle check where the float64 restatement stays quick
        ref_y, cache = oracle.dit_lin_fwd(c["x"], c["Wd"], c["A"], c["B"], 1.0, c["m"], c["bns"], c["bias"])
        ref = oracle.dit_lin_bwd(c["dy"], cache)
        res = {"y": rel_l2(got[1]["y"], ref_y), "dx": rel_l2(got[1]["dx"], ref["dx"]),
               "dA": rel_l2(got[1]["dA"], ref["dA"]), "dB": rel_l2(got[1]["dB"], ref["dB"]),
               "dm": rel_l2(got[1]["dm"], ref["dm"])}
        assert all(v < TOL for v in res.values()), res


@pytest.mark.parametrize("accumulate", [False, True])
def test_tail_split_gemms_match_oracle(ctx, accumulate):
    """4352 token rows, 1536 -> 1536: the dX GEMM has 102 256 x 256 pair tiles for 74 CTA pairs,
    so its last, partial round runs as two K halves per tile added into dx (zeroed first, or the
    existing dx when accumulating); every other output goes through the whole-tile path."""
    import torch
    S, inn, out = 4352, 1536, 1536
    c = _case("q8_0", S, inn, out, 16, 41)
    w = ctx.upload(c["raw"], "q8_0", inn, out)
    x, dy = _dev(c["x"]), _dev(c["dy"])
    y = torch.empty(S, out, device="cuda")
    ctx.linear_fwd(w, x, y)
    dx0 = torch.randn(S, inn, device="cuda") if accumulate else torch.zeros(S, inn, device="cuda")
    dx = dx0.clone()
    ctx.linear_bwd(w, x, y, dy, dx, accumulate=accumulate)
    ctx.sync()
    ref_y, cache = oracle.dit_lin_fwd(c["x"], c["Wd"], None, None, 1.0, None, None, None)
    ref = oracle.dit_lin_bwd(c["dy"], cache)
    assert rel_l2(y.cpu().numpy(), ref_y) < TOL
    assert rel_l2((dx - dx0).cpu().numpy(), ref["dx"]) < TOL


def test_linear_accumulate(ctx):
    import torch
    c = _case("q8_0", 96, 256, 256, 16, 5)
    w = ctx.upload(c["raw"], "q8_0", 256, 256)
    x, dy = _dev(c["x"]), _dev(c["dy"])
    A, B = _dev(c["A"]), _dev(c["B"])
    ad = ctx.adapter(A, B, 1.0)
    y = torch.empty(96, 256, device="cuda")
    ctx.linear_fwd(w, x, y, ad=ad)
    dx = torch.zeros(96, 256, device="cuda")
    dA = torch.zeros(16, 256, device="cuda")
    dB = torch.zeros(256, 16, device="cuda")
    for _ in range(2):
        ctx.linear_bwd(w, x, y, dy, dx, ad=ad, dA=dA, dB=dB, accumulate=True)
    ctx.sync()
    _, cache = oracle.dit_lin_fwd(c["x"], c["Wd"], c["A"], c["B"], 1.0)
    ref = oracle.dit_lin_bwd(c["dy"], cache)
    assert rel_l2(dx.cpu().numpy(), 2 * ref["dx"]) < TOL
    assert rel_l2(dA.cpu().numpy(), 2 * ref["dA"]) < TOL
    assert rel_l2(dB.cpu().numpy(), 2 * ref["dB"]) < TOL


def test_host_buffer_entry_point(ctx):
    c = _case("q8_0", 64, 256, 128, 16, 6)
    w = ctx.upload(c["raw"], "q8_0", 256, 128)
    import sa3k
    ad = sa3k.Context.adapter(c["A"], c["B"], 1.0, c["m"], c["bns"])
    y = np.empty((64, 128), np.float32)
    dx = np.empty((64, 256), np.float32)
    dA = np.empty((16, 256), np.float32)
    dB = np.empty((128, 16), np.float32)
    dm = np.empty(128, np.float32)
    ctx.linear_fwd_bwd_host(w, c["x"], c["dy"], y, dx, ad=ad, bias=c["bias"], dA=dA, dB=dB, dm=dm)
    ref_y, cache = oracle.dit_lin_fwd(c["x"], c["Wd"], c["A"], c["B"], 1.0, c["m"], c["bns"], c["bias"])
    ref = oracle.dit_lin_bwd(c["dy"], cache)
    assert rel_l2(y, ref_y) < TOL
    for name, got in (("dx", dx), ("dA", dA), ("dB", dB), ("dm", dm)):
        assert rel_l2(got, ref[name]) < TOL, name


def test_bad_arguments_raise(ctx):
    import sa3k
    c = _case("q8_0", 8, 256, 128, 2, 7)
    with pytest.raises(sa3k.Sa3kError):
        ctx.upload(c["raw"], "q4_k", 256 + 64, 128)      # Q4_K needs in % 256 == 0


@pytest.mark.parametrize("tmem", [0, 1])
def test_dequant_and_cache_paths_agree(ctx, tmem):
    """Every operand path rounds the same exact f32 dequantized value once to f16.  The in-kernel
    dequantization into a shared-memory B tile (tmem 0) runs the cache path's MMA sequence, so the
    forward matches it bit for bit; with the weight as the tensor-memory operand (tmem 1) the
    product is computed transposed, so only the f32 accumulation order differs."""
    import torch
    import sa3k
    outs = {}
    for qtype, S, inn, out in (("q4_k", 300, 512, 768), ("q8_0", 260, 384, 200)):
        c = _case(qtype, S, inn, out, 16, 21)
        for smem in (0, 1):
            ctx.set_option(sa3k.OPT_SMEM_DEQUANT, smem)
            ctx.set_option(sa3k.OPT_DEQUANT_TMEM, tmem)
            w = ctx.upload(c["raw"], qtype, inn, out)
            y = torch.empty(S, out, device="cuda")
            dx = torch.empty(S, inn, device="cuda")
            ctx.linear_fwd(w, _dev(c["x"]), y)
            ctx.linear_bwd(w, _dev(c["x"]), y, _dev(c["dy"]), dx)
            ctx.sync()
            outs[(qtype, smem)] = (y.cpu().numpy(), dx.cpu().numpy())
    ctx.set_option(sa3k.OPT_SMEM_DEQUANT, 0)
    ctx.set_option(sa3k.OPT_DEQUANT_TMEM, 1)
    for qtype in ("q4_k", "q8_0"):
        for a, b in zip(outs[(qtype, 0)], outs[(qtype, 1)]):
            if tmem == 0:
                assert np.array_equal(a.view(np.uint32), b.view(np.uint32)), qtype
            else:
                assert rel_l2(b, a) < 1e-6, (qtype, rel_l2(b, a))


def test_linear_step_replays_from_cuda_graph(ctx):
    """The whole forward + backward is capturable: replaying the captured graph on fresh inputs
    reproduces an eager call on the same inputs (y and dx bit for bit; dA, dB and dm go through
    f32 atomic column sums of the DoRA backward, so only to rounding)."""
    import torch
    c = _case("q8_0", 512, 768, 1024, 16, 31)
    w = ctx.upload(c["raw"], "q8_0", 768, 1024)
    A, B, m, bns = _dev(c["A"]), _dev(c["B"]), _dev(c["m"]), _dev(c["bns"])
    ad = ctx.adapter(A, B, 1.0, m, bns)
    x, dy = _dev(c["x"]), _dev(c["dy"])
    outs = {k: torch.empty(*s, device="cuda") for k, s in
            (("y", (512, 1024)), ("dx", (512, 768)), ("dA", (16, 768)), ("dB", (1024, 16)), ("dm", (1024,)))}

    def run():
        ctx.linear_fwd_bwd(w, x, dy, outs["y"], outs["dx"], ad=ad, dA=outs["dA"], dB=outs["dB"], dm=outs["dm"])

    run()                       # eager warm-up sizes the scratch buffers
    ctx.sync()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        ctx.set_stream(torch.cuda.current_stream().cuda_stream)
        run()
    ctx.set_stream(torch.cuda.current_stream().cuda_stream)
    x.copy_(_dev(c["x"][::-1].copy()))          # new inputs for the replay
    g.replay()
    torch.cuda.synchronize()
    got = {k: v.cpu().numpy().copy() for k, v in outs.items()}
    run()
    ctx.sync()
    for k, v in outs.items():
        if k in ("y", "dx"):
            assert np.array_equal(got[k].view(np.uint32), v.cpu().numpy().view(np.uint32)), k
        else:
            assert rel_l2(got[k], v.cpu().numpy()) < 1e-5, k
