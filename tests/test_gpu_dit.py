"""GPU parity of the whole DiT adapter-training step (sa3k_dit_*) against float64 torch autograd
through the oracle's restatement of dit_head / dit_block / dit_tail and the MSE loss.

A small DiT (dim 256, 2 blocks, 4 heads, 64 memory tokens' worth of layout at reduced size) with
Q8_0 base weights and DoRA-rows adapters on self.qkv / self.out / ff.proj / ff.out; both samples
of the batch run in one pass.  Checked: per-sample loss, every adapter gradient (dA, dB, dm) and
the parameters after one clipped AdamW update; with standard and with differential attention
(src/dit.h:151-158, 214-240: qkv = [q | k | v | qd | kd], cross q = [cq | cqd], cross kv =
[ck | ckd | cv], each attention output the difference of two softmax streams)."""
import math

import numpy as np
import pytest

import oracle

pytestmark = pytest.mark.gpu

CFG = dict(io=64, dim=256, depth=2, heads=4, head_dim=64, cond_dim=64, mem_tokens=8, rot=32, time_dim=64,
           ff_inner=512, differential=0, rope_base=10000.0, norm_eps=1e-5, qk_eps=1e-6, time_min_freq=0.5,
           time_max_freq=10000.0)
B, T, CTX, RANK, ALPHA = 2, 56, 16, 4, 8.0


def rel_l2(a, b):
    a = np.asarray(a, np.float64)
    b = np.asarray(b, np.float64)
    return float(np.linalg.norm(a - b) / max(np.linalg.norm(b), 1e-30))


def _build(ctx, cfg, seed=0, scope="config4", adapter="dora-rows"):
    import sa3k
    import dit_synth
    rng = np.random.default_rng(seed)
    shapes = dit_synth.tensor_shapes(cfg)
    dit = sa3k.Dit(ctx, cfg)
    deq = {}
    for name, shape in shapes.items():
        if dit_synth.is_weight(name):
            std = 1.0 / math.sqrt(shape[1])
            w = dit_synth.synth_tensor(name, shape, rng, std)
            if shape[1] % 32:   # the inpaint local.0 width (dit.local_dim) is no quant-block multiple
                dit.set_tensor(name, "f32", w, shape[1], shape[0])
                deq[name] = w
                continue
            raw = oracle.quantize(w, "q8_0")
            dit.set_tensor(name, "q8_0", raw, shape[1], shape[0])
            deq[name] = oracle.dequantize(raw, "q8_0", shape[0], shape[1])
        else:
            v = dit_synth.synth_tensor(name, shape, rng, 0.0)
            dit.set_tensor(name, "f32", v, shape[-1], shape[0] if len(shape) > 1 else 1)
            deq[name] = v
    targets = dit_synth.scope_targets(cfg, scope)
    dit.init_adapters(adapter, RANK, ALPHA, targets)
    # adapter values: A ~ N(0, 1/sqrt(in)), B ~ N(0, 0.05), m = row norm * U(0.9, 1.1)
    flat = np.zeros(dit.size(), np.float32)
    dit.copy(0, flat, to_model=False)   # m initialised by the device (row norms)
    ad = {}
    for i, name in enumerate(targets):
        oa, ob, om = dit.offsets(i)
        out, inn = shapes[name]
        A = rng.normal(0, 1 / math.sqrt(inn), (RANK, inn)).astype(np.float32)
        Bm = rng.normal(0, 0.05, (out, RANK)).astype(np.float32)
        flat[oa:oa + A.size] = A.ravel()
        flat[ob:ob + Bm.size] = Bm.ravel()
        m_dev = m = None
        if om >= 0:
            m_dev = flat[om:om + out].copy()
            m = (m_dev * rng.uniform(0.9, 1.1, out)).astype(np.float32)
            flat[om:om + out] = m
        ad[name] = dict(A=A, B=Bm, m=m, m_dev=m_dev, offs=(oa, ob, om))
    dit.copy(0, flat, to_model=True)
    return dit, deq, ad, targets, rng


def _inputs(rng):
    x_t = rng.standard_normal((B, T, CFG["io"])).astype(np.float32)
    target = rng.standard_normal((B, T, CFG["io"])).astype(np.float32)
    ts = [0.3, 0.8]
    tfeat = np.stack([oracle.expo_features(t, CFG["time_dim"], CFG["time_min_freq"], CFG["time_max_freq"])
                      for t in ts]).astype(np.float32)
    cross = rng.standard_normal((B, CTX, CFG["cond_dim"])).astype(np.float32)
    glob = rng.standard_normal((B, CFG["cond_dim"])).astype(np.float32)
    return x_t, target, tfeat, cross, glob


def _reference(cfg, deq, ad, inputs):
    import torch
    x_t, target, tfeat, cross, glob = inputs
    c = oracle.DitCfg(io=cfg["io"], dim=cfg["dim"], depth=cfg["depth"], heads=cfg["heads"], cond_dim=cfg["cond_dim"],
                      mem_tokens=cfg["mem_tokens"], rot=cfg["rot"], time_dim=cfg["time_dim"], ff_inner=cfg["ff_inner"],
                      differential=bool(cfg["differential"]))
    T64 = lambda a: torch.tensor(np.asarray(a, np.float64))
    Wd = {k: T64(v) for k, v in deq.items()}
    lora, leaves = {}, {}
    for name, p in ad.items():
        A, Bm = T64(p["A"]).requires_grad_(True), T64(p["B"]).requires_grad_(True)
        if p["m"] is None:
            lora[name] = dict(A=A, B=Bm, scale=ALPHA / RANK)
            leaves[name] = (A, Bm)
            continue
        m = T64(p["m"]).requires_grad_(True)
        bns, _ = oracle.row_norms(deq[name])
        lora[name] = dict(A=A, B=Bm, m=m, bns=T64(bns), scale=ALPHA / RANK)
        leaves[name] = (A, Bm, m)
    losses = [oracle.dit_loss(Wd, lora, T64(x_t[b]), T64(tfeat[b]), T64(cross[b]), T64(glob[b]), T64(target[b]), c)
              for b in range(B)]
    sum(losses).backward()
    # (adapters the loss does not reach, the local.* ones without a local input, get no gradient)
    grads = {n: tuple(np.zeros(t.shape) if t.grad is None else t.grad.numpy() for t in v) for n, v in leaves.items()}
    return np.array([float(l.detach()) for l in losses]), grads


# (differential, scope, adapter): the benchmark's four per-block targets, and the reference's
# `full` (every linear, head and tail included) and `core` (per-block projections) scopes
CASES = [(0, "config4", "dora-rows", 0), (1, "config4", "dora-rows", 0), (0, "full", "dora-rows", 0),
         (1, "full", "lora", 0), (0, "core", "lora", 0), (0, "full", "dora-rows", 65)]


@pytest.mark.parametrize("differential,scope,adapter,local_dim", CASES)
def test_dit_step_matches_oracle(ctx, differential, scope, adapter, local_dim):
    """local_dim > 0: the model carries the inpaint local.* projections (local.0 with a width the
    GEMM engine does not tile, kept on the host); the step has no local input, so their adapters
    must come out with exactly zero gradients, as in the reference without an inpaint input."""
    cfg = dict(CFG, differential=differential, local_dim=local_dim)
    dit, deq, ad, targets, rng = _build(ctx, cfg, scope=scope, adapter=adapter)
    # the device initialises m to the dequantized base row norms (train_row_norms)
    for name in targets:
        if ad[name]["m_dev"] is not None:
            _, nrm = oracle.row_norms(deq[name])
            np.testing.assert_allclose(ad[name]["m_dev"], nrm, rtol=1e-6)
    inputs = _inputs(rng)
    ref_loss, ref_grads = _reference(cfg, deq, ad, inputs)

    dit.zero_grads()
    loss = np.zeros(B, np.float32)
    dit.forward_backward(B, T, CTX, *inputs, loss=loss)
    ctx.sync()
    assert np.max(np.abs(loss - ref_loss) / ref_loss) < 1e-3, (loss, ref_loss)
    grads = np.zeros(dit.size(), np.float32)
    dit.copy(1, grads, to_model=False)
    worst = {}
    for name in targets:
        oa, ob, om = ad[name]["offs"]
        ref = ref_grads[name]
        gA, gB = ref[0], ref[1]
        got = [grads[oa:oa + gA.size].reshape(gA.shape), grads[ob:ob + gB.size].reshape(gB.shape)]
        if len(ref) == 3:
            got.append(grads[om:om + ref[2].size])
        if ".local." in name:
            for g in got:
                assert not np.any(g), name
            continue
        for lab, g, r in zip(("dA", "dB", "dm"), got, ref):
            worst[f"{name}:{lab}"] = rel_l2(g, r)
    # the north star's bar for 16-bit operands, per tensor: every adapter gradient within rel-L2
    # 1e-2 of the float64 reference
    top = sorted(((v, k) for k, v in worst.items()), reverse=True)[:6]
    print(f"[{differential} {scope} {adapter}] worst:", "; ".join(f"{k} {v:.3g}" for v, k in top))
    bad = sorted((v, k) for k, v in worst.items() if not v < 1e-2)
    assert not bad, "; ".join(f"{k} {v:.3g}" for v, k in bad)

    # one averaged (count = B) + clipped AdamW update on the flat state
    import sa3k
    p0 = np.zeros(dit.size(), np.float32)
    dit.copy(0, p0, to_model=False)
    hp = sa3k.AdamWParams(1e-3, 0.9, 0.999, 1e-8, 0.01, 1.0)
    norm = dit.apply_adamw(B, hp, 1, want_norm=True)
    p1 = np.zeros(dit.size(), np.float32)
    dit.copy(0, p1, to_model=False)
    g = grads.copy()
    ref_norm = oracle.average_and_clip([g], B, 1.0)
    rp = p0.copy()
    oracle.adamw_f32(rp, g, np.zeros_like(rp), np.zeros_like(rp), 1e-3, 0.9, 0.999, 1e-8, 0.01, 1)
    assert abs(norm - ref_norm) <= 1e-6 * ref_norm
    np.testing.assert_allclose(p1, rp, rtol=1e-6, atol=1e-8)


def test_dit_rejects_misshaped_tensors(ctx):
    """Every tensor is checked against the config's shape on upload (a differential config wants
    a 5 dim qkv projection, 2 dim cross q and 3 dim cross kv); unknown names are refused."""
    import sa3k
    for diff in (0, 1):
        dit = sa3k.Dit(ctx, dict(CFG, differential=diff))
        D = CFG["dim"]
        bad_rows = (3 if diff else 5) * D
        w = np.zeros((bad_rows, D), np.float32)
        with pytest.raises(sa3k.Sa3kError, match="expected"):
            dit.set_tensor("dit.0.self.qkv.weight", "q8_0", oracle.quantize(w, "q8_0"), D, bad_rows)
        kv_rows = (2 if diff else 3) * D
        with pytest.raises(sa3k.Sa3kError, match="expected"):
            dit.set_tensor("dit.1.cross.kv.weight", "f32", np.zeros((kv_rows, D), np.float32), D, kv_rows)
        with pytest.raises(sa3k.Sa3kError, match="not a tensor"):
            dit.set_tensor("dit.2.ssg", "f32", np.zeros(6 * D, np.float32), 6 * D, 1)   # depth is 2
        with pytest.raises(sa3k.Sa3kError, match="not a tensor"):
            dit.set_tensor("vae.encoder.weight", "f32", np.zeros((D, D), np.float32), D, D)
        ok = (5 if diff else 3) * D
        dit.set_tensor("dit.0.self.qkv.weight", "f32", np.zeros((ok, D), np.float32), D, ok)
        dit.close()


def test_step_graph_replay_matches_eager(ctx):
    """sa3k_dit_forward_backward runs eagerly on its first call at a shape, records the step as a
    CUDA graph on the second and replays it afterwards; every call must give the eager result
    (up to the order of f32 atomic additions), and a changed context option re-records."""
    import sa3k
    ctx.set_option(sa3k.OPT_STEP_GRAPH, 1)
    dit, deq, ad, targets, rng = _build(ctx, dict(CFG))
    inputs = _inputs(rng)
    res = []
    for call in range(5):
        if call == 3:
            ctx.set_option(sa3k.OPT_PDL, 1)   # any option change drops the recorded graph
        dit.zero_grads()
        loss = np.zeros(B, np.float32)
        dit.forward_backward(B, T, CTX, *inputs, loss=loss)
        ctx.sync()
        g = np.zeros(dit.size(), np.float32)
        dit.copy(1, g, to_model=False)
        res.append((loss, g))
    for loss, g in res[1:]:
        np.testing.assert_allclose(loss, res[0][0], rtol=1e-5)
        assert rel_l2(g, res[0][1]) < 1e-5
    dit.close()


@pytest.mark.parametrize("differential", [0, 1])
def test_step_in_kernel_dequant_matches_cache(ctx, differential):
    """The step with every frozen-base GEMM dequantizing the Q8_0 codes in the kernel (the weight
    as the tensor-memory operand, SA3K_OPT_SMEM_DEQUANT) computes the same products as the step on
    the f16 operand cache: losses and gradients agree to the f32 accumulation order."""
    import sa3k
    res = []
    for smem in (0, 1):
        ctx.set_option(sa3k.OPT_SMEM_DEQUANT, smem)
        dit, deq, ad, targets, rng = _build(ctx, dict(CFG, differential=differential), scope="full")
        inputs = _inputs(rng)
        dit.zero_grads()
        loss = np.zeros(B, np.float32)
        dit.forward_backward(B, T, CTX, *inputs, loss=loss)
        ctx.sync()
        g = np.zeros(dit.size(), np.float32)
        dit.copy(1, g, to_model=False)
        res.append((loss, g))
        dit.close()
    ctx.set_option(sa3k.OPT_SMEM_DEQUANT, 0)
    np.testing.assert_allclose(res[1][0], res[0][0], rtol=1e-5)
    assert rel_l2(res[1][1], res[0][1]) < 1e-4


@pytest.mark.parametrize("padding_attention", [True, False])
def test_dit_step_inpaint_matches_oracle(ctx, padding_attention):
    """The inpaint objective (src/train_inpaint.h:165-201, src/dit.h:244-254): a model with the
    local.* projections (local_dim 65, zero-padded to 128 for the GEMM engine), the local-add
    conditioning of a random frame mask in every block, and the weighted loss; loss and every
    adapter gradient against float64 autograd.  Adapters on the local.* projections are refused."""
    import sa3k
    cfg = dict(CFG, local_dim=65)
    dit, deq, ad, targets, rng = _build(ctx, cfg, scope="config4")
    x_t, target, tfeat, cross, glob = _inputs(rng)
    z = rng.standard_normal((B, T, CFG["io"])).astype(np.float32)
    locals_, weights = [], []
    for b in range(B):
        mask = (rng.uniform(0, 1, T) < 0.4).astype(np.float32)
        lc, w = oracle.inpaint_inputs(z[b], mask, CFG["io"], 65, mask_loss_weight=0.5,
                                      mask_padding_attention=padding_attention)
        locals_.append(lc)
        weights.append(w)
    local = np.stack(locals_)
    lw = np.stack(weights)
    dit.zero_grads()
    loss = np.zeros(B, np.float32)
    dit.forward_backward_inpaint(B, T, CTX, x_t, target, tfeat, cross, glob, local, lw, loss=loss)
    ctx.sync()
    grads = np.zeros(dit.size(), np.float32)
    dit.copy(1, grads, to_model=False)

    import torch
    c = oracle.DitCfg(io=cfg["io"], dim=cfg["dim"], depth=cfg["depth"], heads=cfg["heads"], cond_dim=cfg["cond_dim"],
                      mem_tokens=cfg["mem_tokens"], rot=cfg["rot"], time_dim=cfg["time_dim"], ff_inner=cfg["ff_inner"])
    T64 = lambda a: torch.tensor(np.asarray(a, np.float64))
    Wd = {k: T64(v) for k, v in deq.items()}
    lora, leaves = {}, {}
    for name, p in ad.items():
        A, Bm, m = (T64(p[k]).requires_grad_(True) for k in ("A", "B", "m"))
        bns, _ = oracle.row_norms(deq[name])
        lora[name] = dict(A=A, B=Bm, m=m, bns=T64(bns), scale=ALPHA / RANK)
        leaves[name] = (A, Bm, m)
    ref_loss = []
    for b in range(B):
        lb = oracle.dit_loss(Wd, lora, T64(x_t[b]), T64(tfeat[b]), T64(cross[b]), T64(glob[b]), T64(target[b]), c,
                             local=T64(local[b]), loss_weight=T64(lw[b]))
        lb.backward()
        ref_loss.append(float(lb.detach()))
    np.testing.assert_allclose(loss, ref_loss, rtol=1e-3)
    worst = {}
    for name in targets:
        oa, ob, om = ad[name]["offs"]
        for lab, off, t in zip(("dA", "dB", "dm"), (oa, ob, om), leaves[name]):
            r = t.grad.numpy()
            worst[f"{name}:{lab}"] = rel_l2(grads[off:off + r.size].reshape(r.shape), r)
    top = sorted(((v, k) for k, v in worst.items()), reverse=True)[:4]
    print(f"[inpaint padding_attention={padding_attention}] worst:", "; ".join(f"{k} {v:.3g}" for v, k in top))
    bad = sorted((v, k) for k, v in worst.items() if not v < 1e-2)
    assert not bad, bad
    dit.close()

    full, _, _, _, _ = _build(ctx, cfg, scope="full")
    with pytest.raises(sa3k.Sa3kError, match="local"):
        full.forward_backward_inpaint(B, T, CTX, x_t, target, tfeat, cross, glob, local, lw)
    full.close()
