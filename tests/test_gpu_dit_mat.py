"""GPU parity of the DiT adapter-training step with materialized adapter families (dora-cols,
bora, the -xs forms; src/train_dit.h:90-164: W_eff = train_lora_effective_weight overrides each
target's weight) against float64 torch autograd through the oracle's dit_loss.  The same small
Q8_0 DiT as tests/test_gpu_dit.py; checked: per-sample loss, the device magnitude init (row and
column norms of the dequantized base, src/train_lora.h:141-190) and every adapter gradient, with
the same tolerance as the functional step (every tensor within rel-L2 1e-2)."""
import math

import numpy as np
import pytest

import oracle

pytestmark = pytest.mark.gpu

CFG = dict(io=64, dim=256, depth=2, heads=4, head_dim=64, cond_dim=64, mem_tokens=8, rot=32, time_dim=64,
           ff_inner=512, differential=0, rope_base=10000.0, norm_eps=1e-5, qk_eps=1e-6, time_min_freq=0.5,
           time_max_freq=10000.0, local_dim=0)
B, T, CTX, RANK, ALPHA = 2, 56, 16, 4, 8.0
NAMES = ("A", "B", "m_r", "m_c", "M")


def rel_l2(a, b):
    a = np.asarray(a, np.float64)
    b = np.asarray(b, np.float64)
    return float(np.linalg.norm(a - b) / max(np.linalg.norm(b), 1e-30))


def _build(ctx, cfg, adapter_type, scope, seed=0):
    import sa3k
    import dit_synth
    rng = np.random.default_rng(seed)
    shapes = dit_synth.tensor_shapes(cfg)
    dit = sa3k.Dit(ctx, cfg)
    deq = {}
    for name, shape in shapes.items():
        if dit_synth.is_weight(name):
            w = dit_synth.synth_tensor(name, shape, rng, 1.0 / math.sqrt(shape[1]))
            raw = oracle.quantize(w, "q8_0")
            dit.set_tensor(name, "q8_0", raw, shape[1], shape[0])
            deq[name] = oracle.dequantize(raw, "q8_0", shape[0], shape[1])
        else:
            v = dit_synth.synth_tensor(name, shape, rng, 0.0)
            dit.set_tensor(name, "f32", v, shape[-1], shape[0] if len(shape) > 1 else 1)
            deq[name] = v
    targets = dit_synth.scope_targets(cfg, scope)
    dit.init_adapters(adapter_type, RANK, ALPHA, targets)
    flat = np.zeros(dit.size(), np.float32)
    dit.copy(0, flat, to_model=False)
    ad = {}
    for i, name in enumerate(targets):
        offs = dit.layout(i)
        out, inn = shapes[name]
        sizes = (RANK * inn, out * RANK, out, inn, RANK * RANK)
        shp = ((RANK, inn), (out, RANK), (out,), (inn,), (RANK, RANK))
        p = {"offs": offs, "init": {}}
        for k, (key, off) in enumerate(zip(NAMES, offs)):
            if off < 0:
                continue
            if key in ("m_r", "m_c"):
                p["init"][key] = flat[off:off + sizes[k]].copy()
                v = (p["init"][key] * rng.uniform(0.9, 1.1, sizes[k])).astype(np.float32)
            elif key == "A":
                v = rng.normal(0, 1 / math.sqrt(inn), shp[k]).astype(np.float32)
            elif key == "B":
                v = rng.normal(0, 0.05, shp[k]).astype(np.float32)
            else:
                v = rng.normal(0, 0.5, shp[k]).astype(np.float32)
            flat[off:off + sizes[k]] = v.ravel()
            p[key] = v
        if offs[4] >= 0:
            p["U"] = np.linalg.qr(rng.normal(size=(out, RANK)))[0].astype(np.float32)
            p["V"] = np.linalg.qr(rng.normal(size=(inn, RANK)))[0].astype(np.float32)
            dit.set_xs_bases(name, p["U"], p["V"])
        ad[name] = p
    dit.copy(0, flat, to_model=True)
    return dit, deq, ad, targets, rng


def _inputs(rng):
    x_t = rng.standard_normal((B, T, CFG["io"])).astype(np.float32)
    target = rng.standard_normal((B, T, CFG["io"])).astype(np.float32)
    tfeat = np.stack([oracle.expo_features(t, CFG["time_dim"], CFG["time_min_freq"], CFG["time_max_freq"])
                      for t in (0.3, 0.8)]).astype(np.float32)
    cross = rng.standard_normal((B, CTX, CFG["cond_dim"])).astype(np.float32)
    glob = rng.standard_normal((B, CFG["cond_dim"])).astype(np.float32)
    return x_t, target, tfeat, cross, glob


def _reference(cfg, deq, ad, adapter_type, inputs):
    import torch
    x_t, target, tfeat, cross, glob = inputs
    c = oracle.DitCfg(io=cfg["io"], dim=cfg["dim"], depth=cfg["depth"], heads=cfg["heads"], cond_dim=cfg["cond_dim"],
                      mem_tokens=cfg["mem_tokens"], rot=cfg["rot"], time_dim=cfg["time_dim"], ff_inner=cfg["ff_inner"],
                      differential=bool(cfg["differential"]))
    T64 = lambda a: torch.tensor(np.asarray(a, np.float64))
    Wd = {k: T64(v) for k, v in deq.items()}
    fam, _ = oracle.split_adapter_type(adapter_type)
    lora, leaves = {}, {}
    for name, p in ad.items():
        q = dict(type=adapter_type, scale=ALPHA / RANK)
        lv = {}
        for key in NAMES:
            if key in p:
                lv[key] = T64(p[key]).requires_grad_(True)
        for key in ("U", "V"):
            if key in p:
                q[key] = T64(p[key])
        q.update({k: v for k, v in lv.items() if k in ("A", "B", "M")})
        if fam == "dora-rows":
            q["m"] = lv["m_r"]
        elif fam == "dora-cols":
            q["m"] = lv["m_c"]
        elif fam == "bora":
            q["m_r"], q["m_c"] = lv["m_r"], lv["m_c"]
        lora[name] = q
        leaves[name] = lv
    losses = [oracle.dit_loss(Wd, lora, T64(x_t[b]), T64(tfeat[b]), T64(cross[b]), T64(glob[b]), T64(target[b]), c)
              for b in range(B)]
    sum(losses).backward()
    grads = {n: {k: t.grad.numpy() for k, t in lv.items()} for n, lv in leaves.items()}
    return np.array([float(l) for l in losses]), grads


CASES = [("bora", "config4", 0), ("dora-cols-xs", "full", 0), ("lora-xs", "core", 1), ("dora-rows-xs", "config4", 0)]


@pytest.mark.parametrize("adapter_type,scope,differential", CASES)
def test_dit_step_materialized_matches_oracle(ctx, adapter_type, scope, differential):
    cfg = dict(CFG, differential=differential)
    dit, deq, ad, targets, rng = _build(ctx, cfg, adapter_type, scope)
    for name in targets:   # magnitude init: base row / column norms
        W = deq[name].astype(np.float64)
        if "m_r" in ad[name]["init"]:
            np.testing.assert_allclose(ad[name]["init"]["m_r"], np.sqrt((W * W).sum(1)), rtol=1e-6)
        if "m_c" in ad[name]["init"]:
            np.testing.assert_allclose(ad[name]["init"]["m_c"], np.sqrt((W * W).sum(0)), rtol=1e-6)
    inputs = _inputs(rng)
    ref_loss, ref_grads = _reference(cfg, deq, ad, adapter_type, inputs)
    dit.zero_grads()
    loss = np.zeros(B, np.float32)
    dit.forward_backward(B, T, CTX, *inputs, loss=loss)
    ctx.sync()
    assert np.max(np.abs(loss - ref_loss) / ref_loss) < 1e-3, (loss, ref_loss)
    grads = np.zeros(dit.size(), np.float32)
    dit.copy(1, grads, to_model=False)
    worst = {}
    for name in targets:
        offs = ad[name]["offs"]
        for key, off in zip(NAMES, offs):
            if off < 0:
                continue
            r = ref_grads[name][key]
            worst[f"{name}:d{key}"] = rel_l2(grads[off:off + r.size].reshape(r.shape), r)
    top = sorted(((v, k) for k, v in worst.items()), reverse=True)[:6]
    print(f"[{adapter_type} {scope} {differential}] worst:", "; ".join(f"{k} {v:.3g}" for v, k in top))
    # the north star's bar for 16-bit operands, per tensor
    bad = sorted((v, k) for k, v in worst.items() if not v < 1e-2)
    assert not bad, "; ".join(f"{k} {v:.3g}" for v, k in bad)


@pytest.mark.parametrize("adapter_type", ["bora", "dora-cols-xs"])
def test_materialized_adapter_file_round_trip(ctx, tmp_path, adapter_type):
    """The adapter file holds each target's tensors under the reference's names and shapes
    (write_train_lora_gguf, src/train_checkpoint.h:68-99: lora_A / lora_B or U / V / M_xs, then
    magnitude or magnitude_r / magnitude_c), read here with the independent gguf package; loading
    it into a freshly initialised model and writing it again reproduces the file byte for byte."""
    import gguf
    import dit_synth
    dit, _, ad, targets, _ = _build(ctx, CFG, adapter_type, "config4")
    f1 = tmp_path / "a.gguf"
    dit.save_adapter(str(f1))
    shapes = dit_synth.tensor_shapes(CFG)
    r = gguf.GGUFReader(str(f1))
    got = {t.name: tuple(int(x) for x in t.shape) for t in r.tensors}
    fam, xs = oracle.split_adapter_type(adapter_type)
    want = {}
    for name in targets:
        st = name[:-len(".weight")]
        out, inn = shapes[name]
        if xs:
            want.update({st + ".U": (RANK, out), st + ".V": (RANK, inn), st + ".M_xs": (RANK, RANK)})
        else:
            want.update({st + ".lora_A": (inn, RANK), st + ".lora_B": (RANK, out)})
        if fam == "bora":
            want.update({st + ".magnitude_r": (out,), st + ".magnitude_c": (inn,)})
        elif fam == "dora-cols":
            want[st + ".magnitude"] = (inn,)
    assert got == want
    dit2, _, _, _, _ = _build(ctx, CFG, adapter_type, "config4", seed=7)
    dit2.load_adapter(str(f1))
    f2 = tmp_path / "b.gguf"
    dit2.save_adapter(str(f2))
    assert f1.read_bytes() == f2.read_bytes()
