"""The boundary driven from compiled code on the GPU.

- tests/c/abi_linear.c: a C program against include/sa3k.h runs one LoRA linear step of a Q8_0
  base through the C ABI with host buffers and checks it against its own float64 loops.
- tests/c/train_api.cpp: a C++ program drives the reference's training API (include/sa3_train.h)
  as tools/sa3-train.cpp:578-632,709-714 does -- load_gguf, DitConfig::from,
  enumerate_train_lora_targets, init_train_lora_state (seeded), TrainDiffusionSampler,
  build_train_dit_ckpt, run_train_dit_accumulate_ckpt per sample, train_apply_accumulated_adamw
  per batch of 2 -- for two optimizer steps on a small Q8_0 DiT written as a GGUF file by the
  independent gguf package.  Checked against the float64 oracle: each step's accumulated adapter
  gradients (per tensor rel-L2 <= 1e-2; dA exactly zero on the first step, where B = 0), the losses,
  the DoRA magnitude init (base row norms), the kaiming-uniform A draw, and the parameters and
  moments after each update (the reference's averaged, clipped AdamW of those gradients)."""
import math
import subprocess

import numpy as np
import pytest

import host_programs
import oracle
import stdrng

pytestmark = pytest.mark.gpu

CFG = dict(io=64, dim=256, depth=2, heads=4, head_dim=64, cond_dim=64, mem_tokens=8, rot=32, time_dim=64,
           ff_inner=512, differential=0, rope_base=10000.0, norm_eps=1e-5, qk_eps=1e-6, time_min_freq=0.5,
           time_max_freq=10000.0)
T, CTX, RANK, ALPHA, NS = 56, 16, 4, 8.0, 4


def rel_l2(a, b):
    a, b = np.asarray(a, np.float64), np.asarray(b, np.float64)
    return float(np.linalg.norm(a - b) / max(np.linalg.norm(b), 1e-30))


def test_c_program_linear_step(ctx, tmp_path):
    exe = host_programs.build("abi_linear.c", str(tmp_path))
    r = subprocess.run([exe], capture_output=True, text=True, timeout=300)
    assert r.returncode == 0 and "OK" in r.stdout, r.stdout + r.stderr


def _write_model(path, rng):
    import gguf
    import dit_synth
    w = gguf.GGUFWriter(str(path), "sa3-dit")
    for k in ("io", "dim", "depth", "heads", "head_dim", "cond_dim", "mem_tokens", "rot", "time_dim", "differential"):
        w.add_uint32(f"dit.{k}", int(CFG[k]))
    for k in ("rope_base", "norm_eps", "qk_eps", "time_min_freq", "time_max_freq"):
        w.add_float32(f"dit.{k}", float(CFG[k]))
    deq = {}
    for name, shape in dit_synth.tensor_shapes(CFG).items():
        if dit_synth.is_weight(name):
            v = dit_synth.synth_tensor(name, shape, rng, 1.0 / math.sqrt(shape[1]))
            q = gguf.quants.quantize(v, gguf.GGMLQuantizationType.Q8_0)
            w.add_tensor(name, q, raw_dtype=gguf.GGMLQuantizationType.Q8_0)
            deq[name] = oracle.dequantize(np.ascontiguousarray(q).ravel(), "q8_0", shape[0], shape[1])
        else:
            v = dit_synth.synth_tensor(name, shape, rng, 0.0)
            w.add_tensor(name, v)
            deq[name] = v
    w.write_header_to_file()
    w.write_kv_data_to_file()
    w.write_tensors_to_file()
    w.close()
    return deq


def _oracle_grads(deq, targets, params, samples, conds):
    """float64 torch autograd of the summed per-sample losses; params: name -> (A, B, m)."""
    import torch
    c = oracle.DitCfg(**{k: CFG[k] for k in ("io", "dim", "depth", "heads", "head_dim", "cond_dim", "mem_tokens",
                                             "rot", "time_dim", "ff_inner")}, differential=False)
    T64 = lambda a: torch.tensor(np.asarray(a, np.float64))
    Wd = {k: T64(v) for k, v in deq.items()}
    lora, leaves = {}, {}
    for name in targets:
        A, B, m = (T64(x).requires_grad_(True) for x in params[name])
        bns, _ = oracle.row_norms(deq[name])
        lora[name] = dict(A=A, B=B, m=m, bns=T64(bns), scale=ALPHA / RANK)
        leaves[name] = (A, B, m)
    losses = []
    for (t, xt, v), (cross, glob) in zip(samples, conds):
        tf = oracle.expo_features(t, CFG["time_dim"], CFG["time_min_freq"], CFG["time_max_freq"])
        loss = oracle.dit_loss(Wd, lora, T64(xt), T64(tf), T64(cross), T64(glob), T64(v), c)
        loss.backward()
        losses.append(float(loss.detach()))
    return losses, {n: tuple(x.grad.numpy() for x in leaves[n]) for n in targets}


def test_train_api_two_steps_match_oracle(ctx, tmp_path):
    import dit_synth
    rng = np.random.default_rng(5)
    deq = _write_model(tmp_path / "dit.gguf", rng)
    z = rng.standard_normal((NS, T, CFG["io"])).astype(np.float32)
    cross = rng.standard_normal((NS, CTX, CFG["cond_dim"])).astype(np.float32)
    glob = rng.standard_normal((NS, CFG["cond_dim"])).astype(np.float32)
    with open(tmp_path / "inputs.bin", "wb") as f:
        f.write(np.array([NS, T, CTX], np.int32).tobytes())
        f.write(z.tobytes() + cross.tobytes() + glob.tobytes())
    exe = host_programs.build("train_api.cpp", str(tmp_path))
    out = tmp_path / "out"
    out.mkdir()
    r = subprocess.run([exe, "gpu", str(tmp_path / "dit.gguf"), str(tmp_path / "inputs.bin"), str(out)],
                       capture_output=True, text=True, timeout=600)
    assert r.returncode == 0 and "OK" in r.stdout, r.stdout + r.stderr

    targets = (out / "order.txt").read_text().split()
    shapes = dit_synth.tensor_shapes(CFG)
    assert targets == sorted(n for n in dit_synth.default_targets(CFG))

    def unflat(flat):
        res, o = {}, 0
        for n in targets:
            fo, fi = shapes[n]
            A = flat[o:o + RANK * fi].reshape(RANK, fi); o += RANK * fi
            B = flat[o:o + fo * RANK].reshape(fo, RANK); o += fo * RANK
            m = flat[o:o + fo]; o += fo
            res[n] = (A, B, m)
        assert o == flat.size
        return res

    # the seeded init: A from mt19937_64(1234), B = 0, m = the dequantized base row norms
    p0 = unflat(np.fromfile(out / "state0.f32", np.float32))
    A_ref = stdrng.lora_init_A(1234, [(shapes[n][1], shapes[n][0]) for n in targets], RANK)
    for n, a in zip(targets, A_ref):
        assert np.array_equal(p0[n][0].ravel(), a), n
        assert not np.any(p0[n][1])
        np.testing.assert_allclose(p0[n][2], oracle.row_norms(deq[n])[1], rtol=1e-6)

    params = p0
    m_st = {n: [np.zeros_like(x) for x in params[n]] for n in targets}
    v_st = {n: [np.zeros_like(x) for x in params[n]] for n in targets}
    for step in (1, 2):
        idx = [2 * (step - 1), 2 * (step - 1) + 1]
        samples, conds, losses = [], [], []
        for i in idx:
            tl = np.fromfile(out / f"s{i}_t.f32", np.float32)
            xt = np.fromfile(out / f"s{i}_xt.f32", np.float32).reshape(T, CFG["io"])
            v = np.fromfile(out / f"s{i}_v.f32", np.float32).reshape(T, CFG["io"])
            samples.append((float(tl[0]), xt, v))
            conds.append((cross[i], glob[i]))
            losses.append(float(tl[1]))
        ref_losses, ref = _oracle_grads(deq, targets, params, samples, conds)
        np.testing.assert_allclose(losses, ref_losses, rtol=1e-3)
        got = unflat(np.fromfile(out / f"grad{step}.f32", np.float32))
        worst = 0.0
        for n in targets:
            for k, lab in enumerate(("dA", "dB", "dm")):
                if step == 1 and lab == "dA":
                    assert not np.any(got[n][0]) and not np.any(ref[n][0]), n   # B = 0: no gradient into A
                    continue
                e = rel_l2(got[n][k], ref[n][k])
                worst = max(worst, e)
                assert e < 1e-2, (step, n, lab, e)
        print(f"step {step}: worst adapter-gradient rel-L2 {worst:.3g}")
        # the update: average over the 2 samples, clip at 1.0, AdamW (lr 1e-3, wd 0.01), on the
        # gradients the device accumulated
        flat_g = np.concatenate([np.concatenate([x.ravel() for x in got[n]]) for n in targets]).astype(np.float32)
        ref_norm = oracle.average_and_clip([flat_g], 2, 1.0)
        norm = float(np.fromfile(out / f"norm{step}.f64", np.float64)[0])
        assert abs(norm - ref_norm) <= 1e-6 * ref_norm
        flat_p = np.concatenate([np.concatenate([x.ravel() for x in params[n]]) for n in targets]).astype(np.float32)
        flat_m = np.concatenate([np.concatenate([x.ravel() for x in m_st[n]]) for n in targets]).astype(np.float32)
        flat_v = np.concatenate([np.concatenate([x.ravel() for x in v_st[n]]) for n in targets]).astype(np.float32)
        oracle.adamw_f32(flat_p, flat_g, flat_m, flat_v, 1e-3, 0.9, 0.999, 1e-8, 0.01, step)
        new = np.fromfile(out / f"state{step}.f32", np.float32)
        np.testing.assert_allclose(new, flat_p, rtol=1e-6, atol=1e-9)
        mv = np.fromfile(out / f"moments{step}.f32", np.float32)
        o, mm, vv = 0, [], []
        for n in targets:
            for x in params[n]:
                mm.append(mv[o:o + x.size]); o += x.size
                vv.append(mv[o:o + x.size]); o += x.size
        np.testing.assert_allclose(np.concatenate(mm), flat_m, rtol=1e-6, atol=1e-12)
        np.testing.assert_allclose(np.concatenate(vv), flat_v, rtol=1e-6, atol=1e-15)
        params = unflat(new)
        m_st = unflat(flat_m)
        v_st = unflat(flat_v)
