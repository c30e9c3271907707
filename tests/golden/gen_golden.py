"""Generate the golden fixtures under tests/golden/ (committed; the GPU box never runs this).

Sources, none of which is this project's own arithmetic:
  q8_0.npz       gguf-py 0.19.0 gguf.quants.Q8_0.quantize_blocks / dequantize_blocks (which
                 state bit-exactness with ggml-quants.c) on seeded inputs plus edge blocks.
  q4_k.npz       gguf-py gguf.quants.Q4_K.dequantize_blocks over seeded random Q4_K bytes
                 (random scales/mins/nibbles: any byte pattern is a valid Q4_K block) and over
                 blocks produced by oracle/quant.c's encoder.
  optimizer.npz  the reference's own src/train_optimizer.h, compiled by oracle/Makefile into
                 oracle/_ref/libsa3ref.so: a 6-step AdamW trajectory and inverse_lr values, plus
                 the inverse_lr constants quoted by the reference's tests/train_optimizer_test.cpp
                 (read from that file as text).
  diffusion.npz  the reference's src/train_diffusion.h sample_at (x_t, v target, noise).

Run:  python tests/golden/gen_golden.py   (needs gguf-py and a reference checkout)
"""
import os
import re
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
REPO = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, os.path.join(REPO, "oracle"))
import oracle  # noqa: E402

REFERENCE = os.environ.get("SA3_REFERENCE", "")   # a reference checkout (its tests/ hold the known answers)


def gen_q8_0():
    from gguf import quants
    from gguf.constants import GGMLQuantizationType as T
    rng = np.random.default_rng(8000)
    x = rng.normal(0.0, 0.02, size=(6, 128)).astype(np.float32)
    edge = np.zeros((6, 128), np.float32)
    edge[0, :32] = 0.0                                          # all-zero block -> d = 0
    edge[0, 32:64] = np.linspace(-1, 1, 32, dtype=np.float32)   # symmetric ramp
    edge[0, 64:96] = -3.0                                       # negative max magnitude
    edge[0, 96:128] = 1e-8                                      # tiny values (subnormal f16 d)
    edge[1] = (np.arange(128) % 7 - 3).astype(np.float32) * 0.5  # exact .5 ties in x/d
    edge[2] = rng.normal(0, 1e4, 128).astype(np.float32)         # large values
    edge[3] = rng.normal(0, 1, 128).astype(np.float32)
    edge[4, ::2] = 127.0
    edge[4, 1::2] = -127.0
    edge[5] = rng.normal(0, 0.5, 128).astype(np.float32)
    x = np.concatenate([x, edge], 0)
    raw = quants.quantize(x, T.Q8_0)
    deq = quants.dequantize(raw, T.Q8_0).astype(np.float32)
    np.savez_compressed(os.path.join(HERE, "q8_0.npz"), x=x, raw=raw, deq=deq)


def gen_q4_k():
    from gguf import quants
    from gguf.constants import GGMLQuantizationType as T
    rng = np.random.default_rng(4000)
    nb = 24
    rand = rng.integers(0, 256, size=(nb, 144), dtype=np.uint8)
    # keep d / dmin finite, small normal f16 values (random bits could be inf / nan)
    for b in range(nb):
        rand[b, 0:2] = np.array([rng.uniform(1e-4, 1e-2)], np.float16).view(np.uint8)
        rand[b, 2:4] = np.array([rng.uniform(1e-4, 1e-2)], np.float16).view(np.uint8)
    rand = rand.reshape(4, 6 * 144)
    w = rng.normal(0.0, 0.02, size=(4, 1536)).astype(np.float32)
    enc = oracle.quantize(w, "q4_k")
    deq_rand = quants.dequantize(rand, T.Q4_K).astype(np.float32)
    deq_enc = quants.dequantize(enc, T.Q4_K).astype(np.float32)
    np.savez_compressed(os.path.join(HERE, "q4_k.npz"), raw_rand=rand, deq_rand=deq_rand,
                        w=w, raw_enc=enc, deq_enc=deq_enc)


def quoted_inverse_lr():
    """(step0, lr) pairs quoted in the reference's tests/train_optimizer_test.cpp:35-39."""
    if not REFERENCE:
        raise SystemExit("set SA3_REFERENCE to a reference checkout")
    path = os.path.join(REFERENCE, "tests", "train_optimizer_test.cpp")
    txt = open(path).read()
    pairs = re.findall(r"\{\s*(\d+)\s*,\s*([0-9.eE+-]+)f\s*\}", txt)
    return np.array([[int(a), float(b)] for a, b in pairs], np.float64)


def gen_optimizer():
    import ctypes
    ref = oracle.ref()
    rng = np.random.default_rng(7)
    n = 1031
    p0 = rng.normal(0, 0.05, n).astype(np.float32)
    grads = rng.normal(0, 1e-2, (6, n)).astype(np.float32)
    grads[:, :5] = [0.0, 1e-30, -1e-30, 5.0, -5.0]
    hp = dict(lr=1e-4, beta1=0.9, beta2=0.999, eps=1e-8, weight_decay=0.01)
    p = p0.copy()
    m = np.zeros(n, np.float32)
    v = np.zeros(n, np.float32)
    traj = []
    err = ctypes.create_string_buffer(256)
    for step in range(1, 7):
        rc = ref.sa3ref_adamw_update(oracle._ptr(p), oracle._ptr(grads[step - 1]), oracle._ptr(m),
                                     oracle._ptr(v), n, hp["lr"], hp["beta1"], hp["beta2"],
                                     hp["eps"], hp["weight_decay"], step, err, 256)
        assert rc == 0, err.value
        traj.append(np.stack([p.copy(), m.copy(), v.copy()]))
    quoted = quoted_inverse_lr()
    steps = np.array([0, 1, 10, 100, 500, 1000, 2499, 5000], np.int32)
    lrs = np.array([ref.sa3ref_inverse_lr(1e-4, int(s), 1e6, 0.5, 0.995, 0.0) for s in steps], np.float32)
    np.savez_compressed(os.path.join(HERE, "optimizer.npz"), p0=p0, grads=grads,
                        traj=np.stack(traj), hp=np.array([hp["lr"], hp["beta1"], hp["beta2"],
                                                          hp["eps"], hp["weight_decay"]], np.float32),
                        inv_steps=steps, inv_lr=lrs, quoted_inverse_lr=quoted)


def gen_diffusion():
    ref = oracle.ref()
    rng = np.random.default_rng(11)
    z = rng.normal(0, 1, 64 * 16).astype(np.float32)
    noise = np.empty_like(z)
    xt = np.empty_like(z)
    vt = np.empty_like(z)
    rc = ref.sa3ref_diffusion_sample_at(1234, oracle._ptr(z), z.size, 0.3, oracle._ptr(noise),
                                        oracle._ptr(xt), oracle._ptr(vt))
    assert rc == 0
    np.savez_compressed(os.path.join(HERE, "diffusion.npz"), z=z, t=np.float32(0.3), noise=noise,
                        x_t=xt, v=vt)


if __name__ == "__main__":
    gen_q8_0()
    gen_q4_k()
    gen_optimizer()
    gen_diffusion()
    for f in sorted(os.listdir(HERE)):
        if f.endswith(".npz"):
            print(f, os.path.getsize(os.path.join(HERE, f)))
