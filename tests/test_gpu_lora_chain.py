"""Inference with a chain of functional adapters over a frozen quantized base (build_functional_lora,
src/lora.h:372-622, and the dit_lin term path, src/dit.h:108-117) on the GPU against the oracle's
float64 restatement: fused single-GEMM chains (<= 16 ranks), grouped chains (> 16 ranks), and a
chain whose base scale is 0 on some rows (a zero magnitude)."""
import numpy as np
import pytest

import oracle

pytestmark = pytest.mark.gpu


def rel_l2(a, b):
    a, b = np.asarray(a, np.float64), np.asarray(b, np.float64)
    return float(np.linalg.norm(a - b) / max(np.linalg.norm(b), 1e-30))


@pytest.mark.parametrize("spec,fused", [
    ([("lora", 8, 1.0)], True),
    ([("dora", 16, 1.0)], True),
    ([("lora", 4, 0.75), ("dora", 8, 1.0)], True),
    ([("dora", 4, 1.0), ("lora", 4, 0.5), ("dora", 8, 1.0)], True),
    ([("lora", 16, 1.0), ("dora", 16, 1.0)], False),
    ([("dora", 16, 1.0), ("lora", 16, 1.0), ("dora", 16, 1.0), ("lora", 8, 0.5)], False),
])
def test_chain_forward_matches_oracle(ctx, spec, fused):
    import torch
    rng = np.random.default_rng(7)
    inn, out, S = 512, 384, 300
    W = rng.normal(0, 0.02, (out, inn)).astype(np.float32)
    raw = oracle.quantize(W, "q8_0")
    Wd = oracle.dequantize(raw, "q8_0", out, inn)
    w = ctx.upload(raw, "q8_0", inn, out)
    dev = torch.device("cuda", 0)
    terms, dterms = [], []
    for kind, r, strength in spec:
        A = rng.normal(0, 1 / np.sqrt(inn), (r, inn)).astype(np.float32)
        B = rng.normal(0, 0.05, (out, r)).astype(np.float32)
        m = rng.uniform(0.5, 1.5, out).astype(np.float32) if kind == "dora" else None
        s = 16.0 / r * strength
        terms.append((A, B, m, s))
        dterms.append((torch.from_numpy(A).to(dev), torch.from_numpy(B).to(dev),
                       None if m is None else torch.from_numpy(m).to(dev), s))
    chain = ctx.lora_chain(w, dterms)
    R, is_fused = chain.info()
    assert R == sum(t[1] for t in spec) and is_fused == fused
    x = rng.standard_normal((S, inn)).astype(np.float32)
    bias = rng.normal(0, 0.1, out).astype(np.float32)
    y = torch.empty(S, out, device=dev)
    ctx.linear_fwd_chain(w, chain, torch.from_numpy(x).to(dev), y, bias=torch.from_numpy(bias).to(dev))
    ctx.sync()
    ref = oracle.functional_chain_forward(x, Wd, terms, bias=bias)
    assert rel_l2(y.cpu().numpy(), ref) < 1e-2
    chain.free()
    w.free()


def test_chain_with_zero_magnitude_rows(ctx):
    """A magnitude of 0 zeroes the base on that row; the chain then runs the grouped path (the
    fused form would divide by the base scale)."""
    import torch
    rng = np.random.default_rng(8)
    inn, out, S = 256, 128, 100
    W = rng.normal(0, 0.02, (out, inn)).astype(np.float32)
    w = ctx.upload(W.view(np.uint8).reshape(out, -1), "f32", inn, out)
    dev = torch.device("cuda", 0)
    A1 = rng.normal(0, 1 / 16, (4, inn)).astype(np.float32)
    B1 = rng.normal(0, 0.05, (out, 4)).astype(np.float32)
    m1 = rng.uniform(0.5, 1.5, out).astype(np.float32)
    m1[::7] = 0.0
    A2 = rng.normal(0, 1 / 16, (4, inn)).astype(np.float32)
    B2 = rng.normal(0, 0.05, (out, 4)).astype(np.float32)
    terms = [(A1, B1, m1, 2.0), (A2, B2, None, 2.0)]
    T = lambda a: torch.from_numpy(a).to(dev)
    chain = ctx.lora_chain(w, [(T(A1), T(B1), T(m1), 2.0), (T(A2), T(B2), None, 2.0)])
    assert chain.info() == (8, False)
    x = rng.standard_normal((S, inn)).astype(np.float32)
    y = torch.empty(S, out, device=dev)
    ctx.linear_fwd_chain(w, chain, T(x), y)
    ctx.sync()
    ref = oracle.functional_chain_forward(x, W, terms)
    assert rel_l2(y.cpu().numpy(), ref) < 1e-2
    chain.free()
    w.free()
