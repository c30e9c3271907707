"""The oracle's mode (ii): the activation rounding of ggml's CPU matrix multiply over a quantized
weight (Q8_0 weights take Q8_0 activation blocks, Q4_K weights Q8_K blocks).  The Q8_0 activation
quantizer is pinned bit for bit against gguf-py's (which states it matches ggml); the Q8_K one
(not in gguf-py) by the properties of its definition."""
import numpy as np

import oracle


def test_q8_0_activation_round_trip_matches_gguf_py():
    from gguf import quants
    from gguf.constants import GGMLQuantizationType as T
    rng = np.random.default_rng(11)
    x = rng.standard_normal((9, 128)).astype(np.float32) * rng.uniform(0.01, 10.0, (9, 1)).astype(np.float32)
    x[3, :32] = 0.0                                   # an all-zero block
    x[4, 40] = 1e4                                    # one outlier per block
    ref = quants.dequantize(quants.quantize(x, T.Q8_0), T.Q8_0)
    got = oracle.act_round_q8_0(x)
    assert np.array_equal(got.astype(np.float32), ref)


def test_q8_k_activation_round_trip_properties():
    rng = np.random.default_rng(12)
    x = rng.standard_normal((6, 512)).astype(np.float32)
    x[2, :256] = 0.0
    r = oracle.act_round_q8_k(x)
    assert not np.any(r[2, :256])
    b = x.reshape(-1, 256)
    rb = r.reshape(-1, 256)
    for xb, yb in zip(b, rb):
        if not np.any(xb):
            continue
        j = np.abs(xb).argmax()
        d = abs(xb[j]) / 127.0
        # the signed extreme maps to -127 exactly (one f32 rounding of the scale), every value
        # to within half a step
        assert abs(yb[j] - xb[j]) <= 1e-6 * abs(xb[j])
        assert np.all(np.abs(yb - xb) <= 0.5 * d * (1 + 1e-5) + 1e-12)


def test_mode2_changes_only_the_base_product():
    """Within ggml_cpu_numerics the base term sees the rounded activation and the adapter terms
    the exact one; the backward (OUT_PROD) passes the gradient straight through."""
    import torch
    rng = np.random.default_rng(13)
    W = torch.tensor(rng.normal(0, 0.02, (48, 64)))
    x = torch.tensor(rng.standard_normal((5, 64)), requires_grad=True)
    A = torch.tensor(rng.normal(0, 0.1, (4, 64)))
    B = torch.tensor(rng.normal(0, 0.1, (48, 4)))
    lora = {"w": dict(A=A, B=B, scale=2.0)}
    with oracle.ggml_cpu_numerics({"w": "q8_0"}):
        y = oracle.lin({"w": W}, lora, "w", x)
    xr = torch.tensor(oracle.act_round_q8_0(x.detach().numpy()))
    expect = xr @ W.t() + 2.0 * (x.detach() @ A.t()) @ B.t()
    assert torch.allclose(y.detach(), expect, rtol=1e-12, atol=1e-12)
    y.sum().backward()
    gexp = torch.ones(5, 48, dtype=torch.float64) @ W + 2.0 * (torch.ones(5, 48, dtype=torch.float64) @ B) @ A
    assert torch.allclose(x.grad, gexp)
    assert not oracle.ACT_QUANT   # the context restores exact numerics
