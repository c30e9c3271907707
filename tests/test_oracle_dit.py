"""Pin the float64 restatement of dit_lin and the DiT block (oracle/oracle.py).

The checks mirror the reference's tests/dit_lin_functional_test.cpp: functional LoRA / DoRA-rows
equals the materialized W_eff product (< 1e-4, :82-83), and the adapter / activation gradients
match central finite differences (h = 1e-3 for A, B, m and 1e-2 for x, rel < 2e-2, :132-246),
at the same sizes (IN 8, OUT 6, rank 2, SEQ 4, alpha 4).  The hand-written backward is also
compared with torch float64 autograd through the same forward.
"""
import numpy as np
import pytest

import oracle

IN, OUT, RK, SEQ, ALPHA = 8, 6, 2, 4, 4.0


def _case(seed, scale_ab=1.0):
    rng = np.random.default_rng(seed)
    W = rng.normal(0, 0.5, (OUT, IN))
    A = rng.normal(0, 0.5, (RK, IN)) * scale_ab
    B = rng.normal(0, 0.5, (OUT, RK)) * scale_ab
    x = rng.normal(0, 0.5, (SEQ, IN))
    nrm = np.sqrt((W * W).sum(1))
    m = nrm * 1.1 + 0.05
    bns = (W * W).sum(1) + IN * 1e-12
    return W, A, B, x, m, bns


@pytest.mark.parametrize("dora", [False, True])
def test_functional_matches_materialized(dora):
    W, A, B, x, m, bns = _case(1234)
    s = ALPHA / RK
    y, _ = oracle.dit_lin_fwd(x, W, A, B, s, m if dora else None, bns if dora else None)
    Weff = oracle.effective_weight(W, A, B, s, m if dora else None)
    ref = x @ Weff.T
    maxrel = np.max(np.abs(ref - y) / (np.abs(ref) + 1e-4))
    assert maxrel < 1e-4


def test_no_adapter_is_plain_matmul():
    W, A, B, x, m, bns = _case(5)
    y, _ = oracle.dit_lin_fwd(x, W)
    assert np.array_equal(y, x @ W.T)


def _loss(x, W, A, B, m, bns, tgt, s):
    y, _ = oracle.dit_lin_fwd(x, W, A, B, s, m, bns)
    return ((y - tgt) ** 2).sum()


def test_dora_gradients_match_finite_differences():
    W, A, B, x, m, bns = _case(99, 0.3)
    m = np.sqrt((W * W).sum(1)) + 0.1
    tgt = np.random.default_rng(3).normal(0, 0.5, (SEQ, OUT))
    s = ALPHA / RK
    y, cache = oracle.dit_lin_fwd(x, W, A, B, s, m, bns)
    g = oracle.dit_lin_bwd(2.0 * (y - tgt), cache)
    for name, arr, h, floor in (("dA", A, 1e-3, 1e-2), ("dB", B, 1e-3, 1e-2),
                                ("dm", m, 1e-3, 1e-2), ("dx", x, 1e-2, 1e-1)):
        worst = 0.0
        for idx in np.ndindex(arr.shape):
            save = arr[idx]
            arr[idx] = save + h
            lp = _loss(x, W, A, B, m, bns, tgt, s)
            arr[idx] = save - h
            lm = _loss(x, W, A, B, m, bns, tgt, s)
            arr[idx] = save
            num = (lp - lm) / (2 * h)
            worst = max(worst, abs(num - g[name][idx]) / (abs(num) + floor))
        assert worst < 2e-2, (name, worst)


def test_manual_backward_matches_torch_autograd():
    torch = pytest.importorskip("torch")
    rng = np.random.default_rng(17)
    out, inn, r, S = 40, 64, 16, 12
    W = rng.normal(0, 0.02, (out, inn))
    A = rng.normal(0, 1 / np.sqrt(inn), (r, inn))
    B = rng.normal(0, 0.01, (out, r))
    x = rng.normal(0, 1, (S, inn))
    m = np.sqrt((W * W).sum(1)) * 1.05
    bns = (W * W).sum(1) + inn * 1e-12
    bias = rng.normal(0, 0.1, out)
    dy = rng.normal(0, 1, (S, out))
    y, cache = oracle.dit_lin_fwd(x, W, A, B, 1.0, m, bns, bias)
    g = oracle.dit_lin_bwd(dy, cache)
    T = lambda a, rg=False: torch.tensor(a, dtype=torch.float64, requires_grad=rg)
    tx, tA, tB, tm = T(x, True), T(A, True), T(B, True), T(m, True)
    Wd = {"w": T(W)}
    lora = {"w": dict(A=tA, B=tB, m=tm, bns=T(bns), scale=1.0)}
    ty = oracle.lin(Wd, lora, "w", tx, T(bias))
    assert np.allclose(ty.detach().numpy(), y, rtol=1e-12, atol=1e-12)
    ty.backward(T(dy))
    for name, t in (("dx", tx), ("dA", tA), ("dB", tB), ("dm", tm)):
        ref = t.grad.numpy()
        assert np.allclose(g[name], ref, rtol=1e-9, atol=1e-12), name


def test_rope_neox_partial_rotation_properties():
    torch = pytest.importorskip("torch")
    x = torch.randn(5, 3, 64, dtype=torch.float64)
    pos = torch.arange(5)
    y = oracle.rope_neox(x, pos, 32, 10000.0)
    assert torch.equal(y[..., 32:], x[..., 32:])             # dims >= n_dims untouched
    assert torch.allclose(y[0], x[0])                        # position 0 is the identity
    # rotation preserves the norm of each (i, i + 16) pair
    n0 = x[..., :16] ** 2 + x[..., 16:32] ** 2
    n1 = y[..., :16] ** 2 + y[..., 16:32] ** 2
    assert torch.allclose(n0, n1)


def test_band_attention_equals_dense_when_window_covers_sequence():
    torch = pytest.importorskip("torch")
    q, k, v = (torch.randn(2, 9, 8, dtype=torch.float64) for _ in range(3))
    a = oracle.sdpa(q, k, v, 0.3, None)
    b = oracle.sdpa(q, k, v, 0.3, 8)
    assert torch.allclose(a, b)
    c = oracle.sdpa(q, k, v, 0.3, 0)          # window 0: each query sees only itself
    assert torch.allclose(c, v)
