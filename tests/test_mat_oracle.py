"""The oracle's materialized adapter families (CPU only): the hand-written backward against torch
autograd of the definition (src/train_lora.h:275-329), the known answers of the reference's
tests/train_lora_test.cpp:130-223 (the -xs forward and the finite-difference M_xs gradient), and
functional == materialized for lora / dora-rows (tests/dit_lin_functional_test.cpp)."""
import numpy as np
import pytest

import oracle

TYPES = ["lora", "dora-rows", "dora-cols", "bora", "lora-xs", "dora-rows-xs", "dora-cols-xs", "bora-xs"]


def _params(rng, out, inn, r, adapter_type):
    fam, xs = oracle.split_adapter_type(adapter_type)
    p = {}
    if xs:
        p["U"] = rng.standard_normal((out, r))
        p["V"] = rng.standard_normal((inn, r))
        p["M"] = rng.standard_normal((r, r)) * 0.3
    else:
        p["A"] = rng.standard_normal((r, inn)) * 0.3
        p["B"] = rng.standard_normal((out, r)) * 0.3
    if fam == "dora-rows":
        p["m"] = rng.uniform(0.5, 1.5, out)
    elif fam == "dora-cols":
        p["m"] = rng.uniform(0.5, 1.5, inn)
    elif fam == "bora":
        p["m_r"] = rng.uniform(0.5, 1.5, out)
        p["m_c"] = rng.uniform(0.5, 1.5, inn)
    return p


def _torch_weff(torch, W, p, adapter_type, s):
    """The definition, written with torch ops (rms_norm of ggml: x / sqrt(mean x^2 + eps))."""
    fam, xs = oracle.split_adapter_type(adapter_type)
    delta = p["U"] @ p["M"] @ p["V"].T if xs else p["B"] @ p["A"]
    v = W + s * delta
    out, inn = W.shape

    def rms(x, n):   # along the last dim, then / sqrt(n)
        return x / torch.sqrt((x * x).mean(-1, keepdim=True) + 1e-12) / np.sqrt(n)

    if fam == "lora":
        return v
    if fam == "dora-rows":
        return rms(v, inn) * p["m"][:, None]
    if fam == "dora-cols":
        return (rms(v.T, out) * p["m"][:, None]).T
    rowed = rms(v, inn) * p["m_r"][:, None]
    return (rms(rowed.T, out) * p["m_c"][:, None]).T


@pytest.mark.parametrize("adapter_type", TYPES)
def test_mat_backward_matches_autograd(adapter_type):
    import torch
    rng = np.random.default_rng(5)
    S, out, inn, r, s = 5, 7, 9, 3, 0.8
    W = rng.standard_normal((out, inn))
    p = _params(rng, out, inn, r, adapter_type)
    x = rng.standard_normal((S, inn))
    dy = rng.standard_normal((S, out))
    bias = rng.standard_normal(out)
    y, c = oracle.mat_lin_fwd(x, W, p, adapter_type, s, bias)
    g = oracle.mat_lin_bwd(dy, c)

    tp = {k: torch.tensor(v, dtype=torch.float64, requires_grad=True) for k, v in p.items()}
    tx = torch.tensor(x, requires_grad=True)
    weff = _torch_weff(torch, torch.tensor(W), tp, adapter_type, s)
    ty = tx @ weff.T + torch.tensor(bias)
    (ty * torch.tensor(dy)).sum().backward()
    assert np.abs(ty.detach().numpy() - y).max() < 1e-12
    assert np.abs(tx.grad.numpy() - g["dx"]).max() < 1e-10
    names = {"A": "dA", "B": "dB", "M": "dM", "m": "dm", "m_r": "dm_r", "m_c": "dm_c"}
    for k, t in tp.items():
        if k in ("U", "V"):
            continue          # the frozen SVD bases get no gradient
        assert np.abs(t.grad.numpy() - g[names[k]]).max() < 1e-10, k
    assert set(g) == {"dx"} | {names[k] for k in tp if k not in ("U", "V")}


# tests/train_lora_test.cpp:130-223: IN 4, OUT 6, rank 2, alpha 3, W = 0.1 (k + 1)
_UM = np.array([[0.2, -0.1], [0.3, 0.4], [-0.5, 0.2], [0.1, 0.1], [0.6, -0.3], [-0.2, 0.5]])
_VM = np.array([[0.4, 0.1], [-0.2, 0.3], [0.5, -0.4], [0.1, 0.2]])
_MM = np.array([[0.7, -0.2], [0.3, 0.9]])
_MAG = np.array([1.1, 0.9, 1.3, 0.7, 1.0, 1.2])


def _xs_case():
    IN, OUT, RK, alpha = 4, 6, 2, 3.0
    W = 0.1 * (np.arange(IN * OUT, dtype=np.float64) + 1).reshape(OUT, IN)
    return W, {"U": _UM, "V": _VM, "M": _MM, "m": _MAG}, alpha / RK


def test_xs_forward_known_answers():
    W, p, s = _xs_case()
    vref = W + s * np.einsum("oa,ab,ib->oi", _UM, _MM, _VM)
    weff, _ = oracle.mat_effective_weight(W, p, "lora-xs", s)
    assert np.abs(weff - vref).max() < 1e-4
    weff2, _ = oracle.mat_effective_weight(W, p, "dora-rows-xs", s)
    expect = _MAG[:, None] * vref / np.sqrt((vref * vref).sum(1))[:, None]
    assert np.abs(weff2 - expect).max() < 1e-4


def test_xs_core_gradient_matches_finite_differences():
    """loss = sum (W_eff - tgt)^2, tgt = 0.05 (k + 1): dM from the oracle against central
    differences with the reference test's step (1e-2) and bound (1e-2 relative)."""
    W, p, s = _xs_case()
    tgt = 0.05 * (np.arange(W.size, dtype=np.float64) + 1).reshape(W.shape)

    def loss(M):
        q = dict(p, M=M)
        weff, _ = oracle.mat_effective_weight(W, q, "lora-xs", s)
        return ((weff - tgt) ** 2).sum()

    weff, c = oracle.mat_effective_weight(W, p, "lora-xs", s)
    dM = oracle.mat_weight_grads(2.0 * (weff - tgt), c)["dM"]
    for a in range(2):
        for b in range(2):
            e = np.zeros((2, 2))
            e[a, b] = 1e-2
            num = (loss(_MM + e) - loss(_MM - e)) / 2e-2
            assert abs(num - dM[a, b]) / (abs(num) + 1e-4) < 1e-2


@pytest.mark.parametrize("adapter_type", ["lora", "dora-rows"])
def test_functional_equals_materialized(adapter_type):
    """The functional dit_lin (the path the trainer takes for these two families) and the
    materialized override agree, as tests/dit_lin_functional_test.cpp checks (<= 1e-4)."""
    rng = np.random.default_rng(9)
    S, out, inn, r, s = 6, 10, 12, 2, 0.5
    W = rng.standard_normal((out, inn))
    p = _params(rng, out, inn, r, adapter_type)
    x, dy, bias = rng.standard_normal((S, inn)), rng.standard_normal((S, out)), rng.standard_normal(out)
    dora = adapter_type == "dora-rows"
    bns = (W * W).sum(1) + inn * 1e-12
    yf, cf = oracle.dit_lin_fwd(x, W, p["A"], p["B"], s, p.get("m") if dora else None, bns if dora else None, bias)
    gf = oracle.dit_lin_bwd(dy, cf)
    ym, cm = oracle.mat_lin_fwd(x, W, p, adapter_type, s, bias)
    gm = oracle.mat_lin_bwd(dy, cm)
    assert np.abs(yf - ym).max() < 1e-10
    for k in ("dx", "dA", "dB") + (("dm",) if dora else ()):
        assert np.abs(gf[k] - gm[k]).max() < 1e-9, k


@pytest.mark.parametrize("adapter_type", TYPES)
def test_torch_weight_equals_numpy_weight(adapter_type):
    """The oracle's two forms of W_eff (torch, used inside the DiT restatement; numpy, used by the
    linear-level tests) agree."""
    import torch
    rng = np.random.default_rng(3)
    out, inn, r, s = 6, 10, 2, 0.7
    W = rng.standard_normal((out, inn))
    p = _params(rng, out, inn, r, adapter_type)
    ref, _ = oracle.mat_effective_weight(W, p, adapter_type, s)
    tp = {k: torch.tensor(v, dtype=torch.float64) for k, v in p.items()}
    got = oracle.mat_weight_torch(torch.tensor(W), tp, adapter_type, s).numpy()
    assert np.abs(got - ref).max() < 1e-12
