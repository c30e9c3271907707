"""CPU oracle for the sa3.cpp adapter-training hot path.

TEST INFRASTRUCTURE ONLY.  Only tests/, __graft_entry__.smoke() and bench.py's cpu_baseline /
reference legs import this module, and only as the checker; the product path (the sa3k CUDA
library and its host API) never calls it.

It restates, in float64 numpy (and float64 torch autograd where a whole block is differentiated),
the reference's math for the path:

  quant formats      oracle/quant.c (C), pinned against gguf-py golden vectors
  dit_lin            src/dit.h:92-149        functional LoRA / DoRA-rows linear, forward
  dit_lin backward   what ggml_build_backward_expand (src/train_ckpt.h:400) derives for the ops
                     of src/dit.h:106-147, written out by hand (pinned by finite differences,
                     as tests/dit_lin_functional_test.cpp:132-260 does)
  W_eff              src/train_lora.h:301-329 (materialized effective weight, dora-rows)
  materialized       src/train_lora.h:275-329 (every family: lora, dora-rows, dora-cols, bora,
  families           and their -xs forms, delta = U M V^T) + src/train_dit.h:96-164 (which
                     families take the materialized path); the backward is written out by hand
                     and checked against torch autograd of the definition and against the
                     known answers of tests/train_lora_test.cpp:130-223
  row norms          src/train_lora.h:141-174
  rms_norm           src/nn.h:40-42
  rope_neox          src/nn.h:53-59 (partial NeoX rotation of the first n_dims of each head)
  sdpa               src/nn.h:135-144 (+ the band mask |q-k| <= window of src/same_ae.h:96-106)
  dit_diff_attn      src/dit.h:152-158
  dit_block          src/dit.h:164-266 (autodiff_safe form, no local-cond)
  dit_head/tail      src/dit.h:286-323
  loss               src/train_ckpt.h:226-228 (mean squared error over io*frames)
  average + clip     src/train_loop.h:147-171
  AdamW              src/train_optimizer.h:42-65 (the reference's own compiled code is
                     oracle/_ref/libsa3ref.so; adamw_f32 below restates it)
  expo_features      src/sa3_pipeline.h:57-67
  functional chain   src/lora.h:372-622 (build_functional_lora: base scale and row-scaled B' of a
                     chain of lora / dora-rows adapters) + src/dit.h:108-117 (its dit_lin terms)

Layout convention: ggml [ne0, ne1] is row-major [ne1][ne0].  So W [in,out] is W[out][in]
(quant blocks run along `in`), x [in,S] is x[S][in], A [in,r] is A[r][in], B [r,out] is B[out][r].
"""
from __future__ import annotations

import ctypes
import math
import os

import numpy as np

_HERE = os.path.dirname(os.path.abspath(__file__))
QK8_0, Q8_0_BYTES = 32, 34
QK_K, Q4_K_BYTES = 256, 144


# --------------------------------------------------------------------------------------------
# C restatement (oracle/quant.c) and the reference's own compiled headers (oracle/_ref)
# --------------------------------------------------------------------------------------------
def _load(path):
    if not os.path.exists(path):
        raise FileNotFoundError(f"{path} missing: run `make -C oracle` (or __graft_entry__.build())")
    return ctypes.CDLL(path)


_lib = None
_ref = None


def lib():
    global _lib
    if _lib is None:
        _lib = _load(os.path.join(_HERE, "liboracle.so"))
        P, I64 = ctypes.c_void_p, ctypes.c_int64
        for name in ("oracle_quantize_q8_0", "oracle_dequantize_q8_0", "oracle_quantize_q4_k",
                     "oracle_dequantize_q4_k"):
            getattr(_lib, name).argtypes = [P, P, I64]
            getattr(_lib, name).restype = None
        _lib.oracle_row_norm_sq.argtypes = [P, I64, I64, ctypes.c_float, P, P]
        _lib.oracle_row_norm_sq.restype = None
    return _lib


def ref_available():
    return os.path.exists(os.path.join(_HERE, "_ref", "libsa3ref.so"))


def ref():
    """The reference's own train_optimizer.h / train_diffusion.h, compiled by oracle/Makefile."""
    global _ref
    if _ref is None:
        _ref = _load(os.path.join(_HERE, "_ref", "libsa3ref.so"))
        P, F, I = ctypes.c_void_p, ctypes.c_float, ctypes.c_int
        _ref.sa3ref_adamw_update.argtypes = [P, P, P, P, ctypes.c_long, F, F, F, F, F, I,
                                             ctypes.c_char_p, I]
        _ref.sa3ref_adamw_update.restype = I
        _ref.sa3ref_inverse_lr.argtypes = [F, I, F, F, F, F]
        _ref.sa3ref_inverse_lr.restype = F
        _ref.sa3ref_diffusion_sample_at.argtypes = [ctypes.c_ulonglong, P, ctypes.c_long, F, P, P, P]
        _ref.sa3ref_diffusion_sample_at.restype = I
    return _ref


def _ptr(a):
    return a.ctypes.data_as(ctypes.c_void_p)


def quantize(w: np.ndarray, qtype: str) -> np.ndarray:
    """Row-wise quantize W[out][in] (blocks along `in`) into raw GGUF bytes [out][row_bytes]."""
    w = np.ascontiguousarray(w, dtype=np.float32)
    out, inn = w.shape
    if qtype == "q8_0":
        assert inn % QK8_0 == 0
        raw = np.empty((out, inn // QK8_0 * Q8_0_BYTES), np.uint8)
        lib().oracle_quantize_q8_0(_ptr(w), _ptr(raw), w.size)
    elif qtype == "q4_k":
        assert inn % QK_K == 0
        raw = np.empty((out, inn // QK_K * Q4_K_BYTES), np.uint8)
        lib().oracle_quantize_q4_k(_ptr(w), _ptr(raw), w.size)
    elif qtype == "f16":
        raw = np.ascontiguousarray(w.astype(np.float16)).view(np.uint8).reshape(out, inn * 2)
    elif qtype == "f32":
        raw = w.view(np.uint8).reshape(out, inn * 4).copy()
    else:
        raise ValueError(qtype)
    return raw


def dequantize(raw: np.ndarray, qtype: str, out: int, inn: int) -> np.ndarray:
    raw = np.ascontiguousarray(raw, dtype=np.uint8)
    y = np.empty((out, inn), np.float32)
    if qtype == "q8_0":
        lib().oracle_dequantize_q8_0(_ptr(raw), _ptr(y), y.size)
    elif qtype == "q4_k":
        lib().oracle_dequantize_q4_k(_ptr(raw), _ptr(y), y.size)
    elif qtype == "f16":
        y[...] = raw.view(np.float16).reshape(out, inn).astype(np.float32)
    elif qtype == "f32":
        y[...] = raw.view(np.float32).reshape(out, inn)
    else:
        raise ValueError(qtype)
    return y


def row_norms(w: np.ndarray, eps: float = 1e-12):
    """(base_norm_sq, norm) per output row, f64 accumulation: src/train_lora.h:141-174."""
    w = np.ascontiguousarray(w, dtype=np.float32)
    out, inn = w.shape
    nsq = np.empty(out, np.float32)
    nrm = np.empty(out, np.float32)
    lib().oracle_row_norm_sq(_ptr(w), inn, out, ctypes.c_float(eps), _ptr(nsq), _ptr(nrm))
    return nsq, nrm


# --------------------------------------------------------------------------------------------
# dit_lin: functional LoRA / DoRA-rows linear (src/dit.h:92-149), forward and backward
# --------------------------------------------------------------------------------------------
def dit_lin_fwd(x, W, A=None, B=None, scale=1.0, m=None, bns=None, bias=None, dtype=np.float64):
    """y[S][out].  x[S][in], W[out][in], A[r][in], B[out][r], m/bns[out].  float64 by default
    (dtype=np.float32 is the timed CPU-baseline variant: ggml's CPU backend computes in f32).

    y = g * (x W^T + s (x A^T) B^T) + bias,  g = m / sqrt(bns + 2s t2 + s^2 t3)  (dora)
    t2[o] = sum_r (W A^T)[o,r] B[o,r]          (src/dit.h:132-135)
    t3[o] = sum_r B[o,r] (B A A^T)[o,r]         (src/dit.h:136-138)
    """
    x = np.asarray(x, dtype)
    W = np.asarray(W, dtype)
    z = x @ W.T
    cache = {"x": x, "W": W, "dtype": dtype}
    if A is not None:
        A = np.asarray(A, dtype)
        B = np.asarray(B, dtype)
        u = x @ A.T
        z = z + scale * (u @ B.T)
        cache.update(A=A, B=B, u=u, scale=scale)
        if m is not None:
            m = np.asarray(m, dtype)
            bns = np.asarray(bns, dtype)
            P = W @ A.T
            AAt = A @ A.T
            BAAt = B @ AAt
            t2 = (P * B).sum(1)
            t3 = (BAAt * B).sum(1)
            nsq = bns + 2.0 * scale * t2 + scale * scale * t3
            g = m / np.sqrt(nsq)
            cache.update(m=m, P=P, BAAt=BAAt, nsq=nsq, g=g, z=z)
            y = z * g
        else:
            y = z
    else:
        y = z
    if bias is not None:
        y = y + np.asarray(bias, dtype)
    return y, cache


def dit_lin_bwd(dy, cache):
    """Gradients of dit_lin for upstream dy[S][out]: dict(dx, dA, dB, dm)."""
    dy = np.asarray(dy, cache.get("dtype", np.float64))
    x, W = cache["x"], cache["W"]
    out = {}
    if "g" in cache:
        g, z, m, nsq = cache["g"], cache["z"], cache["m"], cache["nsq"]
        dz = dy * g
        dg = (dy * z).sum(0)
        out["dm"] = dg / np.sqrt(nsq)
        dnsq = -0.5 * dg * g / nsq
    else:
        dz = dy
        dnsq = None
    dx = dz @ W
    if "A" in cache:
        A, B, u, s = cache["A"], cache["B"], cache["u"], cache["scale"]
        dB = s * dz.T @ u
        du = s * dz @ B
        dA = du.T @ x
        dx = dx + du @ A
        if dnsq is not None:
            P, BAAt = cache["P"], cache["BAAt"]
            dt2 = 2.0 * s * dnsq
            dt3 = s * s * dnsq
            # t2 = sum_r P B:  dB += dt2 P ; dP = dt2 B ; dA += dP^T W
            dB = dB + dt2[:, None] * P
            dA = dA + (dt2[:, None] * B).T @ W
            # t3 = |B A|_row^2:  dB += 2 dt3 (B A A^T) ; dA += 2 (B^T diag(dt3) B) A
            dB = dB + 2.0 * dt3[:, None] * BAAt
            dA = dA + 2.0 * (B.T @ (dt3[:, None] * B)) @ A
        out["dA"] = dA
        out["dB"] = dB
    out["dx"] = dx
    return out


def effective_weight(W, A, B, scale, m=None):
    """Materialized W_eff[out][in] (src/train_lora.h:301-329): lora or dora-rows."""
    W = np.asarray(W, np.float64)
    v = W + scale * (np.asarray(B, np.float64) @ np.asarray(A, np.float64))
    if m is None:
        return v
    inn = W.shape[1]
    # rms_norm(v, 1e-12) / sqrt(in) == v / sqrt(sum v^2 + in*1e-12)
    nrm = np.sqrt((v * v).sum(1) + inn * 1e-12)
    return v / nrm[:, None] * np.asarray(m, np.float64)[:, None]


MAT_FAMILIES = ("lora", "dora-rows", "dora-cols", "bora")
MAT_EPS = 1e-12


def split_adapter_type(adapter_type):
    """("bora", True) for "bora-xs" (src/train_lora.h:309-310)."""
    xs = adapter_type.endswith("-xs")
    fam = adapter_type[:-3] if xs else adapter_type
    if fam not in MAT_FAMILIES:
        raise ValueError(f"unknown adapter type {adapter_type}")
    return fam, xs


def mat_delta(p, xs):
    """Low-rank update [out][in] (train_lora_delta, src/train_lora.h:290-297): B A, or for the -xs
    forms U M V^T with U [out][r], M [r][r] (M[a][b] = M_xs data[a*r+b]), V [in][r]."""
    f = lambda k: np.asarray(p[k], np.float64)
    if xs:
        return f("U") @ f("M") @ f("V").T
    return f("B") @ f("A")


def mat_effective_weight(W, p, adapter_type, scale):
    """W_eff [out][in] of any family (src/train_lora.h:299-329), float64, and the cache of the
    backward.  p: A, B (standard) or U, V, M (-xs); m (dora-rows [out] / dora-cols [in]);
    m_r [out] and m_c [in] (bora).  rms_norm(v, 1e-12) / sqrt(n) along a row of n values is
    v / sqrt(sum v^2 + n * 1e-12)."""
    fam, xs = split_adapter_type(adapter_type)
    W = np.asarray(W, np.float64)
    out, inn = W.shape
    V = W + scale * mat_delta(p, xs)
    c = {"fam": fam, "xs": xs, "V": V, "s": scale, "p": p}
    if fam == "lora":
        return V, c
    if fam == "dora-rows":
        m = np.asarray(p["m"], np.float64)
        rn = np.sqrt((V * V).sum(1) + inn * MAT_EPS)
        c.update(rn=rn, m=m)
        return V * (m / rn)[:, None], c
    if fam == "dora-cols":
        m = np.asarray(p["m"], np.float64)
        cn = np.sqrt((V * V).sum(0) + out * MAT_EPS)
        c.update(cn=cn, m=m)
        return V * (m / cn)[None, :], c
    mr, mc = np.asarray(p["m_r"], np.float64), np.asarray(p["m_c"], np.float64)
    rn = np.sqrt((V * V).sum(1) + inn * MAT_EPS)
    R = V * (mr / rn)[:, None]
    cn = np.sqrt((R * R).sum(0) + out * MAT_EPS)
    c.update(rn=rn, cn=cn, R=R, m_r=mr, m_c=mc)
    return R * (mc / cn)[None, :], c


def mat_weight_grads(G, c):
    """Gradients of the adapter parameters from G = dL/dW_eff [out][in]: dict with dA, dB
    (standard) or dM (-xs), and dm (dora-rows, dora-cols) or dm_r, dm_c (bora).  The derivative
    of v / n(v), n = sqrt(sum v^2 + k eps), along a row or column is (g - v <g, v> / n^2) / n."""
    G = np.asarray(G, np.float64)
    fam, V, p = c["fam"], c["V"], c["p"]
    out = {}
    if fam == "lora":
        dV = G
    elif fam == "dora-rows":
        t = (G * V).sum(1)
        out["dm"] = t / c["rn"]
        dV = (c["m"] / c["rn"])[:, None] * (G - V * (t / c["rn"] ** 2)[:, None])
    elif fam == "dora-cols":
        t = (G * V).sum(0)
        out["dm"] = t / c["cn"]
        dV = (c["m"] / c["cn"])[None, :] * (G - V * (t / c["cn"] ** 2)[None, :])
    else:
        R, rn, cn = c["R"], c["rn"], c["cn"]
        tc = (G * R).sum(0)
        out["dm_c"] = tc / cn
        dR = (c["m_c"] / cn)[None, :] * (G - R * (tc / cn ** 2)[None, :])
        tr = (dR * V).sum(1)
        out["dm_r"] = tr / rn
        dV = (c["m_r"] / rn)[:, None] * (dR - V * (tr / rn ** 2)[:, None])
    dD = c["s"] * dV
    f = lambda k: np.asarray(p[k], np.float64)
    if c["xs"]:
        out["dM"] = f("U").T @ dD @ f("V")
    else:
        out["dB"] = dD @ f("A").T
        out["dA"] = f("B").T @ dD
    return out


def mat_lin_fwd(x, W, p, adapter_type, scale, bias=None):
    """y = x W_eff^T + bias through the materialized effective weight (src/train_dit.h:160-164:
    the weight override that dit_lin then multiplies)."""
    Weff, c = mat_effective_weight(W, p, adapter_type, scale)
    x = np.asarray(x, np.float64)
    y = x @ Weff.T
    if bias is not None:
        y = y + np.asarray(bias, np.float64)
    c.update(x=x, Weff=Weff)
    return y, c


def mat_lin_bwd(dy, c):
    """dx and the adapter gradients of mat_lin_fwd for upstream dy [S][out]."""
    dy = np.asarray(dy, np.float64)
    out = mat_weight_grads(dy.T @ c["x"], c)
    out["dx"] = dy @ c["Weff"]
    return out


def functional_chain(W, terms, bns=None):
    """build_functional_lora (src/lora.h:372-622) for one target, in float64.  terms: list of
    (A [r][in], B [out][r], m [out] or None, s) in chain order (s = alpha / rank * strength).
    Returns (b [out] or None, [g_k [out]]): the base scale and each residual's row coefficient,
    walked as the reference does (:531-554) from the low-rank quantities nsq0 = |W|^2 + in eps,
    T2_k = rowdot(W A_k^T, B_k) and G_kl = rowdot(B_k (A_k A_l^T), B_l)."""
    W = np.asarray(W, np.float64)
    out, inn = W.shape
    nsq0 = (W * W).sum(1) + inn * 1e-12 if bns is None else np.asarray(bns, np.float64)
    A = [np.asarray(t[0], np.float64) for t in terms]
    B = [np.asarray(t[1], np.float64) for t in terms]
    n = len(terms)
    T2 = [((W @ A[k].T) * B[k]).sum(1) for k in range(n)]
    G = [[((B[k] @ (A[k] @ A[l].T)) * B[l]).sum(1) for l in range(n)] for k in range(n)]
    b = None
    g = [None] * n
    one = lambda v: 1.0 if v is None else v
    for j in range(n):
        if terms[j][2] is None:
            continue
        nsq = nsq0 * (one(b) ** 2)
        for k in range(j + 1):
            nsq = nsq + T2[k] * one(g[k]) * 2.0 * terms[k][3] * one(b)
        for k in range(j + 1):
            for l in range(k, j + 1):
                nsq = nsq + G[k][l] * one(g[k]) * one(g[l]) * terms[k][3] * terms[l][3] * (1.0 if k == l else 2.0)
        d = np.asarray(terms[j][2], np.float64) / np.sqrt(nsq)
        b = d if b is None else b * d
        for k in range(j + 1):
            g[k] = d if g[k] is None else g[k] * d
    return b, [np.ones(out) if x is None else x for x in g]


def functional_chain_forward(x, W, terms, bias=None):
    """dit_lin with a term chain (src/dit.h:108-117): y = b (x W^T) + sum_k s_k (x A_k^T) (g_k B_k)^T + bias."""
    x = np.asarray(x, np.float64)
    b, g = functional_chain(W, terms)
    y = x @ np.asarray(W, np.float64).T
    if b is not None:
        y = y * b
    for k, (A, B, m, s) in enumerate(terms):
        y = y + s * (x @ np.asarray(A, np.float64).T) @ (g[k][:, None] * np.asarray(B, np.float64)).T
    if bias is not None:
        y = y + bias
    return y


def chain_weight(W, terms):
    """The chain by its definition: adapters applied in order to the materialized weight, each
    lora adding s B A, each dora-rows rescaling every row of the sum to its magnitude
    (merge order of the reference's adapter chain)."""
    V = np.asarray(W, np.float64)
    inn = V.shape[1]
    for A, B, m, s in terms:
        V = V + s * (np.asarray(B, np.float64) @ np.asarray(A, np.float64))
        if m is not None:
            V = V / np.sqrt((V * V).sum(1) + inn * 1e-12)[:, None] * np.asarray(m, np.float64)[:, None]
    return V


# --------------------------------------------------------------------------------------------
# attention pieces (float64 torch so the whole block can be differentiated by autograd)
# --------------------------------------------------------------------------------------------
def _torch():
    import torch
    return torch


def rms_norm(x, gamma, eps):
    """src/nn.h:40-42: x / sqrt(mean(x^2) + eps) * gamma over the last dim."""
    torch = _torch()
    return x * torch.rsqrt((x * x).mean(-1, keepdim=True) + eps) * gamma


def rope_neox(x, pos, n_dims, base):
    """src/nn.h:53-59 (ggml_rope_ext, NEOX, freq_scale 1, no extrapolation): x[..., S, H, D]
    with pos[S]; pairs (i, i + n_dims/2) for i < n_dims/2 rotate by pos * base^(-2i/n_dims);
    dims >= n_dims pass through."""
    torch = _torch()
    half = n_dims // 2
    i = torch.arange(half, dtype=torch.float64)
    theta = pos.to(torch.float64)[:, None] * torch.pow(torch.tensor(base, dtype=torch.float64), -2.0 * i / n_dims)
    c = torch.cos(theta)[:, None, :].to(x.dtype)
    s = torch.sin(theta)[:, None, :].to(x.dtype)
    x0, x1, rest = x[..., :half], x[..., half:n_dims], x[..., n_dims:]
    return torch.cat([x0 * c - x1 * s, x0 * s + x1 * c, rest], -1)


def sdpa(q, k, v, scale, window=None):
    """src/nn.h:135-144: softmax(scale q k^T) v per head.  q[H,Sq,D], k/v[H,Sk,D].
    window: None = dense (the DiT); w = keep |i - j| <= w (the band of src/same_ae.h:96-106)."""
    torch = _torch()
    s = torch.matmul(q, k.transpose(-1, -2)) * scale
    if window is not None:
        iq = torch.arange(q.shape[-2])[:, None]
        ik = torch.arange(k.shape[-2])[None, :]
        s = s.masked_fill((iq - ik).abs() > window, float("-inf"))
    p = torch.softmax(s, -1)
    return torch.matmul(p, v)


def silu(x):
    torch = _torch()
    return x * torch.sigmoid(x)


# --------------------------------------------------------------------------------------------
# the DiT (src/dit.h) in float64 torch; weights are dequantized float tensors
# --------------------------------------------------------------------------------------------
class DitCfg:
    def __init__(self, io=64, dim=1536, depth=24, heads=24, head_dim=64, cond_dim=768,
                 mem_tokens=64, rot=32, time_dim=256, ff_inner=6144, differential=False,
                 rope_base=10000.0, norm_eps=1e-5, qk_eps=1e-6, time_min_freq=0.5,
                 time_max_freq=10000.0):
        self.io, self.dim, self.depth, self.heads, self.head_dim = io, dim, depth, heads, head_dim
        self.cond_dim, self.mem_tokens, self.rot, self.time_dim = cond_dim, mem_tokens, rot, time_dim
        self.ff_inner, self.differential, self.rope_base = ff_inner, differential, rope_base
        self.norm_eps, self.qk_eps = norm_eps, qk_eps
        self.time_min_freq, self.time_max_freq = time_min_freq, time_max_freq

    @property
    def qkv_mult(self):
        return 5 if self.differential else 3


def expo_features(t, dim, min_f, max_f):
    """src/sa3_pipeline.h:57-67 ([cos, sin] of t * f * 2pi, f log-spaced), float32 like the host."""
    half = dim // 2
    lmin, lmax = np.float32(math.log(min_f)), np.float32(math.log(max_f))
    out = np.empty(dim, np.float32)
    for i in range(half):
        ramp = np.float32(i / (half - 1)) if half > 1 else np.float32(0)
        freq = np.float32(np.exp(np.float32(ramp * (lmax - lmin) + lmin)))
        arg = np.float32(np.float32(t) * freq * np.float32(6.28318530717958648))
        out[i] = np.cos(arg)
        out[half + i] = np.sin(arg)
    return out


def mat_weight_torch(W, p, adapter_type, scale):
    """W_eff of a materialized family over torch tensors (differentiable), the definition of
    src/train_lora.h:275-329: ggml's rms_norm(v, 1e-12) / sqrt(n) along rows (dora-rows, bora's
    first step) or columns (dora-cols, bora's second step), scaled by the magnitudes."""
    torch = _torch()
    fam, xs = split_adapter_type(adapter_type)
    delta = p["U"] @ p["M"] @ p["V"].t() if xs else p["B"] @ p["A"]
    v = W + scale * delta
    out, inn = W.shape

    def rms(a, n):   # along the last dim, then / sqrt(n)
        return a / torch.sqrt((a * a).mean(-1, keepdim=True) + MAT_EPS) / math.sqrt(n)

    if fam == "lora":
        return v
    if fam == "dora-rows":
        return rms(v, inn) * p["m"][:, None]
    if fam == "dora-cols":
        return (rms(v.t(), out) * p["m"][:, None]).t()
    rowed = rms(v, inn) * p["m_r"][:, None]
    return (rms(rowed.t(), out) * p["m_c"][:, None]).t()


# --------------------------------------------------------------------------------------------
# mode (ii): the activation rounding of ggml's CPU matrix multiply over a quantized weight
# --------------------------------------------------------------------------------------------
# In ggml's published design the CPU mul_mat converts the activation operand to the weight type's
# vec_dot_type before the dot products: Q8_0 weights take Q8_0 activation blocks (32 values, an
# f16 scale d = max|x| / 127, q = round(x / d)), Q4_K weights take Q8_K blocks (256 values, an f32
# scale from the signed element of largest magnitude, iscale = -127 / max, q = min(127,
# round(iscale x)), d = 1 / iscale); F16 weights take f16 activations.  The backward (OUT_PROD)
# reads the f32-dequantized weight and is not rounded.  The ggml source is not available here, so
# these two quantizers are restated from that design (the Q8_0 one is checked bit for bit against
# gguf-py's, which states it matches ggml): "unverified" in the sense of the reference's own code.
ACT_QUANT = {}   # weight name -> "q8_0" | "q8_k" | "f16": set by ggml_cpu_numerics()


def act_round_q8_0(x):
    """Q8_0 quantize + dequantize along the last dim (blocks of 32), float64 numpy."""
    x = np.asarray(x, np.float64)
    b = x.reshape(-1, 32).astype(np.float32)
    d = np.abs(b).max(axis=1, keepdims=True) / np.float32(127)
    with np.errstate(divide="ignore"):
        idv = np.where(d == 0, 0, 1 / d).astype(np.float32)
    q = np.sign(b * idv) * np.floor(np.abs(b * idv) + np.float32(0.5))   # roundf: half away from zero
    dh = d.astype(np.float16).astype(np.float64)
    return (q.astype(np.float64) * dh).reshape(x.shape)


def act_round_q8_k(x):
    """Q8_K quantize + dequantize along the last dim (blocks of 256), float64 numpy."""
    x = np.asarray(x, np.float64)
    b = x.reshape(-1, 256).astype(np.float32)
    idx = np.abs(b).argmax(axis=1)
    mx = b[np.arange(b.shape[0]), idx][:, None]
    out = np.zeros_like(b, dtype=np.float64)
    nz = (mx != 0)[:, 0]
    iscale = (np.float32(-127.0) / mx[nz]).astype(np.float32)
    v = iscale * b[nz]
    q = np.minimum(np.float32(127), np.sign(v) * np.floor(np.abs(v) + np.float32(0.5)))
    out[nz] = q.astype(np.float64) * (np.float32(1.0) / iscale).astype(np.float64)
    return out.reshape(x.shape)


class ggml_cpu_numerics:
    """Context manager: within it, lin() rounds the activation of every base-weight product whose
    weight name is in `qtypes` (name -> "q8_0" | "q4_k" | "f16") the way ggml's CPU backend would."""

    def __init__(self, qtypes):
        self.map = {n: {"q8_0": "q8_0", "q4_k": "q8_k", "f16": "f16"}[t] for n, t in qtypes.items()}

    def __enter__(self):
        ACT_QUANT.clear()
        ACT_QUANT.update(self.map)
        return self

    def __exit__(self, *a):
        ACT_QUANT.clear()


def _act_round_ste(x, kind):
    """The rounded activation forward, the identity backward (OUT_PROD does not see the rounding)."""
    torch = _torch()
    xd = x.detach().cpu().numpy()
    if kind == "q8_0":
        r = act_round_q8_0(xd)
    elif kind == "q8_k":
        r = act_round_q8_k(xd)
    else:
        r = xd.astype(np.float16).astype(np.float64)
    r = torch.tensor(r, dtype=x.dtype, device=x.device)
    return x + (r - x).detach()


def lin(Wd, lora, name, x, bias=None):
    """dit_lin over torch tensors: Wd[name] is W[out][in]; lora[name] = dict(A,B,m,bns,scale), or
    for a materialized family dict(type, scale, A, B | U, V, M, m | m_r, m_c): x W_eff^T, the
    weight override of src/train_dit.h:159-164."""
    torch = _torch()
    W = Wd[name]
    p = lora.get(name) if lora else None
    if p is not None and p.get("type"):
        y = torch.matmul(x, mat_weight_torch(W, p, p["type"], p["scale"]).t())
        return y + bias if bias is not None else y
    xb = _act_round_ste(x, ACT_QUANT[name]) if name in ACT_QUANT else x
    y = torch.matmul(xb, W.t())
    if p is not None:
        A, B, s = p["A"], p["B"], p["scale"]
        y = y + s * torch.matmul(torch.matmul(x, A.t()), B.t())
        if p.get("m") is not None:
            P = torch.matmul(W, A.t())
            t2 = (P * B).sum(1)
            t3 = (torch.matmul(B, torch.matmul(A, A.t())) * B).sum(1)
            nsq = p["bns"] + 2.0 * s * t2 + s * s * t3
            y = y * (p["m"] / torch.sqrt(nsq))
    if bias is not None:
        y = y + bias
    return y


def dit_block(Wd, lora, pfx, x, context, gcond, pos, c: DitCfg, window=None, local=None):
    """src/dit.h:164-266 for one sample: x[S][dim], context[Ctx][dim], gcond[6*dim]; local
    [T][local_dim] (inpaint local conditioning, src/dit.h:244-254) or None."""
    torch = _torch()
    dim, hd, nh = c.dim, c.head_dim, c.heads
    S, Ctx = x.shape[0], context.shape[0]
    scale = 1.0 / math.sqrt(hd)
    ssg = Wd[pfx + "ssg"] + gcond
    sc_a, sh_a, g_a, sc_f, sh_f, g_f = [ssg[i * dim:(i + 1) * dim] for i in range(6)]

    def heads(a, n):
        return a.reshape(n, nh, hd)

    def to_attn(a):  # [n, H, D] -> [H, n, D]
        return a.permute(1, 0, 2)

    def attn(qa, ka, va, win):
        o = sdpa(to_attn(qa), to_attn(ka), to_attn(va), scale, win)   # [H, Sq, D]
        return o.permute(1, 0, 2).reshape(-1, dim)

    gate = lambda h, g: h / (torch.exp(g - 1.0) + 1.0)   # h * sigmoid(1 - g), src/dit.h:186-193
    res = x
    h = rms_norm(x, Wd[pfx + "pre_norm.gamma"], c.norm_eps) * (1.0 + sc_a) + sh_a
    qkv = lin(Wd, lora, pfx + "self.qkv.weight", h)
    sl = lambda t, i: t[:, i * dim:(i + 1) * dim]
    q = rms_norm(heads(sl(qkv, 0), S), Wd[pfx + "self.q_norm.gamma"], c.qk_eps)
    k = rms_norm(heads(sl(qkv, 1), S), Wd[pfx + "self.k_norm.gamma"], c.qk_eps)
    v = heads(sl(qkv, 2), S)
    q = rope_neox(q, pos, c.rot, c.rope_base)
    k = rope_neox(k, pos, c.rot, c.rope_base)
    o = attn(q, k, v, window)
    if c.differential:
        qd = rope_neox(rms_norm(heads(sl(qkv, 3), S), Wd[pfx + "self.q_norm.gamma"], c.qk_eps), pos, c.rot, c.rope_base)
        kd = rope_neox(rms_norm(heads(sl(qkv, 4), S), Wd[pfx + "self.k_norm.gamma"], c.qk_eps), pos, c.rot, c.rope_base)
        o = o - attn(qd, kd, v, window)
    o = lin(Wd, lora, pfx + "self.out.weight", o)
    x = res + gate(o, g_a)

    hc = rms_norm(x, Wd[pfx + "cross_norm.gamma"], c.norm_eps)
    qf = lin(Wd, lora, pfx + "cross.q.weight", hc)
    kv = lin(Wd, lora, pfx + "cross.kv.weight", context)
    cq = rms_norm(heads(sl(qf, 0), S), Wd[pfx + "cross.q_norm.gamma"], c.qk_eps)
    ck = rms_norm(heads(sl(kv, 0), Ctx), Wd[pfx + "cross.k_norm.gamma"], c.qk_eps)
    if c.differential:
        cqd = rms_norm(heads(sl(qf, 1), S), Wd[pfx + "cross.q_norm.gamma"], c.qk_eps)
        ckd = rms_norm(heads(sl(kv, 1), Ctx), Wd[pfx + "cross.k_norm.gamma"], c.qk_eps)
        cv = heads(sl(kv, 2), Ctx)
        oc = attn(cq, ck, cv, None) - attn(cqd, ckd, cv, None)
    else:
        cv = heads(sl(kv, 1), Ctx)
        oc = attn(cq, ck, cv, None)
    oc = lin(Wd, lora, pfx + "cross.out.weight", oc)
    x = x + oc
    if local is not None:
        # local.0 -> SiLU -> local.2, added to the T real tokens (the memory tokens get + 0)
        le = silu(lin(Wd, lora, pfx + "local.0.weight", local, Wd[pfx + "local.0.bias"]))
        le = lin(Wd, lora, pfx + "local.2.weight", le, Wd[pfx + "local.2.bias"])
        x = torch.cat([x[:c.mem_tokens], x[c.mem_tokens:] + le], 0)

    res = x
    f = rms_norm(x, Wd[pfx + "ff_norm.gamma"], c.norm_eps) * (1.0 + sc_f) + sh_f
    f = lin(Wd, lora, pfx + "ff.proj.weight", f, Wd[pfx + "ff.proj.bias"])
    inner = f.shape[1] // 2
    f = f[:, :inner] * silu(f[:, inner:])
    f = lin(Wd, lora, pfx + "ff.out.weight", f, Wd[pfx + "ff.out.bias"])
    return res + gate(f, g_f)


def mlp_silu(Wd, lora, pfx, x, bias):
    h = lin(Wd, lora, pfx + "0.weight", x, Wd[pfx + "0.bias"] if bias else None)
    return lin(Wd, lora, pfx + "2.weight", silu(h), Wd[pfx + "2.bias"] if bias else None)


def dit_head(Wd, lora, x_in, t_feat, cross, glob, c: DitCfg):
    """src/dit.h:286-310: returns (x0[mem+T][dim], context[Ctx][dim], gcond[6*dim])."""
    torch = _torch()
    te = mlp_silu(Wd, lora, "dit.time_embed.", t_feat, True)
    g = mlp_silu(Wd, lora, "dit.global_embed.", glob, False) + te
    gcond = mlp_silu(Wd, lora, "dit.gce.", g, True)
    context = mlp_silu(Wd, lora, "dit.cond_embed.", cross, False)
    x = lin(Wd, lora, "dit.pre_conv.weight", x_in) + x_in
    x = lin(Wd, lora, "dit.proj_in.weight", x)
    return torch.cat([Wd["dit.memory_tokens"], x], 0), context, gcond


def dit_tail(Wd, lora, x, c: DitCfg):
    """src/dit.h:314-323: drop memory tokens, proj_out, residual post_conv -> [T][io]."""
    x = x[c.mem_tokens:]
    x = lin(Wd, lora, "dit.proj_out.weight", x)
    return lin(Wd, lora, "dit.post_conv.weight", x) + x


def dit_loss(Wd, lora, x_t, t_feat, cross, glob, target, c: DitCfg, window=None, local=None, loss_weight=None):
    """One sample's loss: mean((v - target)^2) over io*frames (src/train_ckpt.h:226-228); with an
    inpaint input, sum(loss_weight * (v - target)^2) (src/train_ckpt.h:369, the weights of
    build_train_inpaint, src/train_inpaint.h:165-201) and the local conditioning in every block."""
    torch = _torch()
    x0, context, gcond = dit_head(Wd, lora, x_t, t_feat, cross, glob, c)
    pos = torch.arange(x0.shape[0])
    x = x0
    for l in range(c.depth):
        x = dit_block(Wd, lora, f"dit.{l}.", x, context, gcond, pos, c, window, local)
    vel = dit_tail(Wd, lora, x, c)
    d = vel - target
    if loss_weight is not None:
        return (loss_weight * d * d).sum()
    return (d * d).sum() / (c.io * target.shape[0])


def inpaint_inputs(z, mask, io, local_dim, mask_loss_weight=1.0, mask_padding_attention=True):
    """The local conditioning [T][local_dim] and loss weight [T][io] of build_train_inpaint
    (src/train_inpaint.h:165-201): channel 0 the frame mask, channels 1..io the masked latent;
    weights 1 / (io n_gen) on generated frames and 0 on context frames (mask_padding_attention),
    else normalised with mask_loss_weight on the context frames."""
    z = np.asarray(z, np.float32)
    T = z.shape[0]
    local = np.zeros((T, local_dim), np.float32)
    local[:, 0] = mask
    local[:, 1:1 + io] = z * mask[:, None]
    n_ctx = int(np.sum(mask > 0.5))
    n_gen = T - n_ctx
    f = np.float32
    if mask_padding_attention:
        wg, wc = f(1.0) / (f(io) * f(n_gen) + f(1e-8)), f(0.0)
    else:
        den = f(io) * f(n_gen) + f(mask_loss_weight) * f(io) * f(n_ctx) + f(1e-8)
        wg, wc = f(1.0) / den, f(mask_loss_weight) / den
    w = np.where(mask[:, None] > 0.5, wc, wg).astype(np.float32) * np.ones((1, io), np.float32)
    return local, w


# --------------------------------------------------------------------------------------------
# optimizer side (src/train_loop.h:147-211, src/train_optimizer.h:42-65)
# --------------------------------------------------------------------------------------------
def average_and_clip(grads, count, grad_clip):
    """In place over a list of float32 arrays.  Returns the pre-clip global norm (f64)."""
    if count > 1:
        inv = np.float32(1.0) / np.float32(count)
        for g in grads:
            g *= inv
    sumsq = 0.0
    for g in grads:
        sumsq += float(np.dot(g.astype(np.float64).ravel(), g.astype(np.float64).ravel()))
    norm = math.sqrt(sumsq)
    if grad_clip > 0.0 and norm > grad_clip:
        scale = np.float32(grad_clip / (norm + 1e-6))
        for g in grads:
            g *= scale
    return norm


def adamw_f32(p, g, m, v, lr, b1, b2, eps, wd, step):
    """In-place float32 restatement of adamw_update_vector (src/train_optimizer.h:42-65)."""
    f = np.float32
    b1c = f(1.0) - f(math.pow(f(b1), f(step)))
    b2c = f(1.0) - f(math.pow(f(b2), f(step)))
    m[...] = f(b1) * m + (f(1.0) - f(b1)) * g
    v[...] = f(b2) * v + (f(1.0) - f(b2)) * g * g
    mh = m / b1c
    vh = v / b2c
    p[...] = p - f(lr) * (mh / (np.sqrt(vh) + f(eps)) + f(wd) * p)
