"""sa3k_attention_bwd_noalloc (fixed library scratch, no device allocation) against
sa3k_attention_bwd (context scratch) on the same inputs, through the C ABI.

Collected last on purpose (file name): it must pass both alone in a fresh process, where its first
call looks up the fixed scratch, and after every other test has used the library."""
import math

import pytest

pytestmark = pytest.mark.gpu


def _inputs(B, H, Sq, Sk, seed):
    import torch
    g = torch.Generator(device="cuda").manual_seed(seed)
    # token-major [B][S][H][64], the layout of the DiT's fused projection outputs
    bf = lambda S: torch.randn(B, S, H, 64, generator=g, device="cuda").to(torch.float16)
    return bf(Sq), bf(Sk), bf(Sk), bf(Sq)


@pytest.mark.parametrize("B,H,Sq,Sk,window", [
    (2, 4, 333, 333, -1),      # dense self-attention, ragged length
    (2, 3, 300, 128, -1),      # cross-attention shape
    (1, 2, 700, 700, 100),     # band |i - j| <= 100
])
def test_noalloc_matches_context_scratch_twice(ctx, B, H, Sq, Sk, window):
    import torch
    import sa3k
    q, k, v, dO = _inputs(B, H, Sq, Sk, seed=Sq + 7 * H)
    qs, ks = (Sq * H * 64, 64, H * 64), (Sk * H * 64, 64, H * 64)
    T4 = sa3k.t4
    o = torch.empty_like(q)
    lse = torch.empty(B * H * Sq, device="cuda")
    scale = 1.0 / math.sqrt(64)
    ctx.attention_fwd(B, H, Sq, Sk, scale, window, T4(q, *qs), T4(k, *ks), T4(v, *ks), T4(o, *qs), lse)

    def grads(fn):
        nan = lambda t: torch.full(t.shape, float("nan"), dtype=torch.float32, device="cuda")
        dq, dk, dv = nan(q), nan(k), nan(v)
        fn(B, H, Sq, Sk, scale, window, T4(q, *qs), T4(k, *ks), T4(v, *ks), T4(o, *qs), T4(dO, *qs), lse,
           T4(dq, *qs), T4(dk, *ks), T4(dv, *ks))
        return dq, dk, dv

    ref = grads(ctx.attention_bwd)
    first = grads(ctx.attention_bwd_noalloc)
    second = grads(ctx.attention_bwd_noalloc)      # two calls in a row reuse the same scratch
    ctx.sync()
    for got in (first, second):
        for name, a, b in zip(("dq", "dk", "dv"), got, ref):
            assert torch.isfinite(a).all(), name
            torch.testing.assert_close(a, b, rtol=1e-5, atol=1e-6, msg=name)


def test_noalloc_rejects_sizes_beyond_its_scratch(ctx):
    import torch
    import sa3k
    # 2**20 + 64 query rows: refused on the host before anything is launched
    B, H, Sq = 1, 1, (1 << 20) + 64
    t = torch.empty(1, dtype=torch.float16, device="cuda")
    f = torch.empty(1, device="cuda")
    T4 = sa3k.t4
    with pytest.raises(sa3k.Sa3kError, match="exceeds its fixed scratch"):
        ctx.attention_bwd_noalloc(B, H, Sq, 64, 0.125, -1, T4(t, 0, 0, 64), T4(t, 0, 0, 64), T4(t, 0, 0, 64),
                                  T4(t, 0, 0, 64), T4(t, 0, 0, 64), f, T4(f, 0, 0, 64))
