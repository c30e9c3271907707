"""The benchmark's algorithmic models (the numerators of its roofline figures), checked on CPU
against the DiT's layer shapes written out independently: the frozen-base GEMM FLOPs of one step,
the attention FLOPs, and the algorithmic bytes of the memory-bound kernel classes."""
import importlib.util
import os

import pytest

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


@pytest.fixture(scope="module")
def bench():
    spec = importlib.util.spec_from_file_location("bench_models_under_test", os.path.join(REPO, "bench.py"))
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


def test_linear_flops_match_the_layer_shapes(bench):
    cfg = bench.dit_cfg()
    B, T, C = bench.DIT_B, bench.DIT_T, bench.DIT_CTX
    D, I, L = cfg["dim"], cfg["ff_inner"], cfg["depth"]
    M, MC, MT = B * (cfg["mem_tokens"] + T), B * C, B * T
    io, cd, td = cfg["io"], cfg["cond_dim"], cfg["time_dim"]
    # per block, forward: qkv, self.out, cross.q, cross.out, ff.proj, ff.out on the token rows and
    # the context K / V on the context rows; backward: the input gradient of the six token-row
    # linears (the context projections are not differentiated)
    token_macs = M * (D * 3 * D + D * D + D * D + D * D + D * 2 * I + I * D)
    per_block = 2 * token_macs + MC * D * 2 * D
    # head and tail: time / global / gce / cond MLPs, pre_conv, proj_in, proj_out, post_conv, and
    # the input gradients of proj_out and post_conv
    head_tail = (B * td * D + B * D * D + B * cd * D + B * D * D + B * D * D + B * D * 6 * D + MC * cd * D
                 + MC * D * D + MT * io * io + MT * io * D + MT * D * io + MT * io * io + MT * D * io + MT * io * io)
    expect = 2.0 * (L * per_block + head_tail)
    got = bench.dit_linear_flops(cfg, B, T, C)
    assert got == pytest.approx(expect, rel=1e-12)
    assert got / 1e12 == pytest.approx(17.8648, abs=1e-3)   # the figure the bench line quotes


def test_attention_flops(bench):
    cfg = bench.dit_cfg()
    B, T, C = bench.DIT_B, bench.DIT_T, bench.DIT_CTX
    S, H, L = cfg["mem_tokens"] + T, cfg["heads"], cfg["depth"]
    # self: S x S scores, 2 products forward, 5 backward; cross: S x C, 2 forward, 3 backward (dq only)
    per_head_self = 2.0 * S * S * 64
    per_head_cross = 2.0 * S * C * 64
    expect = L * B * H * (7 * per_head_self + 5 * per_head_cross)
    assert bench.dit_attention_flops(cfg, B, T, C) == pytest.approx(expect, rel=1e-12)


def test_head_preparation_bytes_follow_the_path(bench):
    """The self-attention q / k head preparation is counted only when it runs as its own pass
    (differential attention); otherwise it runs in the qkv GEMM's epilogue."""
    cfg = bench.dit_cfg()
    B, T, C = bench.DIT_B, bench.DIT_T, bench.DIT_CTX
    D, L = cfg["dim"], cfg["depth"]
    M, MC = B * (cfg["mem_tokens"] + T), B * C
    cross_only = L * (6.0 * M * D + 12.0 * MC * D)
    assert cfg["differential"] == 0
    assert bench.dit_row_kernel_bytes(cfg, B, T, C)["head_prep_fwd"] == pytest.approx(cross_only)
    diff = dict(cfg, differential=1)
    assert bench.dit_row_kernel_bytes(diff, B, T, C)["head_prep_fwd"] == pytest.approx(cross_only + L * 16.0 * M * D)
    for name, v in bench.dit_row_kernel_bytes(cfg, B, T, C).items():
        assert v > 0, name
