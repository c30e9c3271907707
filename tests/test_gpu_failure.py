"""Failure path of the bounded device waits, made without a GPU fault.

Every pipeline wait of the library (TMA stages, MMA hand-offs, accumulators) is bounded: when it
runs out, the kernel records a code in the context's device error word and returns, and
sa3k_sync reports it.  sa3k_check_bounded_wait launches one kernel whose only wait is on a
barrier that nothing completes, so that path runs for real: the test checks that the timeout is
reported once, is cleared, and that the same context then computes correctly (a dequant and a
tcgen05 GEMM checked against the oracle).
"""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu


def test_bounded_wait_runs_out_and_the_context_survives(sa3k_lib):
    import time
    import torch
    import sa3k
    import gguf_blocks
    import oracle
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    ctx = sa3k.Context(0)
    try:
        t0 = time.perf_counter()
        ctx.check_bounded_wait(20000)                     # a 20 ms limit
        with pytest.raises(sa3k.Sa3kError, match="timed out"):
            ctx.sync()
        assert time.perf_counter() - t0 < 5.0             # the wait ended by its limit
        ctx.sync()                                        # reported once, then cleared

        rng = np.random.default_rng(3)
        out, inn, M = 256, 512, 128
        W = rng.normal(0, 0.02, (out, inn)).astype(np.float32)
        raw = gguf_blocks.encode(W, "q8_0")
        Wd = oracle.dequantize(raw, "q8_0", out, inn)
        w = ctx.upload(raw, "q8_0", inn, out)
        dst = torch.empty(out, inn, dtype=torch.float32, device="cuda")
        ctx.dequant(w, dst)
        x = rng.normal(0, 1, (M, inn)).astype(np.float32)
        y = torch.empty(M, out, device="cuda")
        ctx.linear_fwd(w, torch.from_numpy(x).cuda(), y)
        ctx.sync()
        assert np.array_equal(dst.cpu().numpy().view(np.uint32), Wd.view(np.uint32))
        ref = x.astype(np.float64) @ Wd.astype(np.float64).T
        rel = np.linalg.norm(y.cpu().numpy() - ref) / np.linalg.norm(ref)
        assert rel < 1e-2, rel                            # f16 operands, f32 accumulation
        w.free()
    finally:
        ctx.close()
