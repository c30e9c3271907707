"""Data-parallel DiT adapter training on 2 GPUs through the C ABI (sa3k_dp_* over NCCL): two
ranks with two samples each must end with identical adapters, equal (up to the reassociation
of the gradient sums) to one GPU that runs all four samples in one pass.

Needs 2 GPUs; skipped otherwise.  NVLS is off (plain NCCL rings over NVLink)."""
import os
import socket
import tempfile
from datetime import timedelta

import numpy as np
import pytest

pytestmark = pytest.mark.gpu


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _two_rank_inputs(rng_seed):
    import test_gpu_dit as base
    rng = np.random.default_rng(rng_seed)
    return [base._inputs(rng) for _ in range(2)]          # per rank: B = 2 samples


STEPS = 2


def _hp():
    import sa3k
    return sa3k.AdamWParams(1e-3, 0.9, 0.999, 1e-8, 0.01, 1.0)


def _worker(rank, world, port, outdir):
    import torch
    import torch.distributed as dist
    import dp
    import sa3k
    import test_gpu_dit as base
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    torch.cuda.set_device(rank)
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=timedelta(seconds=120))
    comm = None
    try:
        ctx = sa3k.Context(rank)
        dit, _, _, _, _ = base._build(ctx, dict(base.CFG), seed=0)   # same base + adapters on every rank
        uid = dp.exchange_unique_id(rank, sa3k.dp_unique_id, dist.broadcast_object_list)
        comm = sa3k.DpComm(ctx, world, rank, uid)
        tr = dp.DataParallelTrainer(dit, dp.NcclReduce(comm))
        norms = []
        for step in range(STEPS):
            x_t, target, tfeat, cross, glob = _two_rank_inputs(100 + step)[rank]
            tr.begin()
            tr.accumulate(base.B, base.T, base.CTX, x_t, target, tfeat, cross, glob)
            norms.append(tr.apply(_hp(), want_norm=True))
        p = np.zeros(dit.size(), np.float32)
        dit.copy(0, p, to_model=False)
        ctx.sync()
        np.savez(os.path.join(outdir, f"r{rank}.npz"), p=p, norms=np.array(norms))
        comm.close()
        dit.close()
        ctx.close()
    finally:
        dist.destroy_process_group()


def test_two_gpu_dp_step_matches_one_gpu(ctx):
    import torch
    import torch.multiprocessing as mp
    import dp
    import test_gpu_dit as base
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    world = 2
    os.environ["NCCL_NVLS_ENABLE"] = "0"
    with tempfile.TemporaryDirectory() as d:
        mp.start_processes(_worker, args=(world, _free_port(), d), nprocs=world, start_method="spawn")
        r0, r1 = np.load(os.path.join(d, "r0.npz")), np.load(os.path.join(d, "r1.npz"))
    assert np.array_equal(r0["p"], r1["p"]), "ranks disagree after the all-reduce + AdamW"

    dit, _, _, _, _ = base._build(ctx, dict(base.CFG), seed=0)
    p0 = np.zeros(dit.size(), np.float32)
    dit.copy(0, p0, to_model=False)
    tr = dp.DataParallelTrainer(dit)
    norms = []
    for step in range(STEPS):
        per_rank = _two_rank_inputs(100 + step)
        joined = [np.concatenate([per_rank[0][i], per_rank[1][i]]) for i in range(5)]
        tr.begin()
        tr.accumulate(2 * base.B, base.T, base.CTX, *joined)
        norms.append(tr.apply(_hp(), want_norm=True))
    p1 = np.zeros(dit.size(), np.float32)
    dit.copy(0, p1, to_model=False)
    ctx.sync()
    # step 1 sees identical adapters (norms agree to f32 summation order); step 2 sees adapters
    # whose AdamW updates already differ slightly, so its gradient norm is compared loosely
    np.testing.assert_allclose(r0["norms"][0], norms[0], rtol=1e-4)
    np.testing.assert_allclose(r0["norms"][1:], norms[1:], rtol=2e-3)
    upd_dp, upd_one = r0["p"] - p0, p1 - p0
    rel = np.linalg.norm(upd_dp - upd_one) / np.linalg.norm(upd_one)
    assert rel < 1e-2, rel
    assert np.abs(upd_dp - upd_one).max() <= 2 * STEPS * 1e-3 + 1e-6


@pytest.mark.timeout(180, method="thread")
def test_comm_rendezvous_without_peer_times_out(ctx):
    """A two-rank communicator whose second rank never joins: the bounded rendezvous aborts the
    NCCL communicator and reports an error within its limit, and the context stays usable (one
    GPU; nothing runs on the device while the rendezvous waits)."""
    import time
    import torch
    import sa3k
    os.environ["NCCL_NVLS_ENABLE"] = "0"
    uid = sa3k.dp_unique_id()
    t0 = time.monotonic()
    with pytest.raises(sa3k.Sa3kError, match="did not all join"):
        sa3k.DpComm(ctx, 2, 0, uid, timeout_s=3.0)
    assert time.monotonic() - t0 < 60.0
    p = torch.zeros(64, device="cuda")
    g = torch.ones(64, device="cuda")
    m, v = torch.zeros_like(p), torch.zeros_like(p)
    ctx.adamw(p, g, m, v, sa3k.AdamWParams(1e-3, 0.9, 0.999, 1e-8, 0.0, 0.0), 1)
    ctx.sync()
    assert torch.allclose(p, torch.full_like(p, -1e-3), rtol=1e-4)
