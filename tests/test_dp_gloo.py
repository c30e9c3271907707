"""Host logic of data-parallel training on 2 CPU ranks (gloo): the clique-id exchange and the
step semantics of sa3.cpp_b200/dp.py (sum of per-rank gradients, AdamW averaged over
samples-per-rank x ranks), checked against one process that sees every sample.

The model here is a small DoRA linear whose gradients come from the oracle's restatement of
dit_lin (src/dit.h:92-149) and whose update is the oracle's average_and_clip + AdamW; the GPU
form of the same step is tests/test_gpu_dp.py."""
import os
import socket
import tempfile
from datetime import timedelta

import numpy as np
import pytest

IN, OUT, R, S, SCALE = 64, 48, 4, 24, 2.0


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


class OracleDora:
    """Flat [A | B | m] adapter state of one DoRA linear, gradients summed over samples."""

    def __init__(self):
        import oracle
        self.oracle = oracle
        rng = np.random.default_rng(5)
        self.W = rng.normal(0, 0.05, (OUT, IN)).astype(np.float32)
        A = rng.normal(0, 1 / np.sqrt(IN), (R, IN)).astype(np.float32)
        B = rng.normal(0, 0.05, (OUT, R)).astype(np.float32)
        self.bns, m = oracle.row_norms(self.W)
        self.p = np.concatenate([A.ravel(), B.ravel(), m.astype(np.float32)]).astype(np.float32)
        self.g = np.zeros_like(self.p)
        self.am = np.zeros_like(self.p)
        self.av = np.zeros_like(self.p)

    def _split(self, v):
        return v[:R * IN].reshape(R, IN), v[R * IN:R * IN + OUT * R].reshape(OUT, R), v[R * IN + OUT * R:]

    def zero_grads(self):
        self.g[:] = 0

    def forward_backward(self, seed):
        A, B, m = self._split(self.p)
        rng = np.random.default_rng(seed)
        x = rng.normal(0, 1, (S, IN)).astype(np.float32)
        dy = rng.normal(0, 1, (S, OUT)).astype(np.float32)
        _, cache = self.oracle.dit_lin_fwd(x, self.W, A, B, SCALE, m, self.bns, None, dtype=np.float32)
        gr = self.oracle.dit_lin_bwd(dy, cache)
        self.g += np.concatenate([gr["dA"].ravel(), gr["dB"].ravel(), gr["dm"].ravel()]).astype(np.float32)

    def apply_adamw(self, count, hp, step, want_norm=False):
        norm = self.oracle.average_and_clip([self.g], count, hp["clip"])
        self.oracle.adamw_f32(self.p, self.g, self.am, self.av, hp["lr"], 0.9, 0.999, 1e-8, 0.01, step)
        return norm if want_norm else None


class GlooReduce:
    def __init__(self, world):
        self.world = world

    def allreduce_adamw(self, model, samples_per_rank, hp, step, want_norm=False):
        import torch
        import torch.distributed as dist
        t = torch.from_numpy(model.g)
        dist.all_reduce(t)                      # in place on the numpy buffer
        return model.apply_adamw(samples_per_rank * self.world, hp, step, want_norm)


HP = {"lr": 1e-3, "clip": 0.5}


def _worker(rank, world, port, outdir):
    import torch.distributed as dist
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=timedelta(seconds=120))
    try:
        import dp
        import sa3k
        uid = dp.exchange_unique_id(rank, sa3k.dp_unique_id, dist.broadcast_object_list)
        model = OracleDora()
        tr = dp.DataParallelTrainer(model, GlooReduce(world))
        norms = []
        for step in range(3):
            tr.begin()
            for j in range(2):                  # 2 samples per rank per step
                tr.accumulate(1000 * step + 10 * rank + j, samples=1)
            norms.append(tr.apply(HP, want_norm=True))
        np.savez(os.path.join(outdir, f"r{rank}.npz"), p=model.p, uid=np.frombuffer(uid, np.uint8),
                 norms=np.array(norms))
    finally:
        dist.destroy_process_group()


def test_two_rank_gloo_step_matches_single_process(sa3k_lib):
    import torch.multiprocessing as mp
    world = 2
    with tempfile.TemporaryDirectory() as d:
        mp.start_processes(_worker, args=(world, _free_port(), d), nprocs=world, start_method="spawn")
        r0, r1 = np.load(os.path.join(d, "r0.npz")), np.load(os.path.join(d, "r1.npz"))
        assert np.array_equal(r0["uid"], r1["uid"])           # one clique id on every rank
        assert np.array_equal(r0["p"], r1["p"])               # identical adapters on every rank
        # one process that sees all 4 samples of each step
        import dp
        model = OracleDora()
        tr = dp.DataParallelTrainer(model)
        norms = []
        for step in range(3):
            tr.begin()
            for rank in range(world):
                for j in range(2):
                    tr.accumulate(1000 * step + 10 * rank + j, samples=1)
            norms.append(tr.apply(HP, want_norm=True))
        # (g00 + g01) + (g10 + g11) vs ((g00 + g01) + g10) + g11: equal up to f32 reassociation
        np.testing.assert_allclose(r0["p"], model.p, rtol=1e-5, atol=1e-6)
        np.testing.assert_allclose(r0["norms"], norms, rtol=1e-5)
        assert norms[0] > HP["clip"]                          # the clip path was exercised


def test_empty_batch_is_an_error():
    import dp
    tr = dp.DataParallelTrainer(OracleDora())
    tr.begin()
    with pytest.raises(ValueError):
        tr.apply(HP)


def _absent_peer_worker(rank, world, port, outdir):
    """Rank 1 joins the process group and leaves without taking part in the clique-id exchange;
    rank 0 must get an error from the exchange within the group's timeout instead of waiting."""
    import time
    import torch.distributed as dist
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=timedelta(seconds=3))
    if rank == 1:
        return   # leaves between steps: no collective of its own is in flight
    import dp
    import sa3k
    t0 = time.monotonic()
    try:
        dp.exchange_unique_id(rank, sa3k.dp_unique_id, dist.broadcast_object_list)
        outcome = "returned"
    except Exception as e:   # gloo reports the timeout or the closed peer connection
        outcome = f"raised {type(e).__name__}"
    with open(os.path.join(outdir, "r0.txt"), "w") as f:
        f.write(f"{outcome}\n{time.monotonic() - t0:.3f}\n")


def test_absent_peer_ends_the_exchange_with_an_error(sa3k_lib):
    import torch.multiprocessing as mp
    with tempfile.TemporaryDirectory() as d:
        mp.start_processes(_absent_peer_worker, args=(2, _free_port(), d), nprocs=2, start_method="spawn")
        lines = open(os.path.join(d, "r0.txt")).read().splitlines()
        assert lines[0].startswith("raised"), lines
        assert float(lines[1]) < 60.0
