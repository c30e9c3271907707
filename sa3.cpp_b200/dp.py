"""Data-parallel adapter training, one process per GPU (host side).

Every rank runs the forward + backward of its own samples into its flat gradient buffer; the
buffers are summed across ranks and every rank applies the same averaged, clipped AdamW update
with count = samples per rank x ranks.  That is the reference's per-sample host accumulation
(src/train_loop.h:84-134, tools/sa3-train.cpp:709-714) followed by train_average_and_clip
(src/train_loop.h:147-171) and AdamW (src/train_optimizer.h:42-65), spread over GPUs.

The exchange itself is pluggable: `SumAllReduce` objects have `allreduce_adamw(model,
samples_per_rank, hp, step, want_norm)`.  `NcclReduce` is the product path (one sa3k call: NCCL
all-reduce on the context's stream, then the AdamW kernels); tests plug in a gloo-backed one.
"""


def exchange_unique_id(rank, make_id, broadcast_object):
    """Rank 0 makes the clique id, every rank returns the same bytes.

    make_id() -> bytes (only called on rank 0); broadcast_object(obj_list, src) is a
    torch.distributed.broadcast_object_list-like callable."""
    box = [make_id() if rank == 0 else None]
    broadcast_object(box, 0)
    uid = box[0]
    if not isinstance(uid, (bytes, bytearray)) or len(uid) != 128:
        raise RuntimeError("clique id exchange failed")
    return bytes(uid)


class NcclReduce:
    """The sa3k NCCL path: all-reduce + AdamW in one library call on the model's flat state."""

    def __init__(self, comm):
        self.comm = comm
        self.world = comm.nranks

    def allreduce_adamw(self, model, samples_per_rank, hp, step, want_norm=False):
        return model.dp_apply_adamw(self.comm, samples_per_rank, hp, step, want_norm=want_norm)


class LocalReduce:
    """One rank: no exchange."""
    world = 1

    def allreduce_adamw(self, model, samples_per_rank, hp, step, want_norm=False):
        return model.apply_adamw(samples_per_rank, hp, step, want_norm=want_norm)


class DataParallelTrainer:
    """The step loop of one rank: zero_grads, forward_backward over this rank's samples (any
    number of calls), then the exchange + update."""

    def __init__(self, model, reduce=None):
        self.model = model
        self.reduce = reduce or LocalReduce()
        self.step_count = 0
        self.samples = 0

    def begin(self):
        self.model.zero_grads()
        self.samples = 0

    def accumulate(self, *args, samples=None, **kw):
        """model.forward_backward(*args, **kw); its sample count is args[0] (the batch size of
        sa3k.Dit.forward_backward) unless `samples` is given."""
        self.model.forward_backward(*args, **kw)
        self.samples += args[0] if samples is None else samples

    def apply(self, hp, want_norm=False):
        if self.samples <= 0:
            raise ValueError("cannot apply empty gradient batch")
        self.step_count += 1
        return self.reduce.allreduce_adamw(self.model, self.samples, hp, self.step_count, want_norm=want_norm)
