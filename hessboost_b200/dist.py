"""Row sharding over several GPUs of one node (one process per GPU).

Each rank owns a contiguous block of rows whose first row is a multiple of
8 (the logistic gradient's 8-row vectors then line up with the whole
matrix's, src/objective/mod.rs:195) and grows the same tree: its engine
sums every histogram, root total and gradient maximum over the ranks with
NCCL (``hb_comm_init``). torch.distributed only carries the NCCL unique id
and the barriers.
"""

import numpy as np


def shard_bounds(n_rows, world, rank):
    """[begin, end) of `rank`'s rows: near-equal blocks starting on
    multiples of 8."""
    if world < 1 or not 0 <= rank < world:
        raise ValueError("bad world/rank")
    per = -(-n_rows // world)
    per = -(-per // 8) * 8
    begin = min(n_rows, rank * per)
    end = min(n_rows, begin + per)
    return begin, end


def _collective_device(dist):
    import torch

    if dist.get_backend() == "nccl":
        return torch.device("cuda", torch.cuda.current_device())
    return torch.device("cpu")


def broadcast_unique_id(dist, make_id):
    """Rank 0's NCCL unique id on every rank (`dist` = torch.distributed)."""
    import torch

    buf = torch.zeros(128, dtype=torch.uint8, device=_collective_device(dist))
    if dist.get_rank() == 0:
        buf.copy_(torch.from_numpy(np.frombuffer(make_id(), dtype=np.uint8).copy()))
    dist.broadcast(buf, src=0)
    return bytes(buf.cpu().numpy().tobytes())


def all_dense(dist, local_dense):
    """The whole matrix's `dense` flag (every row of every shard complete):
    the split scan's backward pass depends on it, so every rank must use
    the global value, not its shard's."""
    import torch

    t = torch.tensor([1 if local_dense else 0], dtype=torch.int32, device=_collective_device(dist))
    dist.all_reduce(t, op=dist.ReduceOp.MIN)
    return bool(int(t.item()))


def whole_matrix_cuts(x, max_bin, device=None):
    """Cuts of the whole matrix: the device sketch on `device` when given
    (hb_sketch_dense), else, or where it refuses the input, the host sketch;
    both give the same cuts."""
    from . import HB_REFUSED, HbError, cuts_dense, sketch_dense

    if device is not None:
        try:
            off, cuts, _, _, _ = sketch_dense(x, max_bin, device, bins=False)
            return off, cuts
        except HbError as err:
            if err.status != HB_REFUSED:
                raise
    return cuts_dense(x, max_bin)


def shard_matrix(dist, x, max_bin, device=None):
    """This rank's rows of `x` (every rank holds the same `x`), binned
    against cuts rank 0 computes over the whole matrix (on its GPU
    `device` when given): (BinnedMatrix, begin, end)."""
    from . import BinnedMatrix, bin_dense

    world, rank = dist.get_world_size(), dist.get_rank()
    obj = list(whole_matrix_cuts(x, max_bin, device)) if rank == 0 else [None, None]
    dist.broadcast_object_list(obj, src=0)
    off, cuts = obj
    begin, end = shard_bounds(x.shape[0], world, rank)
    cols, miss, dense = bin_dense(x[begin:end], off, cuts)
    return BinnedMatrix(off, cuts, cols, miss, all_dense(dist, dense)), begin, end


def train_sharded(params, x, y, rounds, dist, device=None):
    """Row-sharded training over the ranks of `dist` (torch.distributed, one
    process per GPU, every rank passing the same `x`, `y`): rank r uploads
    its own block of rows, every histogram is summed over the ranks with
    NCCL, and every rank returns the same Model, identical to one-GPU
    training of the whole matrix."""
    import torch

    from . import Engine, Model, base_margin

    params.validate()
    world, rank = dist.get_world_size(), dist.get_rank()
    if device is None:
        device = torch.cuda.current_device()
    n = x.shape[0]
    shard, begin, end = shard_matrix(dist, x, params.max_bin, device)
    y = np.ascontiguousarray(y, np.float32)
    base = base_margin(params, y)
    eng = Engine(device)
    try:
        eng.set_shard(begin, n)
        eng.comm_init(world, rank, broadcast_unique_id(dist, unique_id), n)
        eng.upload(shard)
        nodes, tree_ptr = eng.train(params, y[begin:end], rounds, base)
    finally:
        eng.close()
    return Model(nodes, tree_ptr, float(base), x.shape[1])


def unique_id():
    import ctypes

    from . import _check, lib

    buf = (ctypes.c_uint8 * 128)()
    _check(lib().hb_comm_unique_id(buf), "hb_comm_unique_id")
    return bytes(buf)
