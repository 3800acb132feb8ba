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


def broadcast_unique_id(dist, make_id):
    """Rank 0's NCCL unique id on every rank (`dist` = torch.distributed)."""
    import torch

    buf = torch.zeros(128, dtype=torch.uint8)
    if dist.get_rank() == 0:
        buf[:] = torch.from_numpy(np.frombuffer(make_id(), dtype=np.uint8).copy())
    dist.broadcast(buf, src=0)
    return bytes(buf.numpy().tobytes())


def unique_id():
    import ctypes

    from . import _check, lib

    buf = (ctypes.c_uint8 * 128)()
    _check(lib().hb_comm_unique_id(buf), "hb_comm_unique_id")
    return bytes(buf)
