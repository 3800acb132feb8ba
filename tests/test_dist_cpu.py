"""Host logic of row sharding, on CPU: shard bounds, and the helpers that
run over torch.distributed (unique-id broadcast, the global dense flag,
per-rank binning against rank 0's cuts) as two gloo ranks."""

import os
import socket

import numpy as np
import pytest

import hessboost_b200 as H
from hessboost_b200 import dist as hdist


@pytest.mark.parametrize("n", [0, 1, 7, 8, 9, 1000, 100_003])
@pytest.mark.parametrize("world", [1, 2, 3, 4, 8])
def test_shard_bounds_cover_rows_on_multiples_of_8(n, world):
    pieces = [hdist.shard_bounds(n, world, r) for r in range(world)]
    assert pieces[0][0] == 0 and pieces[-1][1] == n
    for (b0, e0), (b1, e1) in zip(pieces, pieces[1:]):
        assert e0 == b1
    for b, e in pieces:
        assert b <= e and (b % 8 == 0 or b == n)


def test_shard_bounds_refuses_bad_rank():
    with pytest.raises(ValueError):
        hdist.shard_bounds(10, 2, 2)


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, x, out):
    import torch.distributed as dist

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        uid = hdist.broadcast_unique_id(dist, lambda: bytes(range(128)) if rank == 0 else b"")
        # rank 1's shard is dense, rank 0's is not: the global flag is False
        flag = hdist.all_dense(dist, rank == 1)
        m, begin, end = hdist.shard_matrix(dist, x, 64)
        out.put((rank, uid, flag, begin, end, m.columns, None if m.missing is None else m.missing,
                 m.dense, m.feature_offset, m.cut_values))
    finally:
        dist.destroy_process_group()


def test_gloo_two_ranks_shard_the_matrix():
    import torch.multiprocessing as mp

    rng = np.random.default_rng(4)
    n = 1003
    x = rng.standard_normal((n, 6)).astype(np.float32)
    x[rng.random(x.shape) < 0.05] = np.nan
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, x, q)) for r in range(2)]
    for p in procs:
        p.start()
    res = sorted([q.get(timeout=120) for _ in procs], key=lambda t: t[0])
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    whole = H.BinnedMatrix.from_dense(x, 64)
    for rank, uid, flag, begin, end, cols, miss, dense, off, cuts in res:
        assert uid == bytes(range(128))
        assert flag is False
        assert (begin, end) == hdist.shard_bounds(n, 2, rank)
        np.testing.assert_array_equal(off, whole.feature_offset)
        np.testing.assert_array_equal(cuts.view(np.uint32), whole.cut_values.view(np.uint32))
        np.testing.assert_array_equal(cols, whole.columns[:, begin:end])
        assert dense == whole.dense
        bits = np.unpackbits(whole.missing.view(np.uint8), bitorder="little").reshape(6, -1)[:, begin:end]
        got = np.unpackbits(miss.view(np.uint8), bitorder="little").reshape(6, -1)[:, : end - begin]
        np.testing.assert_array_equal(got, bits)
