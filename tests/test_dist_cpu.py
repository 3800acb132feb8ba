"""Host logic of row sharding, on CPU: shard bounds, and the helpers that
run over torch.distributed (unique-id broadcast, the global dense flag,
per-rank binning against rank 0's cuts) as two gloo ranks; and a rank that
leaves between steps, which the other learns of from its next collective."""

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


def _leaving_worker(rank, world, port, x, out):
    import datetime
    import time

    import torch.distributed as dist

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=10))
    if rank == 1:
        # this rank leaves between steps, before the sharding's collectives,
        # without a word to the others
        out.put((rank, "left", 0.0))
        out.close()
        out.join_thread()  # the message leaves before the process does
        os._exit(3)
    t0 = time.monotonic()
    try:
        hdist.shard_matrix(dist, x, 64)
        out.put((rank, "no error", time.monotonic() - t0))
    except Exception as err:  # noqa: BLE001 - the peer's departure, whatever its form
        out.put((rank, type(err).__name__, time.monotonic() - t0))
    out.close()
    out.join_thread()
    os._exit(0)


def test_gloo_rank_that_leaves_ends_the_others_collectives_with_an_error():
    # failure detection on the host: the remaining rank learns of the
    # departure from its next collective, which ends with an error within the
    # process group's timeout instead of waiting for good
    import torch.multiprocessing as mp

    x = np.random.default_rng(5).standard_normal((500, 4)).astype(np.float32)
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_leaving_worker, args=(r, 2, port, x, q)) for r in range(2)]
    for p in procs:
        p.start()
    res = dict((r, (what, dt)) for r, what, dt in [q.get(timeout=120) for _ in procs])
    for p in procs:
        p.join(timeout=60)
    assert procs[1].exitcode == 3
    assert procs[0].exitcode == 0
    what, dt = res[0]
    assert what != "no error", "the collective finished without its peer"
    assert dt < 60.0
