"""Row-sharded training on two GPUs (torch.distributed.run, one process per
GPU, NCCL) grows the same forest, bit for bit, as one GPU on the whole
matrix: the histograms are exact integer sums."""

import os
import socket
import subprocess
import sys

import numpy as np
import pytest

import hessboost_b200 as H

pytestmark = pytest.mark.gpu

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, HERE)
import mgpu_worker  # noqa: E402


def _gpus():
    import torch

    return torch.cuda.device_count()


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


@pytest.mark.skipif("_gpus() < 2")
@pytest.mark.parametrize("exchange", ["peer", "nccl"])
def test_two_gpus_grow_the_one_gpu_forest(tmp_path, exchange):
    """Both level-histogram exchanges: NCCL's allreduce (the default) and
    the peer-memory one (HB_PEER_ALLREDUCE=1)."""
    out = tmp_path / "sharded.npz"
    cmd = ["timeout", "-k", "30", "600", sys.executable, "-m", "torch.distributed.run", "--nnodes=1",
           "--nproc-per-node", "2", "--master-addr", "127.0.0.1", "--master-port", str(_free_port()),
           os.path.join(HERE, "mgpu_worker.py"), str(out)]
    env = dict(os.environ, HB_PEER_ALLREDUCE="1" if exchange == "peer" else "0", NCCL_NVLS_ENABLE="0")
    r = subprocess.run(cmd, capture_output=True, text=True, env=env)
    assert r.returncode == 0, r.stdout[-3000:] + r.stderr[-3000:]
    got = np.load(out)
    for name, x, y, params, rounds in mgpu_worker.cases():
        one = H.train(params, x, y, rounds)
        np.testing.assert_array_equal(got[f"{name}_ptr"], one.tree_ptr, err_msg=name)
        assert got[f"{name}_base"] == np.float32(one.base)
        a, b = got[f"{name}_nodes"], one.nodes
        for k in a.dtype.names:
            np.testing.assert_array_equal(a[k].view(np.uint32) if a[k].dtype == np.float32 else a[k],
                                          b[k].view(np.uint32) if b[k].dtype == np.float32 else b[k],
                                          err_msg=f"{name} {k}")
