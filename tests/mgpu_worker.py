"""One rank of the multi-GPU parity test (run by torch.distributed.run):
row-sharded training with hessboost_b200.dist.train_sharded; rank 0 saves
the model to the path given as the first argument."""

import os
import sys
from datetime import timedelta

import numpy as np
import torch
import torch.distributed as dist

sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))

import hessboost_b200 as H  # noqa: E402
from hessboost_b200 import dist as hdist  # noqa: E402
from hessboost_b200 import synth  # noqa: E402


def cases():
    x, y = synth.logistic_c2(200_003, 28, seed=17)
    yield "logistic", x, y, H.TrainingParams(objective="binary:logistic", max_depth=8, eta=0.1), 4
    x, y = synth.regression_c1(60_001, 28, seed=3)
    yield "regression", x, y, H.TrainingParams(objective="reg:squarederror", max_depth=6, eta=0.1), 4
    x, y = synth.logistic_c2(100_003, 12, seed=21)
    yield "monotone", x, y, H.TrainingParams(objective="binary:logistic", max_depth=6, eta=0.3,
                                             monotone_constraints=(1, -1, 0, 1)), 3


def main():
    local = int(os.environ["LOCAL_RANK"])
    torch.cuda.set_device(local)
    dist.init_process_group("nccl", timeout=timedelta(seconds=120), device_id=torch.device("cuda", local))
    out = {}
    try:
        for name, x, y, params, rounds in cases():
            m = hdist.train_sharded(params, x, y, rounds, dist)
            out[f"{name}_nodes"] = m.nodes
            out[f"{name}_ptr"] = m.tree_ptr
            out[f"{name}_base"] = np.float32(m.base)
        dist.barrier()
    finally:
        dist.destroy_process_group()
    if int(os.environ["RANK"]) == 0:
        np.savez(sys.argv[1], **out)


if __name__ == "__main__":
    main()
