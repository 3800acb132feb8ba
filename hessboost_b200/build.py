"""Build libhb_cuda.so (the C-ABI library of the CUDA hist path) in-tree.

``python -m hessboost_b200.build`` compiles every source under ``csrc/`` with
nvcc for sm_100a into ``hessboost_b200/_lib/libhb_cuda.so``; no GPU is
needed to build.
"""

import os
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
CSRC = os.path.join(HERE, "csrc")
OUT_DIR = os.path.join(HERE, "_lib")
LIB = os.path.join(OUT_DIR, "libhb_cuda.so")
SOURCES = ["hb_kernels.cu", "hb_engine.cu", "hb_peer.cu", "hb_predict.cu", "hb_noalloc.cu", "hb_probe.cu", "hb_sketch.cu",
           "hb_host_bins.cpp", "hb_model_io.cpp"]
NVCC = os.environ.get("NVCC", "/usr/local/cuda/bin/nvcc")
FLAGS = [
    "-gencode", "arch=compute_100a,code=sm_100a",
    "-O3", "-lineinfo", "-std=c++17", "-fmad=false",
    "-Xcompiler", "-fPIC,-O3", "-shared", "-ccbin", "/usr/bin/g++",
]


def needs_build():
    if not os.path.exists(LIB):
        return True
    t = os.path.getmtime(LIB)
    deps = [os.path.join(CSRC, f) for f in os.listdir(CSRC)]
    deps.append(os.path.join(os.path.dirname(HERE), "include", "hb_backend.h"))
    return any(os.path.getmtime(d) > t for d in deps)


def nccl_runpath():
    """The NCCL that PyTorch ships (the nvidia-nccl wheel), searched first at
    run time so that this library and torch share one libnccl.so.2; None
    when the wheel is absent (the system NCCL is used)."""
    try:
        import importlib.util

        spec = importlib.util.find_spec("nvidia.nccl")
    except (ImportError, ValueError):
        return None
    for root in list(getattr(spec, "submodule_search_locations", None) or []):
        d = os.path.join(root, "lib")
        if os.path.exists(os.path.join(d, "libnccl.so.2")):
            return d
    return None


def build(force=False, verbose=False):
    if not force and not needs_build():
        return LIB
    os.makedirs(OUT_DIR, exist_ok=True)
    cmd = [NVCC, *FLAGS, "-o", LIB, *[os.path.join(CSRC, s) for s in SOURCES], "-lnccl"]
    rp = nccl_runpath()
    if rp:
        cmd += ["-Xlinker", "-rpath=" + rp]
    if verbose:
        print(" ".join(cmd))
    subprocess.run(cmd, check=True)
    return LIB


if __name__ == "__main__":
    print(build(force="--force" in sys.argv, verbose=True))
