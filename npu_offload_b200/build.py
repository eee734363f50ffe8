"""Build libmoe_dp.so (the C-ABI library) in-tree with nvcc for sm_100a.

    python -m npu_offload_b200.build [--force]

The library lands next to this file (npu_offload_b200/libmoe_dp.so), so it travels with the source
tree to a GPU host; nothing is installed into site-packages or a JIT cache.
"""
import os
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
CSRC = os.path.join(HERE, "csrc")
ROOT = os.path.dirname(HERE)
LIB = os.path.join(HERE, "libmoe_dp.so")
NVCC = os.environ.get("NVCC", "/usr/local/cuda/bin/nvcc")
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
SOURCES = ["moe_dp.cu", "route.cu", "experts.cu", "decode.cu", "plan.cu", "noalloc.cu"]


def sources():
    srcs = [os.path.join(CSRC, s) for s in SOURCES]
    deps = srcs + [os.path.join(CSRC, f) for f in os.listdir(CSRC) if f.endswith((".cuh", ".h"))]
    deps.append(os.path.join(ROOT, "include", "moe_dp.h"))
    return srcs, deps


def up_to_date():
    if not os.path.exists(LIB):
        return False
    t = os.path.getmtime(LIB)
    return all(os.path.getmtime(d) <= t for d in sources()[1])


def build(force=False, verbose=False, extra=()):
    if not force and up_to_date():
        return LIB
    srcs, _ = sources()
    cmd = [NVCC, *ARCH, "-O3", "-lineinfo", "-std=c++17", "-shared", "-Xcompiler", "-fPIC,-fvisibility=hidden",
           "-I", os.path.join(ROOT, "include"), "-I", CSRC, "-o", LIB + ".tmp", *srcs, "-lcudart", *extra]
    if verbose:
        cmd.insert(1, "-Xptxas=-v")
        print(" ".join(cmd))
    subprocess.check_call(cmd)
    os.replace(LIB + ".tmp", LIB)
    return LIB


if __name__ == "__main__":
    print(build(force="--force" in sys.argv, verbose="-v" in sys.argv))
