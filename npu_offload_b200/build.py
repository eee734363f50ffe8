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
SOURCES = ["moe_dp.cu", "route.cu", "experts.cu", "decode.cu", "noalloc.cu", "prefill.cu", "prefill_tc.cu",
           "block.cu"]


def cute_include():
    """CuTe / CUTLASS headers (descriptor and type definitions for the tcgen05 kernels): the header
    tree vendored with flashinfer, or $CUTLASS_INCLUDE."""
    cand = [os.environ.get("CUTLASS_INCLUDE", "")]
    try:
        import importlib.util
        spec = importlib.util.find_spec("flashinfer")
        if spec and spec.submodule_search_locations:
            cand.append(os.path.join(list(spec.submodule_search_locations)[0], "data", "cutlass", "include"))
    except Exception:
        pass
    for d in cand:
        if d and os.path.exists(os.path.join(d, "cute", "arch", "mma_sm100_desc.hpp")):
            return [d]
    raise RuntimeError("CuTe headers not found: set CUTLASS_INCLUDE to a CUTLASS include directory")


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


def build(force=False, verbose=False, extra=(), out=None):
    """Compiles every source to an object in parallel (objects under _build/), then links the library.
    extra: additional nvcc flags; out: library path (default: the in-tree libmoe_dp.so)."""
    lib = out or LIB
    if not force and out is None and up_to_date():
        return lib
    srcs, _ = sources()
    tag = str(abs(hash((tuple(extra), lib))) % (1 << 32))
    objdir = os.path.join(HERE, "_build", tag)
    os.makedirs(objdir, exist_ok=True)
    common = [NVCC, *ARCH, "-O3", "-lineinfo", "-std=c++17", "-Xcompiler", "-fPIC,-fvisibility=hidden",
              "-I", os.path.join(ROOT, "include"), "-I", CSRC, *[a for d in cute_include() for a in ("-I", d)], *extra]
    if verbose:
        common.insert(1, "-Xptxas=-v")
    jobs = []
    for src in srcs:
        obj = os.path.join(objdir, os.path.basename(src) + ".o")
        cmd = [*common, "-c", src, "-o", obj]
        if verbose:
            print(" ".join(cmd))
        jobs.append((obj, subprocess.Popen(cmd)))
    failed = [obj for obj, p in jobs if p.wait() != 0]
    if failed:
        raise subprocess.CalledProcessError(1, "nvcc " + " ".join(failed))
    link = [NVCC, *ARCH, "-shared", "-o", lib + ".tmp", *[obj for obj, _ in jobs], "-lcudart"]
    subprocess.check_call(link)
    os.replace(lib + ".tmp", lib)
    return lib


if __name__ == "__main__":
    print(build(force="--force" in sys.argv, verbose="-v" in sys.argv))
