"""Build recipe for the CPU checkers (test infrastructure, never the product).

* ``oracle/libmoe_oracle.so`` -- the plain-C restatement in ``moe_oracle.c``.
* ``oracle/_ref/libcpu_kern.so`` -- the reference's own ``track2_opt/solar_engine/csrc/cpu_kern.c``,
  compiled in place from the read-only reference tree (nothing is copied into this repository).
* ``oracle/_ref/cpu_moe_build/cpu_moe_ext.so`` -- the reference's own ``solar_hybrid/cpu_moe.cpp``
  torch extension (``cpu_moe`` / ``set_threads``), built the way ``solar_hybrid/cpu_moe_ext.py:5-8``
  builds it, with ``CXX=/usr/bin/g++``.

The reference's flags are ``-O3 -march=sapphirerapids -fopenmp``; ``REF_ISA`` below names the
same AVX-512 BF16/VNNI instruction sets explicitly so the binaries also run on AVX-512 BF16 hosts
that are not Sapphire Rapids (AMD Zen 4/5).  The reference tree only exists in the build
container; on a GPU box the prebuilt ``oracle/_ref`` files are used as they are.

Usage: ``python oracle/build.py`` (also called from ``__graft_entry__.build()``).
"""
import os
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
# The reference tree: $NPU_OFFLOAD_REF, else a directory named "reference" beside this repository.
REF_ROOT = os.environ.get("NPU_OFFLOAD_REF") or os.path.join(os.path.dirname(os.path.dirname(HERE)), "reference")
REF_DIR = os.path.join(HERE, "_ref")
ORACLE_SO = os.path.join(HERE, "libmoe_oracle.so")
CPU_KERN_SO = os.path.join(REF_DIR, "libcpu_kern.so")
CPU_MOE_DIR = os.path.join(REF_DIR, "cpu_moe_build")
CPU_MOE_SO = os.path.join(CPU_MOE_DIR, "cpu_moe_ext.so")

REF_ISA = ["-march=x86-64-v3", "-mavx512f", "-mavx512bw", "-mavx512vl", "-mavx512dq", "-mavx512cd",
           "-mavx512bf16", "-mavx512vnni"]
GCC = "/usr/bin/gcc" if os.path.exists("/usr/bin/gcc") else "gcc"
GXX = "/usr/bin/g++" if os.path.exists("/usr/bin/g++") else "g++"


def _newer(target, *sources):
    if not os.path.exists(target):
        return False
    t = os.path.getmtime(target)
    return all(os.path.getmtime(s) <= t for s in sources if os.path.exists(s))


def build_oracle(force=False):
    src = os.path.join(HERE, "moe_oracle.c")
    if not force and _newer(ORACLE_SO, src):
        return ORACLE_SO
    cmd = [GCC, "-O2", "-fno-fast-math", "-ffp-contract=off", "-fopenmp", "-shared", "-fPIC", "-std=c11",
           src, "-o", ORACLE_SO, "-lm"]
    subprocess.check_call(cmd)
    return ORACLE_SO


def ref_available():
    return os.path.isdir(os.path.join(REF_ROOT, "solar_hybrid"))


def build_ref(force=False):
    """Compile the reference's CPU kernels from the reference tree (build container only)."""
    if not ref_available():
        return None
    os.makedirs(REF_DIR, exist_ok=True)
    kern_src = os.path.join(REF_ROOT, "track2_opt", "solar_engine", "csrc", "cpu_kern.c")
    if force or not _newer(CPU_KERN_SO, kern_src):
        subprocess.check_call([GCC, "-O3", *REF_ISA, "-fopenmp", "-shared", "-fPIC", kern_src, "-o", CPU_KERN_SO,
                               "-lm"])
    moe_src = os.path.join(REF_ROOT, "solar_hybrid", "cpu_moe.cpp")
    if force or not _newer(CPU_MOE_SO, moe_src):
        os.makedirs(CPU_MOE_DIR, exist_ok=True)
        env_cxx = os.environ.get("CXX")
        os.environ["CXX"] = GXX
        try:
            from torch.utils.cpp_extension import load
            load(name="cpu_moe_ext", sources=[moe_src], extra_cflags=["-O3", *REF_ISA, "-fopenmp"],
                 extra_ldflags=["-fopenmp"], build_directory=CPU_MOE_DIR, verbose=False)
        finally:
            if env_cxx is None:
                os.environ.pop("CXX", None)
            else:
                os.environ["CXX"] = env_cxx
    return REF_DIR


def main():
    force = "--force" in sys.argv
    print("oracle:", build_oracle(force))
    r = build_ref(force)
    print("reference:", r if r else "reference tree absent; using prebuilt oracle/_ref if present")


if __name__ == "__main__":
    main()
