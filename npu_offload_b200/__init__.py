"""B200-native routed-expert MoE data plane (npu-offload's cpu_moe / expert-dispatch path on sm_100a).

The compute lives in libmoe_dp.so (hand-written CUDA for sm_100a behind the C ABI of
include/moe_dp.h); this package is its host-side binding.
"""
from ._lib import MoEError, header_symbols, lib  # noqa: F401

__version__ = "0.1.0"


def __getattr__(name):
    # torch-dependent API loaded on first use so `import npu_offload_b200` stays light
    if name in ("MoEDataPlane", "gpu_moe", "set_threads", "as_bf16"):
        from . import moe
        return getattr(moe, name)
    raise AttributeError(name)
