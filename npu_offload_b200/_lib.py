"""ctypes binding of libmoe_dp.so, the C ABI declared in include/moe_dp.h.

The library is built in-tree by ``python -m npu_offload_b200.build``.  Loading fails loudly when it
is missing: there is no CPU or PyTorch fallback for any operation of this package.
"""
import ctypes
import os
import re

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "libmoe_dp.so")
HEADER = os.path.join(os.path.dirname(HERE), "include", "moe_dp.h")

MOE_OK, MOE_EINVAL, MOE_ENONFINITE, MOE_ECUDA, MOE_ENOMEM, MOE_ESTATE, MOE_ETIMEOUT, MOE_ECOMM = range(8)
MOE_SCORING_SOFTMAX, MOE_SCORING_SIGMOID = 0, 1
MOE_F_HOST, MOE_F_ACCUMULATE, MOE_F_SYNC = 0x1, 0x2, 0x4
MOE_KIND_NONE, MOE_KIND_BF16, MOE_KIND_Q8 = 0, 1, 2
MOE_OPT_FUSED_DECODE, MOE_OPT_WAIT_TIMEOUT_US, MOE_OPT_INJECT_WAIT_TIMEOUT, MOE_OPT_TIMELINE = 1, 2, 3, 4
MOE_OPT_RING_STAGES, MOE_OPT_STAGE_BYTES, MOE_OPT_PREFILL_MIN_T, MOE_OPT_PREFILL_TC = 5, 6, 7, 8
MOE_OPT_LAYER_SLOTS, MOE_OPT_SHARED_INTER, MOE_OPT_Q8_UNIT_COST, MOE_OPT_REDUCERS, MOE_OPT_LATE_BYTES = 9, 10, 11, 12, 13
MOE_OPT_PLANNER = 14
MOE_EP_RECORD_BYTES = 256

STATUS_NAMES = {0: "MOE_OK", 1: "MOE_EINVAL", 2: "MOE_ENONFINITE", 3: "MOE_ECUDA", 4: "MOE_ENOMEM",
                5: "MOE_ESTATE", 6: "MOE_ETIMEOUT", 7: "MOE_ECOMM"}


class MoeConfig(ctypes.Structure):
    _fields_ = [("hidden", ctypes.c_int32), ("inter", ctypes.c_int32), ("n_experts", ctypes.c_int32),
                ("top_k", ctypes.c_int32), ("n_layers", ctypes.c_int32), ("max_tokens", ctypes.c_int32),
                ("scoring", ctypes.c_int32), ("device", ctypes.c_int32), ("ep_rank", ctypes.c_int32),
                ("ep_world", ctypes.c_int32), ("shard_map", ctypes.POINTER(ctypes.c_int32))]


class MoEError(RuntimeError):
    def __init__(self, status, msg):
        super().__init__(f"{STATUS_NAMES.get(status, status)}: {msg}")
        self.status = status


_vp = ctypes.c_void_p
_i = ctypes.c_int
_SIGS = {
    "moe_abi_version": (_i, []),
    "moe_last_error": (ctypes.c_char_p, []),
    "moe_create": (_i, [ctypes.POINTER(MoeConfig), ctypes.POINTER(_vp)]),
    "moe_destroy": (_i, [_vp]),
    "moe_load_expert_bf16": (_i, [_vp, _i, _i, _vp, _vp, _vp, _i]),
    "moe_load_expert_q8": (_i, [_vp, _i, _i, _vp, _vp, _i]),
    "moe_quantize_expert_q8": (_i, [_vp, _i, _i]),
    "moe_expert_kind": (_i, [_vp, _i, _i]),
    "moe_evict_expert": (_i, [_vp, _i, _i]),
    "moe_set_bias": (_i, [_vp, _i, _vp, _i]),
    "moe_forward": (_i, [_vp, _i, _i, _vp, _vp, _vp, _vp, _vp, _i, _vp]),
    "moe_forward_layers": (_i, [_vp, _i, _vp, _i, _vp, _vp, _vp, _i, _vp]),
    "moe_route": (_i, [_vp, _i, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _i, _vp]),
    "moe_experts": (_i, [_vp, _i, _vp, _i, _vp, _vp, _vp, _vp, _vp, _vp, _i, _vp]),
    "moe_ck_moe3": (_i, [_vp, _i, _vp, _vp, _vp, _vp, _i, _vp]),
    "moe_ck_moe_q8w": (_i, [_vp, _i, _vp, _vp, _vp, _vp, _vp, _i, _vp]),
    "moe_place_expert_q8": (_i, [_vp, _vp, _vp, _vp, _vp, _vp, _vp, _i, _vp]),
    "moe_status": (_i, [_vp, _vp]),
    "moe_launch_count": (ctypes.c_int64, [_vp]),
    "moe_ck_moe3_noalloc": (_i, [_i, _vp, _vp, _vp, _vp, _i, _i, _vp]),
    "moe_router_exp": (_i, [_vp, _vp, ctypes.c_int64, _vp]),
    "moe_load_shared": (_i, [_vp, _i, _vp, _vp, _vp, _vp, _i]),
    "moe_shared_router": (_i, [_vp, _i, _i, _vp, _vp, _vp, _vp, _i, _vp]),
    "moe_combine_residual": (_i, [_vp, _i, _vp, _vp, _vp, _vp, _i, _vp]),
    "moe_block_forward": (_i, [_vp, _i, _i, _vp, _vp, _vp, _vp, _vp, _vp, _i, _vp]),
    "moe_ep_export": (_i, [_vp, _vp, _i]),
    "moe_ep_import": (_i, [_vp, _vp, _i]),
    "moe_set_option": (_i, [_vp, _i, ctypes.c_int64]),
    "moe_timeline_read": (_i, [_vp, _vp, _i]),
    "moe_profile": (_i, [_vp, _i]),
    "moe_profile_read": (_i, [_vp, ctypes.POINTER(ctypes.c_double), _i, ctypes.POINTER(ctypes.c_int64)]),
}

_lib = None


def header_symbols():
    """Names of the entry points include/moe_dp.h declares."""
    with open(HEADER) as f:
        return sorted(set(re.findall(r"MOE_API\s+[\w\s\*]+?\b(moe_\w+)\s*\(", f.read())))


def lib():
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            raise ImportError(f"{LIB_PATH} is missing: build it with `python -m npu_offload_b200.build` "
                              "(there is no fallback implementation)")
        L = ctypes.CDLL(LIB_PATH)
        for name, (res, args) in _SIGS.items():
            fn = getattr(L, name)
            fn.restype = res
            fn.argtypes = args
        _lib = L
    return _lib


def last_error():
    return lib().moe_last_error().decode(errors="replace")


def check(status):
    if status != MOE_OK:
        raise MoEError(status, last_error())
    return status
