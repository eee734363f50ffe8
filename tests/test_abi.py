"""C-ABI boundary checks that need no GPU: the library loads, exports every declared entry point,
and rejects bad arguments with a status code instead of crashing."""
import ctypes

import pytest

import npu_offload_b200 as nob
from npu_offload_b200 import _lib
from tests.conftest import has_gpu


def test_library_exports_every_declared_symbol():
    L = nob.lib()
    declared = nob.header_symbols()
    assert len(declared) >= 17
    missing = [s for s in declared if not hasattr(L, s)]
    assert not missing, missing
    assert set(declared) == set(_lib._SIGS), "binding table out of sync with include/moe_dp.h"
    assert L.moe_abi_version() == 1


def _cfg(**kw):
    base = dict(hidden=4096, inter=1280, n_experts=128, top_k=8, n_layers=1, max_tokens=16, scoring=0, device=0,
                ep_rank=0, ep_world=1, shard_map=None)
    base.update(kw)
    return _lib.MoeConfig(*[base[k] for k, _ in _lib.MoeConfig._fields_])


@pytest.mark.parametrize("kw,needle", [
    (dict(hidden=100), "hidden"),
    (dict(inter=1000), "inter"),
    (dict(n_experts=0), "n_experts"),
    (dict(n_experts=300), "n_experts"),
    (dict(top_k=17), "top_k"),
    (dict(top_k=9, n_experts=8), "top_k"),
    (dict(max_tokens=0), "max_tokens"),
    (dict(max_tokens=5000), "max_tokens"),
    (dict(scoring=7), "scoring"),
    (dict(ep_rank=2, ep_world=2), "ep"),
    (dict(n_layers=0), "n_layers"),
])
def test_create_rejects_bad_config(kw, needle):
    h = ctypes.c_void_p()
    st = nob.lib().moe_create(ctypes.byref(_cfg(**kw)), ctypes.byref(h))
    assert st == _lib.MOE_EINVAL
    assert needle in _lib.last_error()
    assert not h.value


def test_null_arguments_return_status():
    L = nob.lib()
    assert L.moe_create(None, None) == _lib.MOE_EINVAL
    assert L.moe_forward(None, 0, 1, None, None, None, None, None, 0, None) == _lib.MOE_EINVAL
    assert L.moe_forward_layers(None, 1, None, 1, None, None, None, 0, None) == _lib.MOE_EINVAL
    assert L.moe_route(None, 1, None, None, None, None, None, None, None, None, None, 0, None) == _lib.MOE_EINVAL
    assert L.moe_experts(None, 1, None, 0, None, None, None, None, None, None, 0, None) == _lib.MOE_EINVAL
    assert L.moe_status(None, None) == _lib.MOE_EINVAL
    assert L.moe_load_expert_bf16(None, 0, 0, None, None, None, 0) == _lib.MOE_EINVAL
    assert L.moe_destroy(None) == _lib.MOE_OK
    assert L.moe_expert_kind(None, 0, 0) == -1
    assert L.moe_launch_count(None) == -1


@pytest.mark.skipif(has_gpu(), reason="checks the no-device error path")
def test_create_without_gpu_reports_cuda_error():
    h = ctypes.c_void_p()
    st = nob.lib().moe_create(ctypes.byref(_cfg()), ctypes.byref(h))
    assert st == _lib.MOE_ECUDA
    assert "device" in _lib.last_error()


def test_cpu_moe_dropin_validates_shapes_before_touching_gpu():
    import torch
    from npu_offload_b200.moe import gpu_moe
    x = torch.zeros(1, 48, dtype=torch.bfloat16)
    with pytest.raises(RuntimeError, match="multiples of 32"):
        gpu_moe(x, [torch.zeros(64, 48, dtype=torch.bfloat16)], [torch.zeros(48, 32, dtype=torch.bfloat16)],
                [torch.zeros(1, dtype=torch.long)], [torch.ones(1)])
    # no experts -> zeros, like the reference (cpu_moe.cpp:42-43)
    out = gpu_moe(torch.zeros(3, 64, dtype=torch.bfloat16), [], [], [], [])
    assert out.shape == (3, 64) and out.dtype == torch.float32 and float(out.abs().sum()) == 0.0


def test_header_constants_match_the_python_binding():
    """Every status code, flag, scoring mode, expert kind and option number the header defines has
    the same value in the Python binding, and the binding defines no option the header lacks."""
    import re
    from npu_offload_b200 import _lib
    defs = {}
    with open(_lib.HEADER) as f:
        for line in f:
            m = re.match(r"#define (MOE_[A-Z0-9_]+) (0x[0-9a-fA-F]+|\d+)\b", line)
            if m and m.group(1) not in ("MOE_DP_ABI_VERSION",):
                defs[m.group(1)] = int(m.group(2), 0)
    assert len(defs) > 30
    for name, value in defs.items():
        assert hasattr(_lib, name), f"{name} missing from the binding"
        assert getattr(_lib, name) == value, f"{name}: header {value}, binding {getattr(_lib, name)}"
    py_opts = {n for n in dir(_lib) if n.startswith("MOE_OPT_")}
    assert py_opts == {n for n in defs if n.startswith("MOE_OPT_")}
