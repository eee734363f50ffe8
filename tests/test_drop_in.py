"""Host logic of the gpu_moe drop-in (no GPU): the cache of device copies of CPU weight tensors.

Runtime._cpu_experts (solar_hybrid/runtime.py:322-336) hands cpu_moe the CPU weight tensors of every
layer's cold experts and swaps experts in place; the cache must neither grow without bound nor
return a stale copy for a tensor that was rewritten or freed and reallocated."""
import gc

import torch

from npu_offload_b200.moe import _WeightCache


def _w(n=1024, v=1.0):
    return torch.full((n,), v, dtype=torch.bfloat16)


def test_hit_on_the_same_unchanged_tensor():
    c = _WeightCache(1 << 20)
    t = _w()
    a = c.get(t, "meta")
    assert c.get(t, "meta") is a
    assert len(c.entries) == 1 and c.bytes == t.numel() * 2


def test_in_place_write_is_copied_again():
    c = _WeightCache(1 << 20)
    t = _w()
    a = c.get(t, "meta")
    t.add_(1)  # an in-place expert swap bumps the version counter
    b = c.get(t, "meta")
    assert b is not a and len(c.entries) == 1 and c.bytes == t.numel() * 2


def test_entries_die_with_their_tensor():
    c = _WeightCache(1 << 20)
    t = _w()
    c.get(t, "meta")
    del t
    gc.collect()
    assert len(c.entries) == 0 and c.bytes == 0


def test_byte_limit_evicts_least_recently_used():
    t = [_w(1024, i) for i in range(4)]  # 2 KiB each
    c = _WeightCache(3 * 2048)
    for x in t[:3]:
        c.get(x, "meta")
    c.get(t[0], "meta")  # t[0] becomes the most recently used
    c.get(t[3], "meta")  # evicts t[1]
    ids = set(c.entries)
    assert id(t[1]) not in ids and {id(t[0]), id(t[2]), id(t[3])} <= ids
    assert c.bytes == 3 * 2048


def test_tensor_larger_than_the_limit_is_not_kept():
    c = _WeightCache(1000)
    t = _w(1024)
    d = c.get(t, "meta")
    assert d.shape == t.shape and len(c.entries) == 0 and c.bytes == 0
