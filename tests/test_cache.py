"""HBM-hot / host-cold expert tier (the reference's LFU-decay follow, solar_hybrid/runtime.py:287-311,
and slot swap, experts_b.rs:162-186): the policy on the CPU, the served layers on a GPU against the
oracle with every expert."""
import numpy as np
import pytest

from npu_offload_b200.cache import SWAP_MIN, choose_victim, follow_candidate


def test_victim_is_the_coldest_unneeded_resident():
    recent = np.array([5.0, 1.0, 1.0, 9.0, 0.5])
    assert choose_victim(recent, {0, 1, 2, 3}, need={0}) == 1  # tie 1/2 -> lower id
    assert choose_victim(recent, {0, 1, 2, 3}, need={1, 2}) == 0
    assert choose_victim(recent, {0, 3}, need={0, 3}) is None


def test_follow_rule_matches_the_reference_threshold():
    E = 8
    recent = np.zeros(E)
    recent[[0, 1, 2]] = [3.0, 1.0, 4.0]
    # hottest non-resident (2, count 4) against the coldest resident (1, count 1): 4 >= 2*1 + 2 -> swap
    assert follow_candidate(recent, {0, 1}, E) == (2, 1)
    recent[2] = 3.9
    assert follow_candidate(recent, {0, 1}, E) is None  # 3.9 < 2*1 + SWAP_MIN
    assert SWAP_MIN == 2
    assert follow_candidate(np.zeros(E), {0}, E) is None  # nothing used: no candidate


@pytest.mark.gpu
def test_cache_layers_match_the_oracle_with_every_expert():
    import torch
    from npu_offload_b200 import synth
    from npu_offload_b200._lib import MoEError
    from npu_offload_b200.cache import ExpertCache
    from npu_offload_b200.moe import MoEDataPlane
    from oracle.oracle import Port
    from tests.parity import assert_close
    H, F, E, K, L, S = 1024, 256, 16, 4, 2, 8  # S >= the distinct experts of a 2-token call
    W = [[synth.expert_weights(13, l, e, H, F) for e in range(E)] for l in range(L)]
    host = [[tuple(torch.from_numpy(a.view(np.int16)).view(torch.bfloat16) for a in W[l][e]) for e in range(E)]
            for l in range(L)]
    p = MoEDataPlane(H, F, E, K, n_layers=L, max_tokens=16)
    try:
        cache = ExpertCache(p, host, S, swap_per_tok=1)
        assert all(len(r) == S for r in cache.resident)
        for step in range(24):
            l, T = step % L, 1 + step % 2
            x = synth.hidden(300 + step, T, H)
            lg = synth.logits(300 + step, T, E, zipf=True)
            out = cache.forward(l, torch.from_numpy(x.view(np.int16)).view(torch.bfloat16).cuda(),
                                torch.from_numpy(lg).cuda())
            ex = {e: ("bf16", np.concatenate(W[l][e][:2], 0), W[l][e][2]) for e in range(E)}
            ref, _, _, st = Port.moe_layer(x, lg, ex, K)
            assert st == 0
            assert_close(out.cpu().numpy(), ref, what=f"step {step}")
            assert all(len(r) <= S for r in cache.resident)
        assert cache.stats["misses"] > 0 and cache.stats["hits"] > 0 and cache.stats["swaps"] > 0
        # an evicted expert reads as not loaded, and routing a token to it is an error, not a fault
        l = 0
        gone = next(e for e in range(E) if e not in cache.resident[l])
        assert p.expert_kind(l, gone) == 0
        lg = np.full((1, E), -4.0, np.float32)
        lg[0, gone] = 4.0
        x = torch.from_numpy(synth.hidden(1, 1, H).view(np.int16)).view(torch.bfloat16).cuda()
        with pytest.raises(MoEError):
            p.forward(l, x, torch.from_numpy(lg).cuda(), sync=True)
        # a full layer refuses another load until a slot is freed
        with pytest.raises(MoEError):
            p.load_expert(l, gone, *host[l][gone])
    finally:
        p.close()
