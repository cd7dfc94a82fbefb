"""Host side of the prefix snapshots (CPU): the snapshot's byte accounting, the level-0 stacking in pack order, and
the token-charged LRU of janus/server.py:98-136 (the eviction relations its test pins, tests/test_server.py:333-340)."""

import numpy as np
import torch

from janus_b200.prefix import PrefixCache, PrefixSnapshot, stack_level0


def _snap(tokens, seed, attention=(False, True)):
    g = torch.Generator().manual_seed(seed)
    states = []
    for att in attention:
        if att:
            states.append((torch.randn(tokens, 2, 8, generator=g).to(torch.bfloat16),
                           torch.randn(tokens, 2, 8, generator=g).to(torch.bfloat16)))
        else:
            states.append((torch.randn(3, 16, generator=g).to(torch.bfloat16), torch.randn(4, 8, 8, generator=g)))
    return PrefixSnapshot(states, attention, np.arange(tokens) + seed)


def test_snapshot_accounting_and_stacking():
    a, b = _snap(5, 1), _snap(7, 2)
    assert a.tokens == 5 and a.kv_bytes == 2 * 5 * 2 * 8 * 2
    assert a.bytes == a.kv_bytes + 3 * 16 * 2 + 4 * 8 * 8 * 4
    lv0 = stack_level0([a, b], a.attention)
    tail, state = lv0[0]
    assert tail.shape == (2, 3, 16) and state.shape == (2, 4, 8, 8)
    assert torch.equal(state[1], b.states[0][1])
    keys, values = lv0[1]
    assert keys.shape == (12, 2, 8) and torch.equal(keys[5:], b.states[1][0]) and torch.equal(values[:5], a.states[1][1])


def test_cache_charges_tokens_and_evicts_the_least_recent():
    a, b = _snap(5, 1), _snap(7, 2)
    charge_a = PrefixCache.charge(a)
    assert charge_a == int(np.ceil(a.bytes * a.tokens / a.kv_bytes)) and charge_a > a.tokens
    small = PrefixCache(1)
    small.put("a", a)
    assert small.snapshot()["entries"] == 0  # an entry above the capacity is not kept
    lru = PrefixCache(max(charge_a, PrefixCache.charge(b)) + 1)  # room for either, not both
    lru.put("a", a)
    lru.put("b", b)  # does not fit beside a: a goes
    assert list(lru.entries) == ["b"] and lru.get("a") is None and lru.get("b") is b
    cache = PrefixCache(10 ** 6)
    cache.put("a", a)
    cache.put("b", b)
    assert cache.get("a") is a and list(cache.entries) == ["b", "a"]  # a hit moves to the recent end
    assert cache.get("c") is None and cache.hits == 1 and cache.misses == 1
    cache.put("a", a)  # a second put of a key replaces its entry, charged once
    assert cache.charged == PrefixCache.charge(a) + PrefixCache.charge(b)
    stats = cache.snapshot()
    assert stats["entries"] == 2 and stats["tokens"] == 12 and stats["bytes"] == a.bytes + b.bytes
    cache.clear()
    assert cache.snapshot()["entries"] == 0 and cache.charged == 0
