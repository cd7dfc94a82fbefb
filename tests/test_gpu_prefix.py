"""Prefix snapshots on the GPU (janus/hybrid.py:1641-1646 encode_prefixes, :1648-1659 encode_many(prefixes=...)),
the relations the reference's own test pins (tests/test_hybrid.py:491-512): a batch of hits answers like the plain
pass, a batch mixing hits and misses too, a snapshot serves its state in another batch, and a snapshot of another
state is refused. A hit runs the branch levels on the same level-0 rows as the plain pass, so its logits are the
plain pass's to fp32 rounding; a state level run as a different batch (the misses of a mixed batch) goes through
cuBLAS GEMMs of another row count, so those are compared within the readout tolerance of the golden tests."""

import pytest

from tests.golden_cases import case_model, load_cases

pytestmark = pytest.mark.gpu


def _max_dev(a, b):
    return max(float((x - y).abs().max()) for pa, pb in zip(a, b) for x, y in zip(pa, pb))


@pytest.mark.parametrize("name", ["tiny_tree", "tiny_listwise", "w4b_tree"])
def test_prefix_snapshots_answer_like_the_plain_pass(name):
    from janus_b200.model import DecisionReadout
    from janus_b200.prefix import PrefixCache
    case = load_cases()[name]
    shape, weights, mode, packs = case_model(case)
    model = DecisionReadout(shape, weights, mode, device="cuda:0")
    plain = model.forward_many(packs)
    snaps = model.encode_prefixes(packs)
    assert [s.tokens for s in snaps] == [p.state_length for p in packs]
    assert all(0 < s.kv_bytes < s.bytes for s in snaps)
    hits = model.forward_many(packs, prefixes=snaps)
    assert _max_dev(hits, plain) <= 1e-5
    tol = max(2e-3, case["bf16_max_dev"])
    p_plain = model.probabilities(packs)
    if len(packs) > 1:
        mixed = model.probabilities(packs, prefixes=[snaps[0]] + [None] * (len(packs) - 1))
        assert _max_dev(mixed, p_plain) <= tol
        # the snapshots serve their states in a batch of another order
        rev = model.probabilities(packs[::-1], prefixes=snaps[::-1])
        assert _max_dev(rev, p_plain[::-1]) <= tol
        # a snapshot of another state is refused before any work
        with pytest.raises(ValueError):
            model.forward_many(packs, prefixes=snaps[::-1])
    # the cache charges a snapshot its tokens scaled by bytes / kv_bytes and evicts the least recent
    cache = PrefixCache(10 ** 9)
    cache.put("a", snaps[0])
    assert cache.get("a") is snaps[0] and cache.get("b") is None
    assert cache.snapshot()["charged_tokens"] >= snaps[0].tokens
