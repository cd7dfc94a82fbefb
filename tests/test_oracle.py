"""The CPU oracle against the reference's own outputs (golden fixtures) and against its own alternative forms."""

import numpy as np
import pytest
import torch

from oracle import hybrid as oracle
from tests.golden_cases import GOLDEN, case_model, load_cases

CASES = load_cases()


@pytest.mark.parametrize("name", sorted(CASES))
def test_oracle_matches_reference_readout(name):
    case = CASES[name]
    shape, weights, mode, packs = case_model(case)
    model = oracle.Oracle(shape, weights)
    for pack, ref_logits, ref_probs in zip(packs, case["logits"], case["probs"]):
        logits = model.logits(pack, mode)
        probs = oracle.probabilities(logits)
        for z, rz, p, rp in zip(logits, ref_logits, probs, ref_probs):
            np.testing.assert_allclose(z.numpy(), np.array(rz), atol=2e-4, rtol=1e-4)
            np.testing.assert_allclose(p.numpy(), np.array(rp), atol=2e-5)


def test_delta_rule_forms_match_reference_vectors():
    v = dict(np.load(GOLDEN / "delta_rule.npz"))
    t = {k: torch.from_numpy(a) for k, a in v.items()}
    for b in range(t["q"].shape[0]):
        q, k = oracle.l2norm(t["q"][b]), oracle.l2norm(t["k"][b])
        o, s = oracle.delta_chunked(q, k, t["v"][b], t["g"][b], t["beta"][b], t["s0"][b])
        np.testing.assert_allclose(o.numpy(), v["o_chunk"][b], atol=2e-5, rtol=1e-4)
        np.testing.assert_allclose(s.numpy(), v["s_chunk"][b], atol=2e-5, rtol=1e-4)
        o, s = oracle.delta_recurrent(q[:9], k[:9], t["v"][b, :9], t["g"][b, :9], t["beta"][b, :9], t["s0"][b])
        np.testing.assert_allclose(o.numpy(), v["o_rec9"][b], atol=2e-5, rtol=1e-4)
        np.testing.assert_allclose(s.numpy(), v["s_rec9"][b], atol=2e-5, rtol=1e-4)
        # chunked == recurrent over the full row (fp32 accumulation order only)
        o_r, s_r = oracle.delta_recurrent(q, k, t["v"][b], t["g"][b], t["beta"][b], t["s0"][b])
        np.testing.assert_allclose(o_r.numpy(), v["o_chunk"][b], atol=1e-4, rtol=1e-3)


def _path_replay(model, pack, mode):
    """Every root-to-leaf path of the tree as one plain causal sequence (how the reference's tests pin its runner,
    tests/test_hybrid.py:80-100): the hidden state of each segment's tokens read from the replay of its path."""
    from oracle.hybrid import tree_levels
    parents = pack.parents.tolist()
    spans = {s: (a, b) for level in tree_levels(pack.segment_ids, pack.parents) for s, a, b in level}
    hidden = torch.zeros(pack.token_count, model.shape.hidden)
    for seg, (a, b) in spans.items():
        chain = [seg]
        while chain[-1] != 0:
            chain.append(parents[chain[-1]])
        idx = torch.cat([torch.arange(*spans[s]) for s in reversed(chain)])
        h, _ = model.run_segment(pack.input_ids[0][idx], pack.position_ids[0][idx], None, None)
        hidden[a:b] = h[-(b - a):]
    return hidden


def test_oracle_tree_forward_equals_path_replay():
    case = CASES["tiny_tree_long"]
    shape, weights, mode, packs = case_model(case)
    model = oracle.Oracle(shape, weights)
    for pack in packs:
        np.testing.assert_allclose(model.encode(pack).numpy(), _path_replay(model, pack, mode).numpy(), atol=2e-4, rtol=1e-4)
