"""The device pass of a readout captured in a CUDA graph and replayed (the capture the reference's LevelGraphs makes
of its level passes, janus/hybrid.py:1169-1400): nothing in `DecisionReadout.run` reads a device value on the
host or copies host data, so the whole pass (every level, every layer, the heads) captures, and a replay gives the
eager pass's logits bit for bit, also after the plan buffer is refilled with another batch of the same shapes."""

import numpy as np
import pytest
import torch

from tests.golden_cases import case_model, load_cases

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("name", ["w4b_tree", "w08b_listwise", "tiny_moe_tree"])
def test_readout_pass_captures_and_replays(name):
    from janus_b200 import synthetic
    from janus_b200.model import DecisionReadout
    from janus_b200.plan import DevicePlan
    shape, weights, mode, packs = case_model(load_cases()[name])
    model = DecisionReadout(shape, weights, mode)
    prepared = model.prepare(packs)
    eager = model.run(prepared).clone()
    stream = torch.cuda.Stream()
    stream.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(stream):  # warm-up on the capture stream (library handles, allocator pools)
        model.run(prepared)
    torch.cuda.current_stream().wait_stream(stream)
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        captured = model.run(prepared)
    graph.replay()
    torch.cuda.synchronize()
    model.check_status()
    assert torch.equal(captured, eager)
    # another batch with the same level shapes (same requests, other token ids): refill the plan buffer, replay
    other = [synthetic.Tokens(shape.vocab, 99) for _ in packs]
    packs2 = []
    for p, tok in zip(packs, other):
        ids = torch.tensor([tok(p.token_count)], dtype=p.input_ids.dtype)
        packs2.append(type(p)(ids, p.position_ids, p.segment_ids, p.parents, p.branches, p.state_length,
                              p.option_counts))
    levels2, readout2 = model.plan(packs2)
    plan2 = DevicePlan(levels2, readout2, model.device, tile_tokens=(model.tile_tokens,))
    assert plan2.index == prepared[2].index
    prepared[2].buffer.copy_(plan2.buffer)
    graph.replay()
    want = model.run((levels2, readout2, plan2))
    torch.cuda.synchronize()
    assert torch.equal(captured, want)
    assert not torch.equal(want, eager)
    np.testing.assert_array_equal(captured.cpu().numpy(), want.cpu().numpy())
