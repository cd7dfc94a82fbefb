"""The drop-in seams (janus_b200/seams.py) inside the reference's own serving runner, on CPU.

The seams are patched into the reference's `janus.hybrid` the way janus/latency.py:48-50 patches its timers, the
reference's `HybridBackbone` runs its serving path (`_serve_level` with `Fused(compile=False, serve=True)`: the
eager form of its fused glue), and the readout must equal the unpatched reference's. With no GPU here, the seams'
packed-level ops (janus_b200.ops) are replaced by a CPU stand-in built from the oracle's restatements (test
infrastructure only), and the seams' bf16 storage type is set to fp32, so the patched readout must equal the
reference's to fp32 rounding: what is checked is the seams' signatures and their mapping of the reference's padded
level tensors, plans and states onto packed rows (a wrong row, range or head shows as an O(1) error); the ops
themselves, in bf16, are checked on the GPU (tests/test_gpu_seams.py).

Needs the reference checkout (REFERENCE_ROOT, default /root/reference); skipped where it is absent.
"""

import os
import sys
from pathlib import Path

import numpy as np
import pytest
import torch
import torch.nn.functional as F

from oracle import hybrid as oracle

REFERENCE = Path(os.environ.get("REFERENCE_ROOT", "/root/reference"))
pytestmark = pytest.mark.skipif(not (REFERENCE / "janus" / "hybrid.py").exists(), reason="reference not present")
I32 = torch.int32


def _store(t):
    from janus_b200 import seams
    return t.to(seams.BF16)


class OracleOps:
    """CPU stand-in for the packed-level ops the seams call, from the oracle's fp32 restatements."""

    @staticmethod
    def gdn_chunk_scan(q, k, v, g, beta, row_start, chunk_start, n_chunks, state_in, state_row, keep_state, scale,
                       status=None, segment=None):
        rs = row_start.tolist()
        outs, states = [], []
        for r in range(len(rs) - 1):
            a, b = rs[r], rs[r + 1]
            s0 = None if state_in is None else state_in[int(state_row[r])]
            o, S = oracle.delta_chunked(q[a:b].float(), k[a:b].float(), v[a:b].float(), g[a:b], beta[a:b], s0)
            outs.append(o)
            states.append(S)
        return _store(torch.cat(outs)), (torch.stack(states) if keep_state else None)

    @staticmethod
    def gdn_fork_recurrent(q, k, v, g, beta, row_start, child_start, state_in, keep_state, scale):
        rs, cs = row_start.tolist(), child_start.tolist()
        parent = np.repeat(np.arange(len(cs) - 1), np.diff(cs))
        outs, states = [], []
        for r in range(len(rs) - 1):
            a, b = rs[r], rs[r + 1]
            s0 = None if state_in is None else state_in[int(parent[r])]
            o, S = oracle.delta_recurrent(q[a:b].float(), k[a:b].float(), v[a:b].float(), g[a:b], beta[a:b], s0)
            outs.append(o)
            states.append(S)
        return _store(torch.cat(outs)), (torch.stack(states) if keep_state else None)

    @staticmethod
    def tree_attention_tile_tokens(D, Hq, Hkv):
        return 64

    @staticmethod
    def tree_attention(q, keys, values, anc_lo, anc_hi, row_start, row_of_token, tiles, gate, scale, out=None,
                       status=None):
        T, Hq, D = q.shape
        rs = row_start.tolist()
        res = torch.zeros(T, Hq, D)
        for r in range(len(rs) - 1):
            a, b = rs[r], rs[r + 1]
            pk = [keys[l][int(anc_lo[l][r]):int(anc_hi[l][r])] for l in range(len(anc_lo))]
            pv = [values[l][int(anc_lo[l][r]):int(anc_hi[l][r])] for l in range(len(anc_lo))]
            k_all = torch.cat(pk + [keys[-1][a:b]]).float()
            v_all = torch.cat(pv + [values[-1][a:b]]).float()
            res[a:b] = oracle.attention(q[a:b].float(), k_all, v_all, k_all.shape[0] - (b - a), scale)
        # the covered query tokens: every tile inside one row, together exactly the level's tokens
        t = tiles.tolist()
        assert sorted(x for s, e in t for x in range(s, e)) == list(range(T))
        return _store((res * torch.sigmoid(gate.float())).reshape(T, Hq * D))

    @staticmethod
    def moe_plan(slot_expert, E):
        return slot_expert, None, None, None, None

    @staticmethod
    def moe_grouped_w4a16(x, codes, scales, plan, gated, k, topk_w=None, out=None, status=None):
        ids = plan[0].reshape(-1).long()
        w = oracle.int4_dequantize(codes, scales).float()
        rows = []
        for a, e in enumerate(ids.tolist()):
            if gated:
                h = x[a // k].float() @ w[e].t()
                I = h.shape[0] // 2
                rows.append(F.silu(h[:I]) * h[I:])
            else:
                rows.append((x[a].float() @ w[e].t()) * topk_w[a])
        return _store(torch.stack(rows))

    @staticmethod
    def moe_reduce_slots(y, k, slot_expert, out=None):
        return y.float().view(-1, k, y.shape[1]).sum(1)

    @staticmethod
    def head_scalar(x, rows, final_w, rms_eps, ln_w, ln_b, ln_eps, w_out, b_out, logits=None):
        assert final_w is None
        h = oracle.layer_norm(x[rows.long()], ln_w, ln_b, ln_eps)
        return h @ w_out + b_out[0]

    @staticmethod
    def head_pointer(x, option_rows, option_question, decision_rows, final_w, rms_eps, ln_w, ln_b, ln_eps, wq, wk,
                     logits=None, workspace=None):
        assert final_w is None
        ln = lambda t: oracle.layer_norm(t, ln_w, ln_b, ln_eps)
        keys = ln(x[option_rows.long()]) @ wk.t()
        query = ln(x[decision_rows.long()]) @ wq.t()
        return (keys * query[option_question.long()]).sum(-1) / np.sqrt(wq.shape[0])


@pytest.fixture()
def reference(monkeypatch):
    sys.path.insert(0, str(REFERENCE))
    from janus import hybrid
    from janus_b200 import seams
    monkeypatch.setattr(seams, "ops", OracleOps)
    monkeypatch.setattr(seams, "BF16", torch.float32)
    yield hybrid, seams
    seams.uninstall()


def _golden_tools():
    sys.path.insert(0, str(Path(__file__).resolve().parent / "golden"))
    import make_golden
    return make_golden


def _reference_model(make_golden, shape, weights, mode, state_chunk_tokens=4096):
    """The reference's DecisionModel on `weights` (fp32), serving path: HybridBackbone with an eager Fused(serve)."""
    from janus import hybrid
    from janus.model import DecisionModel, ModelConfig, PointerHead, ScalarHead
    lm = make_golden.hf_model(shape, weights)
    backbone = hybrid.HybridBackbone(lm, tokenizer=None, attention="sdpa", state_chunk_tokens=state_chunk_tokens)
    backbone.fused = hybrid.Fused(compile=False, serve=True)
    model = DecisionModel.__new__(DecisionModel)
    torch.nn.Module.__init__(model)
    model.config = ModelConfig(backbone="tiny-qwen3_5", backbone_family="qwen3_5", mode=mode, adaptation="frozen",
                               dtype="float32", attention="sdpa", tree_positions="continue")
    model.backbone = backbone
    if mode == "tree":
        model.head = ScalarHead(shape.hidden)
        model.head.out.weight.data = weights["head.out.weight"].float().clone()
        model.head.out.bias.data = weights["head.out.bias"].float().clone()
    else:
        model.head = PointerHead(shape.hidden, shape.head_rank)
        model.head.query.weight.data = weights["head.query.weight"].float().clone()
        model.head.key.weight.data = weights["head.key.weight"].float().clone()
    model.head.norm.weight.data = weights["head.norm.weight"].float().clone()
    model.head.norm.bias.data = weights["head.norm.bias"].float().clone()
    model.last_compute = None
    return model


def _forward(model, packs):
    from janus.packing import Branch as RefBranch, PackedRequest as RefPacked
    refs = [RefPacked(p.input_ids, p.position_ids, p.segment_ids, p.parents,
                      [RefBranch(b.start, b.end, b.question_index, b.option_indices, b.option_positions,
                                 b.decision_position, b.kind, b.leaves) for b in p.branches],
                      p.state_length, p.option_counts) for p in packs]
    with torch.no_grad():
        return [[z.float().clone() for z in per] for per in model.forward_many(refs)]


@pytest.mark.parametrize("case", ["tiny_tree", "tiny_listwise", "tiny_moe_tree", "tiny_tree_long"])
def test_seams_inside_the_reference_serving_runner(reference, monkeypatch, case):
    hybrid, seams = reference
    from tests.golden_cases import case_model, load_cases
    make_golden = _golden_tools()
    shape, weights, mode, packs = case_model(load_cases()[case])
    # a 100-token state chunk: the level-0 attention sees earlier chunks' keys through `state`
    model = _reference_model(make_golden, shape, weights, mode, state_chunk_tokens=100)
    want = _forward(model, packs)
    calls = {"rule": 0, "state": 0, "branch": 0, "experts": 0, "head": 0}

    def counted(name, fn):
        def inner(*a, **kw):
            calls[name] += 1
            return fn(*a, **kw)
        return inner

    seams.install(hybrid, model)
    rule = counted("rule", seams.chunk_gated_delta_rule)
    monkeypatch.setattr(hybrid, "chunk_rule", lambda device, allow_fla=True: rule)
    monkeypatch.setattr(hybrid, "FLA_CHUNK_RULE", rule)
    monkeypatch.setattr(hybrid, "FLA_RECURRENT_RULE", rule)
    monkeypatch.setattr(hybrid, "state_attention", counted("state", hybrid.state_attention))
    monkeypatch.setattr(hybrid, "branch_attention", counted("branch", hybrid.branch_attention))
    model.head.forward = counted("head", model.head.forward)
    if shape.moe:
        for i in range(shape.layers):
            m = f"layers.{i}.mlp.experts."
            mod = seams.W4A16Experts.replace(model.backbone.text_model.layers[i].mlp, weights[m + "gate_up_proj"],
                                             weights[m + "gate_up_proj.scales"], weights[m + "down_proj"],
                                             weights[m + "down_proj.scales"])
            mod.forward = counted("experts", mod.forward)
    got = _forward(model, packs)
    assert all(calls[n] > 0 for n in ("rule", "state", "branch", "head")), calls
    assert calls["experts"] > 0 or not shape.moe
    worst = 0.0
    for per_got, per_want in zip(got, want):
        for a, b in zip(per_got, per_want):
            worst = max(worst, float((a - b).abs().max()))
            np.testing.assert_allclose(a.numpy(), b.numpy(), atol=2e-4, rtol=1e-3)
    print(f"\n{case}: max |logit - reference| {worst:.2e}; seam calls {calls}")


def test_install_and_uninstall_restore_the_reference(reference):
    hybrid, seams = reference
    before = (hybrid.FLA_CHUNK_RULE, hybrid.FLA_RECURRENT_RULE, hybrid.state_attention, hybrid.branch_attention)
    seams.install(hybrid)
    assert hybrid.state_attention is seams.state_attention and hybrid.FLA_CHUNK_RULE is seams.chunk_gated_delta_rule
    seams.uninstall(hybrid)
    assert (hybrid.FLA_CHUNK_RULE, hybrid.FLA_RECURRENT_RULE, hybrid.state_attention, hybrid.branch_attention) == before
