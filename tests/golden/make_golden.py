"""Generates the golden fixtures of tests/golden/ by running the REFERENCE implementation on CPU.

Run in a container where the reference checkout is importable (default /root/reference, or REFERENCE_ROOT):

    python tests/golden/make_golden.py            # readout_cases.json + delta_rule.npz (small cases)
    python tests/golden/make_golden.py --full     # readout_full.json: the benchmark configurations at full depth
    python tests/golden/make_golden.py --argmax   # argmax_4b.npz: 1000 seeded questions at 4B width
    python tests/golden/make_golden.py --nvfp4    # nvfp4.npz: the reference's NVFP4 codec on seeded weights

For every case it builds the seeded synthetic weights (janus_b200.synthetic.make_weights), loads them into a
transformers Qwen3_5TextModel / Qwen3_5MoeTextModel in fp32, wraps it in the reference's janus.hybrid.HybridBackbone
(its plain CPU path: torch chunk/recurrent rules, dense-mask varlen attention), runs the reference's
DecisionModel.forward readout (PointerHead for listwise, ScalarHead for tree) on the synthetic packed requests, and
stores the logits and the temperature-1 probabilities, plus the probabilities of the same reference readout with
the backbone cast to bf16 and their largest deviation from the fp32 ones (the precision noise floor of the case). The int4 experts enter the reference as their dequantised
bf16 values (HF experts hold dense stacks). It also stores per-op vectors of the reference's gated delta rule.

`--full` and `--argmax` also store the probabilities of the CPU oracle (oracle/hybrid.py, test infrastructure) run
with bf16 storage (`Oracle(..., storage="bf16")`: the reference's algorithm with every tensor the B200 path keeps
in bf16 between kernels rounded there), the like-for-like yardstick of the B200 path at its own storage precision;
those requests are rebuilt from their seeds by janus_b200.synthetic and checked against a stored crc of their ids.

The fixtures are written once and not edited afterwards; tests compare the CPU oracle and the CUDA path to them.
"""

import json
import os
import sys
from pathlib import Path

import numpy as np
import torch

HERE = Path(__file__).resolve().parent
sys.path.insert(0, str(HERE.parent.parent))
REFERENCE = os.environ.get("REFERENCE_ROOT", "/root/reference")

from janus_b200.config import SHAPES  # noqa: E402
from janus_b200 import synthetic  # noqa: E402
from janus_b200.packing import Question, pack_listwise, pack_tree  # noqa: E402
from oracle.reference_cpu import hf_model, reference_logits as _reference_logits  # noqa: E402,F401

# name: (shape, overrides of the shape, readout mode, seed, request factory)
def _cases():
    tiny = SHAPES["tiny"]
    t4 = lambda seed: synthetic.tiny_request(vocab=4096, seed=seed, mode="tree")

    def small_tree(vocab, seed, state=200, questions=3, block=12):
        tok = synthetic.Tokens(vocab, seed)
        qs = []
        for qi in range(questions):
            kind = ("choice", "score", "noul")[qi % 3]
            header = tok(block)
            if kind == "noul":
                qs.append(Question(kind, header, (tok(3),)))
            else:
                qs.append(Question(kind, header, tuple(tok(int(tok.rng.integers(2, 5))) for _ in range(int(tok.rng.integers(2, 5))))))
        return pack_tree(tok(state), qs)

    def small_list(vocab, seed, state=192):
        tok = synthetic.Tokens(vocab, seed)
        return pack_listwise(tok(state), [Question("choice", tok(9), tuple(tok(4) for _ in range(3)), tok(3)),
                                          Question("noul", tok(6), (tok(2), tok(2)), tok(3))])

    return {
        "tiny_listwise": (tiny, {}, "listwise", 0, lambda: [synthetic.tiny_request(vocab=4096, seed=0)]),
        "tiny_tree": (tiny, {}, "tree", 1, lambda: [t4(1), t4(2)]),
        "tiny_tree_long": (tiny, {}, "tree", 2, lambda: [small_tree(4096, 5, state=300), small_tree(4096, 6, state=77)]),
        "tiny_moe_tree": (SHAPES["tiny-moe"], {}, "tree", 3, lambda: [small_tree(4096, 7), small_tree(4096, 8, state=90)]),
        "w08b_listwise": (SHAPES["0.8b"], dict(layers=4, vocab=4096), "listwise", 4, lambda: [small_list(4096, 9)]),
        "w4b_tree": (SHAPES["4b"], dict(layers=4, vocab=4096), "tree", 5,
                     lambda: [small_tree(4096, 10, state=160), small_tree(4096, 11, state=100)]),
        "wa3b_tree": (SHAPES["35b-a3b"], dict(layers=4, vocab=4096, experts=32), "tree", 6,
                      lambda: [small_tree(4096, 12, state=96, questions=2)]),
    }


def shape_of(shape, overrides):
    layers = overrides.pop("layers", shape.layers)
    return shape.with_layers(layers, **overrides)


def reference_logits(*args, **kwargs):
    """The reference readout (oracle.reference_cpu.reference_logits) from the checkout at REFERENCE."""
    return _reference_logits(*args, root=REFERENCE, **kwargs)


def pack_to_dict(p):
    return {"input_ids": p.input_ids[0].tolist(), "position_ids": p.position_ids[0].tolist(),
            "segment_ids": p.segment_ids.tolist(), "parents": p.parents.tolist(), "state_length": p.state_length,
            "option_counts": list(p.option_counts),
            "branches": [dict(start=b.start, end=b.end, question_index=b.question_index,
                              option_indices=list(b.option_indices), option_positions=list(b.option_positions),
                              decision_position=b.decision_position, kind=b.kind,
                              leaves=[list(x) for x in b.leaves]) for b in p.branches]}


def delta_rule_vectors():
    """Per-op vectors of the reference's gated delta rule (transformers torch_chunk_gated_delta_rule and
    torch_recurrent_gated_delta_rule as janus.hybrid.chunk_rule returns them on CPU)."""
    sys.path.insert(0, REFERENCE)
    from janus.hybrid import chunk_rule
    from transformers.models.qwen3_5.modeling_qwen3_5 import torch_recurrent_gated_delta_rule
    g = torch.Generator().manual_seed(123)
    B, T, Hk, Hv, D = 2, 150, 2, 4, 32
    q = torch.randn(B, T, Hk, D, generator=g)
    k = torch.randn(B, T, Hk, D, generator=g)
    v = torch.randn(B, T, Hv, D, generator=g)
    b = torch.randn(B, T, Hv, generator=g)
    a = torch.randn(B, T, Hv, generator=g)
    beta = torch.sigmoid(b)
    g_ = -torch.rand(Hv, generator=g).mul(4).exp() * torch.nn.functional.softplus(a + 1.0)
    s0 = torch.randn(B, Hv, D, D, generator=g) * 0.1
    rep = lambda x: x.repeat_interleave(Hv // Hk, dim=2)
    rule = chunk_rule("cpu")
    o_c, s_c = rule(rep(q), rep(k), v, g=g_, beta=beta, initial_state=s0, output_final_state=True, use_qk_l2norm_in_kernel=True)
    o_r, s_r = torch_recurrent_gated_delta_rule(rep(q[:, :9]), rep(k[:, :9]), v[:, :9], g=g_[:, :9], beta=beta[:, :9],
                                                initial_state=s0, output_final_state=True, use_qk_l2norm_in_kernel=True)
    return dict(q=q, k=k, v=v, g=g_, beta=beta, s0=s0, o_chunk=o_c, s_chunk=s_c, o_rec9=o_r, s_rec9=s_r)


# The benchmark configurations at full depth. name: (shape, overrides, mode, weight seed, [(builder, kwargs)]
# [, weight std overrides]). cfg 5 (A3B) keeps its widths and all 256 experts at 4 layers: 40 layers of fp32 experts
# do not fit host memory. Its random router is near-uniform, so bf16 rounding flips top-8 choices and moves the
# readout by ~0.1 in any bf16 path; the "wide router" variant draws the router N(0, 0.2) (top-8 gaps ten times
# wider) so the MoE numerics are held to the dense models' noise floor instead.
def _full_cases():
    return {
        "cfg5_a3b_wide_router_4layers": ("35b-a3b", dict(layers=4), "tree", 51,
                                         [("a3b_request", dict(seed=510, state_tokens=1024))],
                                         {"mlp.gate.weight": 0.2}),
        "cfg2_08b_listwise": ("0.8b", {}, "listwise", 20, [("q08b_request", dict(seed=200))]),
        "cfg3_4b_tree": ("4b", {}, "tree", 30, [("q4b_request", dict(seed=300))]),
        "cfg4_08b_stress": ("0.8b", {}, "tree", 40, [("stress_request", dict(seed=400))]),
        "cfg5_a3b_tree_4layers": ("35b-a3b", dict(layers=4), "tree", 50,
                                  [("a3b_request", dict(seed=500, state_tokens=2048)),
                                   ("a3b_request", dict(seed=501, state_tokens=1024))]),
    }


ARGMAX = dict(shape="4b", overrides=dict(layers=4, vocab=4096), mode="tree", seed=60, requests=125,
              builder="q4b_request", kwargs=dict(vocab=4096, state_tokens=256), first_seed=600)


def ids_crc(pack):
    import zlib
    return zlib.crc32(pack.input_ids[0].numpy().astype(np.int64).tobytes())


def build_packs(specs):
    return [getattr(synthetic, b)(**kw) for b, kw in specs]


def oracle_probs(shape, weights, mode, packs, storage):
    sys.path.insert(0, str(HERE.parent.parent))
    from oracle import hybrid as oracle
    model = oracle.Oracle(shape, weights, storage=storage)
    with torch.no_grad():
        return [[p.tolist() for p in oracle.probabilities(model.logits(pack, mode))] for pack in packs]


def main_full():
    out = HERE / "readout_full.json"
    manifest = json.loads(out.read_text()) if out.exists() else {}
    for name, (base, overrides, mode, seed, specs, *std) in _full_cases().items():
        if name in manifest:
            continue
        std = std[0] if std else None
        shape = shape_of(SHAPES[base], dict(overrides))
        packs = build_packs(specs)
        weights = synthetic.make_weights(shape, seed=seed, head="scalar" if mode == "tree" else "pointer", std=std)
        logits = reference_logits(shape, weights, mode, packs, grouped_branches=True)
        probs = [[torch.softmax(z.float(), -1).tolist() for z in per] for per in logits]
        logits16 = reference_logits(shape, weights, mode, packs, torch.bfloat16, grouped_branches=True)
        probs16 = [[torch.softmax(z.float(), -1).tolist() for z in per] for per in logits16]
        dev16 = max(abs(a - b) for pp, qq in zip(probs, probs16) for p, q in zip(pp, qq) for a, b in zip(p, q))
        po16 = oracle_probs(shape, weights, mode, packs, "bf16")
        manifest[name] = dict(shape=base, overrides=overrides, mode=mode, seed=seed, std=std,
                              checksum=synthetic.weight_checksum(weights),
                              requests=[dict(builder=b, kwargs=kw, ids_crc=ids_crc(p), tokens=p.token_count)
                                        for (b, kw), p in zip(specs, packs)],
                              logits=[[z.float().tolist() for z in per] for per in logits], probs=probs,
                              probs_bf16=probs16, bf16_max_dev=dev16, probs_oracle_bf16=po16)
        print(name, "tokens", [p.token_count for p in packs], "questions", sum(len(p) for p in probs),
              "reference bf16 vs fp32 max |dp|", dev16, flush=True)
        out.write_text(json.dumps(manifest))
        del weights, logits, logits16
    print("wrote", out)


def main_argmax():
    a = ARGMAX
    shape = shape_of(SHAPES[a["shape"]], dict(a["overrides"]))
    specs = [(a["builder"], dict(a["kwargs"], seed=a["first_seed"] + j)) for j in range(a["requests"])]
    packs = build_packs(specs)
    weights = synthetic.make_weights(shape, seed=a["seed"], head="scalar")
    flat = lambda per_pack: np.concatenate([np.asarray(z, dtype=np.float32) for per in per_pack for z in per])
    logits = reference_logits(shape, weights, a["mode"], packs, grouped_branches=True, batch=8)
    p32 = [[torch.softmax(z.float(), -1).numpy() for z in per] for per in logits]
    p16 = [[torch.softmax(z.float(), -1).numpy() for z in per]
           for per in reference_logits(shape, weights, a["mode"], packs, torch.bfloat16, grouped_branches=True,
                                       batch=8)]
    po16 = oracle_probs(shape, weights, a["mode"], packs, "bf16")
    counts = np.array([len(z) for per in p32 for z in per], dtype=np.int32)
    np.savez_compressed(HERE / "argmax_4b.npz", spec=np.array(json.dumps(a)), counts=counts,
                        ids_crc=np.array([ids_crc(p) for p in packs], dtype=np.int64),
                        checksum=np.array(synthetic.weight_checksum(weights)),
                        probs=flat(p32), probs_bf16=flat(p16), probs_oracle_bf16=flat(po16))
    print("wrote", HERE / "argmax_4b.npz", "questions", counts.size, "options", int(counts.sum()))


def main_nvfp4():
    """The reference's NVFP4 codec (janus/hybrid.py:400-440) on a seeded [2, 128, 256] stack: its quantised codes,
    block scales and global scale per expert, its bf16 dequantised values, and its e2m1 encoding of edge values."""
    sys.path.insert(0, REFERENCE)
    from janus import hybrid as ref
    g = torch.Generator().manual_seed(77)
    w = torch.randn(2, 128, 256, generator=g) * 0.02
    w[1, 3, :16] = 0.0  # an all-zero block
    out = {"w": w.numpy()}
    for e in range(2):
        codes, bs, gl = ref.nvfp4_quantize(w[e])
        out[f"codes{e}"] = codes.numpy()
        out[f"bscales{e}"] = bs.view(torch.uint8).numpy()
        out[f"global{e}"] = np.array(float(gl), dtype=np.float32)
        out[f"dequant{e}"] = ref._nvfp4_dequant(codes, bs, gl, torch.bfloat16).float().numpy()
    x = torch.cat([torch.tensor([0.25, 0.75, 1.25, 1.75, 2.5, 3.5, 5.0, 6.0, 7.0, -0.25, -1.25, -5.0, 0.0]),
                   torch.randn(4096, generator=g) * 3])
    out["enc_x"] = x.numpy()
    out["enc_codes"] = ref._e2m1_encode(x).numpy()
    np.savez_compressed(HERE / "nvfp4.npz", **out)
    print("wrote", HERE / "nvfp4.npz")


def main():
    torch.set_num_threads(os.cpu_count() or 8)
    if "--nvfp4" in sys.argv:
        return main_nvfp4()
    if "--full" in sys.argv:
        return main_full()
    if "--argmax" in sys.argv:
        return main_argmax()
    manifest = {}
    for name, (base, overrides, mode, seed, factory) in _cases().items():
        shape = shape_of(base, dict(overrides))
        packs = factory()
        weights = synthetic.make_weights(shape, seed=seed, head="scalar" if mode == "tree" else "pointer")
        logits = reference_logits(shape, weights, mode, packs)
        probs = [[torch.softmax(z.float(), -1).tolist() for z in per] for per in logits]
        # the same reference readout with the backbone in bf16 (its plain CPU path): the precision noise floor
        logits16 = reference_logits(shape, weights, mode, packs, torch.bfloat16)
        probs16 = [[torch.softmax(z.float(), -1).tolist() for z in per] for per in logits16]
        dev16 = max(abs(a - b) for pp, qq in zip(probs, probs16) for p, q in zip(pp, qq) for a, b in zip(p, q))
        manifest[name] = dict(shape=base.name, overrides=overrides, mode=mode, seed=seed,
                              checksum=synthetic.weight_checksum(weights), packs=[pack_to_dict(p) for p in packs],
                              logits=[[z.float().tolist() for z in per] for per in logits], probs=probs,
                              probs_bf16=probs16, bf16_max_dev=dev16)
        print(name, "questions", sum(len(p) for p in probs), "reference bf16 vs fp32 max |dp|", dev16, flush=True)
    (HERE / "readout_cases.json").write_text(json.dumps(manifest))
    vec = delta_rule_vectors()
    np.savez_compressed(HERE / "delta_rule.npz", **{k: v.numpy() for k, v in vec.items()})
    print("wrote", HERE / "readout_cases.json", HERE / "delta_rule.npz")


if __name__ == "__main__":
    main()
