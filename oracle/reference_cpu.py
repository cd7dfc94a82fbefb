"""Runs the REFERENCE's own CPU readout (janus.hybrid.HybridBackbone over a transformers Qwen3.5 model, read out by
janus.model.DecisionModel with its heads) on janus_b200's synthetic weights and packed requests. Test and measurement
infrastructure, not the product: tests/golden/make_golden.py generates the golden fixtures with it, and bench.py's
reference arm times it on the host cores. The reference package is imported from REFERENCE_ROOT if set, else from
baseline/_ref (the copy installed beside this checkout, which travels with it), else from /root/reference.
"""

import os
import sys
from pathlib import Path

import torch

from janus_b200 import synthetic

ROOT = Path(__file__).resolve().parent.parent


def reference_root():
    """The directory holding the reference's `janus` package."""
    env = os.environ.get("REFERENCE_ROOT")
    if env:
        return env
    installed = ROOT / "baseline" / "_ref"
    if (installed / "janus" / "hybrid.py").exists():
        return str(installed)
    return "/root/reference"


def available(root=None):
    """Whether the reference and transformers' Qwen3.5 models import here."""
    root = root or reference_root()
    if not (Path(root) / "janus" / "hybrid.py").exists():
        return False
    try:
        import transformers  # noqa: F401
        from transformers import Qwen3_5TextConfig  # noqa: F401
    except Exception:
        return False
    return True


def hf_model(shape, weights, dtype=torch.float32):
    """A transformers text model of `shape` in `dtype` holding `weights` (int4 experts dequantised)."""
    from transformers import Qwen3_5MoeTextConfig, Qwen3_5TextConfig, Qwen3_5MoeTextModel, Qwen3_5TextModel
    common = dict(vocab_size=shape.vocab, hidden_size=shape.hidden, num_hidden_layers=shape.layers,
                  num_attention_heads=shape.heads, num_key_value_heads=shape.kv_heads, head_dim=shape.head_dim,
                  linear_num_key_heads=shape.lin_k_heads, linear_num_value_heads=shape.lin_v_heads,
                  linear_key_head_dim=shape.lin_k_dim, linear_value_head_dim=shape.lin_v_dim,
                  linear_conv_kernel_dim=shape.conv_kernel, layer_types=list(shape.layer_types),
                  max_position_embeddings=32768, attention_dropout=0.0, use_cache=False, tie_word_embeddings=False,
                  rms_norm_eps=shape.rms_eps)
    if shape.moe:
        cfg = Qwen3_5MoeTextConfig(moe_intermediate_size=shape.moe_intermediate,
                                   shared_expert_intermediate_size=shape.shared_intermediate,
                                   num_experts=shape.experts, num_experts_per_tok=shape.top_k, **common)
        cls = Qwen3_5MoeTextModel
    else:
        cfg = Qwen3_5TextConfig(intermediate_size=shape.intermediate, **common)
        cls = Qwen3_5TextModel
    cfg._attn_implementation = "sdpa"
    # built on the meta device and filled tensor by tensor in fp32: no random init of billions of parameters and no
    # second full-size copy of the weights (the 4B model in fp32 is 16 GB); a bf16 model is then cast as a whole, as
    # before (buffers included: the rotary inv_freq is rounded to bf16 by that cast)
    with torch.device("meta"):
        lm = cls(cfg)
    lm = lm.to_empty(device="cpu").float()
    lm.rotary_emb = type(lm.rotary_emb)(config=cfg)  # to_empty leaves the non-persistent inv_freq buffer empty
    params = dict(lm.named_parameters())
    filled = set()
    with torch.no_grad():
        for name, t in weights.items():
            if name.startswith("head.") or name.endswith(".scales"):
                continue
            if name + ".scales" in weights:
                t = synthetic.int4_dequantize(t, weights[name + ".scales"])
            if name not in params:
                raise RuntimeError(f"state dict mismatch: unexpected {name}")
            params[name].copy_(t.reshape(params[name].shape))
            filled.add(name)
    missing = [n for n in params if n not in filled]
    if missing:
        raise RuntimeError(f"state dict mismatch: missing {missing[:5]}")
    return lm.to(dtype).eval()


def reference_logits(shape, weights, mode, packs, dtype=torch.float32, grouped_branches=False, batch=None, root=None):
    """The reference readout. `grouped_branches`: the plain path's branch levels through `branch_attention` (pieces
    grouped by ancestor, bounded by PIECE_BYTES) instead of its one varlen call (`packed_attention`), whose CPU form
    masks every query against every gathered key: at 8192-token states that is tens of GB (the same softmax over the
    same keys either way, janus/hybrid.py:864, 958-989). `batch`: requests per forward_many call (rows are
    independent, so the split changes nothing but the peak host memory). `root`: where the reference's `janus`
    package is (default `reference_root()`)."""
    model = reference_readout(shape, weights, mode, dtype, grouped_branches, root)
    refs = reference_packs(packs)
    step = batch or len(refs)
    out = []
    with torch.no_grad():
        for i in range(0, len(refs), step):
            out += model.forward_many(refs[i:i + step])
    return out


def reference_readout(shape, weights, mode, dtype=torch.float32, grouped_branches=False, root=None):
    """The reference's DecisionModel (its HybridBackbone over the transformers model of `shape` holding `weights`, and
    its ScalarHead / PointerHead holding the head weights), as the golden fixtures and bench.py's CPU arm run it."""
    root = root or reference_root()
    if root not in sys.path:
        sys.path.insert(0, root)
    from janus import hybrid as ref_hybrid
    from janus.hybrid import HybridBackbone
    ref_hybrid.BRANCH_PACKED = not grouped_branches
    from janus.model import DecisionModel, ModelConfig, PointerHead, ScalarHead
    lm = hf_model(shape, weights, dtype)
    backbone = HybridBackbone(lm, tokenizer=None, attention="sdpa", state_chunk_tokens=4096)
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


def reference_packs(packs):
    """janus_b200.packing requests as the reference's own PackedRequest / Branch objects (the same fields)."""
    from janus.packing import Branch as RefBranch, PackedRequest as RefPacked
    return [RefPacked(p.input_ids, p.position_ids, p.segment_ids, p.parents,
                      [RefBranch(b.start, b.end, b.question_index, b.option_indices, b.option_positions,
                                 b.decision_position, b.kind, b.leaves) for b in p.branches],
                      p.state_length, p.option_counts) for p in packs]


