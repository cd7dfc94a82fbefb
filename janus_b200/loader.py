"""From a transformers Qwen3.5 config and a (LoRA-merged or LoRA-carrying) state dict to this library's model inputs.

The reference serves a Qwen3.5 / Qwen3.5-MoE checkpoint: `HybridBackbone.load` reads the HF config and weights
(janus/hybrid.py:1442-1500), LoRA adapters come from training, and `enable_fast` folds them into the base weights
(`merge_and_unload`, janus/hybrid.py:1554-1567: W + (alpha / r) B A in fp32, rounded once to the serving dtype).
`shape_from_hf_config` reads the fields the decision readout needs into a ModelShape; `weights_from_state_dict`
renames the text model's tensors to the layout `DecisionReadout` takes (janus_b200.synthetic.make_weights: HF
Qwen3_5TextModel names without a prefix, plus `head.*`), folds any unmerged peft LoRA pairs the same way, and turns
dense MoE expert stacks into the int4 group-128 format of the W4A16 grouped GEMMs.
"""

import re

import torch

from .config import FULL, LINEAR, ModelShape

# prefixes under which checkpoints keep the text model (conditional-generation checkpoints, CausalLM wrappers, the
# reference's DecisionModel state dict)
PREFIXES = ("model.language_model.", "language_model.model.", "language_model.", "backbone.text_model.",
            "backbone.lm.", "model.")


def _get(cfg, name, default=None):
    if isinstance(cfg, dict):
        return cfg.get(name, default)
    return getattr(cfg, name, default)


def shape_from_hf_config(config, name="hf", head_rank=128, lora_rank=0):
    """A ModelShape from a transformers Qwen3_5(Moe)TextConfig, a Qwen3_5 conditional-generation config (its
    text_config is read) or the equivalent dict. Rotary: rope_theta and partial_rotary_factor from the config or its
    rope_parameters (transformers 5.x), the transformers defaults otherwise."""
    text = _get(config, "text_config") or config
    g = lambda n, d=None: _get(text, n, d)
    rope = g("rope_parameters") or {}
    rope_theta = _get(rope, "rope_theta", None) or g("rope_theta", 10000.0)
    partial = _get(rope, "partial_rotary_factor", None) or g("partial_rotary_factor", 0.25)
    layer_types = tuple(g("layer_types") or ())
    for t in layer_types:
        if t not in (LINEAR, FULL):
            raise ValueError(f"unsupported layer type {t!r}")
    experts = int(g("num_experts", 0) or 0)
    return ModelShape(
        name=name, hidden=int(g("hidden_size")), layers=int(g("num_hidden_layers")), vocab=int(g("vocab_size")),
        heads=int(g("num_attention_heads")), kv_heads=int(g("num_key_value_heads")), head_dim=int(g("head_dim")),
        lin_k_heads=int(g("linear_num_key_heads")), lin_v_heads=int(g("linear_num_value_heads")),
        lin_k_dim=int(g("linear_key_head_dim")), lin_v_dim=int(g("linear_value_head_dim")),
        intermediate=0 if experts else int(g("intermediate_size")), conv_kernel=int(g("linear_conv_kernel_dim", 4)),
        rms_eps=float(g("rms_norm_eps", 1e-6)), rope_theta=float(rope_theta), partial_rotary=float(partial),
        layer_types=layer_types, experts=experts, top_k=int(g("num_experts_per_tok", 0) or 0),
        moe_intermediate=int(g("moe_intermediate_size", 0) or 0) if experts else 0,
        shared_intermediate=int(g("shared_expert_intermediate_size", 0) or 0) if experts else 0,
        head_rank=head_rank, lora_rank=lora_rank)


def int4_quantize(w, group=128):
    """Dense expert weights [..., K] -> (codes uint8 [..., K/2], scales bf16 [..., K/group]): per group of `group`
    consecutive input elements a symmetric scale max|w| / 7 (rounded to bf16) and codes round(w / scale) clamped to
    [-8, 7], two's complement, two per byte with the even element in the low nibble. The decode is code * scale
    (janus_b200.synthetic.int4_dequantize)."""
    *lead, K = w.shape
    if K % group:
        raise ValueError(f"input width {K} is not a multiple of the int4 group {group}")
    wf = w.float().reshape(*lead, K // group, group)
    scale = (wf.abs().amax(-1) / 7.0).to(torch.bfloat16)
    safe = torch.where(scale.float() == 0, torch.ones_like(scale.float()), scale.float())
    codes = torch.clamp(torch.round(wf / safe[..., None]), -8, 7).to(torch.int16).reshape(*lead, K)
    nib = (codes & 15).to(torch.uint8)
    return (nib[..., 0::2] | (nib[..., 1::2] << 4)).contiguous(), scale.contiguous()


def _strip(name, prefix):
    if prefix is not None:
        return name[len(prefix):] if name.startswith(prefix) else None
    for p in PREFIXES:
        if name.startswith(p):
            return name[len(p):]
    return name


def weights_from_state_dict(state, shape, prefix=None, lora_alpha=None, dtype=torch.bfloat16):
    """name -> tensor in the DecisionReadout layout from a checkpoint's state dict.

    - Text-model tensors are found under `prefix` (default: the first of PREFIXES that matches each name); `head.*`
      tensors (the decision head) are kept as fp32. Tensors of other parts (vision tower, MTP, lm_head) are skipped.
    - Unmerged peft LoRA (`X.base_layer.weight`, `X.lora_A.<adapter>.weight`, `X.lora_B.<adapter>.weight`) is folded
      as W + (alpha / r) B A in fp32 and rounded once to `dtype` (alpha defaults to 2r, the reference's, which makes
      the factor 2; janus/hybrid.py:1549-1559).
    - Dense MoE stacks `experts.gate_up_proj` [E, 2I, H] and `experts.down_proj` [E, H, I] become int4 group-128
      codes and scales (`int4_quantize`), stored under the name and `<name>.scales`.
    Raises ValueError when a tensor the shape needs is missing."""
    merged, lora = {}, {}
    for key, t in state.items():
        if key.startswith("head."):
            merged[key] = t.detach().float().contiguous()
            continue
        name = _strip(key, prefix)
        if name is None or not re.match(r"(embed_tokens|layers|norm)\b", name):
            continue
        m = re.match(r"(.*)\.lora_([AB])\.[^.]+\.weight$", name)
        if m:
            lora.setdefault(m.group(1), {})[m.group(2)] = t.detach()
            continue
        name = name.replace(".base_layer.", ".")
        merged[name] = t.detach()
    for module, ab in lora.items():
        if set(ab) != {"A", "B"} or module + ".weight" not in merged:
            raise ValueError(f"incomplete LoRA pair for {module}")
        A, B = ab["A"].float(), ab["B"].float()
        r = A.shape[0]
        scale = (2.0 * r if lora_alpha is None else float(lora_alpha)) / r
        merged[module + ".weight"] = merged[module + ".weight"].float() + scale * (B @ A)
    out = {}
    for name, t in merged.items():
        if name.startswith("head."):
            out[name] = t
        elif name.endswith("experts.gate_up_proj") or name.endswith("experts.down_proj"):
            if t.dtype == torch.uint8:
                out[name] = t.contiguous()
            else:
                codes, scales = int4_quantize(t)
                out[name], out[name + ".scales"] = codes, scales
        else:
            out[name] = t.to(dtype).contiguous()
    from .synthetic import parameter_shapes
    need = [n for n, _, init in parameter_shapes(shape, head="none") if not n.startswith("head.")]
    missing = [n for n in need if n not in out]
    if missing:
        raise ValueError(f"{len(missing)} tensors missing from the state dict, e.g. {missing[:4]}")
    return out
