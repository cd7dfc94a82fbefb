"""The checkpoint loader (janus_b200/loader.py) on CPU: a transformers Qwen3.5 config gives the ModelShape the
synthetic workloads use, a HF text model's state dict (under a conditional-generation prefix, with unmerged peft
LoRA pairs) gives the tensors DecisionReadout takes, and dense MoE experts become int4 group-128 codes."""

import pytest
import torch

from janus_b200 import loader, synthetic
from janus_b200.config import SHAPES


def _hf_config(shape):
    from transformers import Qwen3_5MoeTextConfig, Qwen3_5TextConfig
    common = dict(vocab_size=shape.vocab, hidden_size=shape.hidden, num_hidden_layers=shape.layers,
                  num_attention_heads=shape.heads, num_key_value_heads=shape.kv_heads, head_dim=shape.head_dim,
                  linear_num_key_heads=shape.lin_k_heads, linear_num_value_heads=shape.lin_v_heads,
                  linear_key_head_dim=shape.lin_k_dim, linear_value_head_dim=shape.lin_v_dim,
                  linear_conv_kernel_dim=shape.conv_kernel, layer_types=list(shape.layer_types), rms_norm_eps=shape.rms_eps)
    if shape.moe:
        return Qwen3_5MoeTextConfig(moe_intermediate_size=shape.moe_intermediate, num_experts=shape.experts,
                                    shared_expert_intermediate_size=shape.shared_intermediate,
                                    num_experts_per_tok=shape.top_k, **common)
    return Qwen3_5TextConfig(intermediate_size=shape.intermediate, **common)


@pytest.mark.parametrize("name", ["tiny", "tiny-moe", "4b", "35b-a3b"])
def test_shape_from_hf_config(name):
    shape = SHAPES[name]
    got = loader.shape_from_hf_config(_hf_config(shape), name=shape.name, lora_rank=shape.lora_rank)
    assert got == shape, (got, shape)


def test_state_dict_with_prefix_and_unmerged_lora():
    shape = SHAPES["tiny"]
    w = synthetic.make_weights(shape, seed=3, head="scalar", lora=False)
    state = {("head." + k[5:] if k.startswith("head.") else "model.language_model." + k): v for k, v in w.items()}
    state["model.visual.blocks.0.weight"] = torch.zeros(3)  # other parts of the checkpoint are skipped
    target = "layers.0.linear_attn.in_proj_qkv"
    base = state.pop(f"model.language_model.{target}.weight")
    g = torch.Generator().manual_seed(0)
    A, B = torch.randn(8, shape.hidden, generator=g), torch.randn(base.shape[0], 8, generator=g) * 0.02
    state[f"model.language_model.{target}.base_layer.weight"] = base
    state[f"model.language_model.{target}.lora_A.default.weight"] = A
    state[f"model.language_model.{target}.lora_B.default.weight"] = B
    out = loader.weights_from_state_dict(state, shape)
    assert set(out) == set(w)
    for k, v in w.items():
        if k != f"{target}.weight":
            assert torch.equal(out[k].float(), v.float()), k
    want = (base.float() + 2.0 * (B @ A)).to(torch.bfloat16)  # alpha = 2r: factor 2, one rounding
    assert torch.equal(out[f"{target}.weight"], want)
    del state["model.language_model.norm.weight"]
    with pytest.raises(ValueError):
        loader.weights_from_state_dict(state, shape)


def test_dense_experts_become_int4_codes_that_decode_close():
    shape = SHAPES["tiny-moe"]
    w = synthetic.make_weights(shape, seed=4, head="scalar")
    dense = {}
    for k, v in w.items():
        if k.endswith(".scales"):
            continue
        dense[k] = synthetic.int4_dequantize(v, w[k + ".scales"]) if k + ".scales" in w else v
    out = loader.weights_from_state_dict(dense, shape)
    name = "layers.0.mlp.experts.gate_up_proj"
    assert out[name].dtype == torch.uint8 and out[name + ".scales"].dtype == torch.bfloat16
    back = synthetic.int4_dequantize(out[name], out[name + ".scales"]).float()
    ref = dense[name].float()
    # within half a step of the new grid plus the bf16 rounding of the decoded value
    step = out[name + ".scales"].float().repeat_interleave(128, -1)
    assert bool(((back - ref).abs() <= 0.5 * step + ref.abs() * 2.0 ** -8 + 1e-7).all())
