"""Model shapes of the Qwen3.5 hybrid family as the decision readout runs them.

The reference builds its backbone from a transformers `Qwen3_5TextConfig` / `Qwen3_5MoeTextConfig`
(janus/hybrid.py:499-521 for the tiny one, HF checkpoints otherwise). This module keeps only the fields the
forward pass reads, with the transformers 5.5 defaults for everything a workload does not set: rms_norm_eps 1e-6,
rope_theta 10000, partial_rotary_factor 0.25, conv kernel 4, silu activation, no attention bias.
"""

from dataclasses import dataclass, field, replace


LINEAR, FULL = "linear_attention", "full_attention"


def hybrid_layer_types(layers, period=4):
    """3:1 DeltaNet:attention, attention last in each group of four (the Qwen3.5 layout)."""
    return [FULL if (i + 1) % period == 0 else LINEAR for i in range(layers)]


@dataclass(frozen=True)
class ModelShape:
    name: str
    hidden: int
    layers: int
    vocab: int
    # gated full attention (Qwen3_5Attention): q_proj emits query and gate per head
    heads: int
    kv_heads: int
    head_dim: int
    # Gated DeltaNet (Qwen3_5GatedDeltaNet)
    lin_k_heads: int
    lin_v_heads: int
    lin_k_dim: int
    lin_v_dim: int
    intermediate: int = 0  # dense SwiGLU width (0 for MoE models)
    conv_kernel: int = 4
    rms_eps: float = 1e-6
    rope_theta: float = 10000.0
    partial_rotary: float = 0.25
    layer_types: tuple = ()
    # sparse MoE feed-forward (qwen3_5_moe)
    experts: int = 0
    top_k: int = 0
    moe_intermediate: int = 0
    shared_intermediate: int = 0
    # readout
    head_rank: int = 128
    lora_rank: int = 0

    def __post_init__(self):
        if not self.layer_types:
            object.__setattr__(self, "layer_types", tuple(hybrid_layer_types(self.layers)))
        if len(self.layer_types) != self.layers:
            raise ValueError("layer_types must have one entry per layer")

    @property
    def rotary_dim(self):
        return int(self.head_dim * self.partial_rotary)

    @property
    def key_dim(self):
        return self.lin_k_heads * self.lin_k_dim

    @property
    def value_dim(self):
        return self.lin_v_heads * self.lin_v_dim

    @property
    def conv_dim(self):
        return 2 * self.key_dim + self.value_dim

    @property
    def moe(self):
        return self.experts > 0

    def with_layers(self, layers, **changes):
        """The same widths at another depth (oracle subsets of the large configs)."""
        return replace(self, layers=layers, layer_types=tuple(hybrid_layer_types(layers)), **changes)


# The five workloads. Widths follow the configs of the benchmark; the attention and DeltaNet head layouts of the
# 0.8B and A3B shapes are the transformers defaults for those families where the workload does not state them.
TINY = ModelShape("tiny", hidden=128, layers=4, vocab=4096, heads=4, kv_heads=2, head_dim=32,
                  lin_k_heads=2, lin_v_heads=4, lin_k_dim=32, lin_v_dim=32, intermediate=512)
Q08B = ModelShape("0.8b", hidden=1024, layers=24, vocab=248320, heads=8, kv_heads=2, head_dim=256,
                  lin_k_heads=16, lin_v_heads=16, lin_k_dim=128, lin_v_dim=128, intermediate=3584, lora_rank=64)
Q4B = ModelShape("4b", hidden=2560, layers=32, vocab=248320, heads=16, kv_heads=4, head_dim=256,
                 lin_k_heads=16, lin_v_heads=32, lin_k_dim=128, lin_v_dim=128, intermediate=9216, lora_rank=16)
A3B = ModelShape("35b-a3b", hidden=2048, layers=40, vocab=248320, heads=16, kv_heads=2, head_dim=256,
                 lin_k_heads=16, lin_v_heads=32, lin_k_dim=128, lin_v_dim=128, experts=256, top_k=8,
                 moe_intermediate=512, shared_intermediate=512)
TINY_MOE = ModelShape("tiny-moe", hidden=128, layers=4, vocab=4096, heads=4, kv_heads=2, head_dim=32,
                      lin_k_heads=2, lin_v_heads=4, lin_k_dim=32, lin_v_dim=32, experts=8, top_k=2,
                      moe_intermediate=128, shared_intermediate=128)

SHAPES = {s.name: s for s in (TINY, Q08B, Q4B, A3B, TINY_MOE)}
