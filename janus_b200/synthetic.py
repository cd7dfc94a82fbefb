"""Seeded synthetic weights and requests for the benchmark workloads (no checkpoint or dataset is involved).

Weights. Every matrix (linear, embedding, depthwise conv, router, expert) is N(0, 0.02); norms, A_log and dt_bias
keep the transformers defaults (Qwen3_5RMSNorm weight 0 since it computes x*(1+w), the gated norm's weight 1,
A_log = log U(0, 16), dt_bias 1: transformers qwen3_5 `_init_weights`). Each parameter draws from its own generator
seeded by (seed, name), so a subset of the layers, or the same model on another device type, is generated without
generating the rest; values are drawn in fp32 and rounded once to bf16, the storage type of the serving model
(the readout head stays fp32 as in the reference, janus/model.py:156-247). A merged LoRA (rank r) adds
2 * B @ A to the targets of janus/hybrid.py:90 in fp32 before that rounding (peft's fold with alpha = 2r,
janus/hybrid.py:1549-1559), A ~ N(0, 1/r) (standard deviation), B ~ N(0, 0.02).

MoE experts (W4A16, int4 with group size 128): codes uniform over the integers [-8, 7], one bf16 scale per 128
consecutive input elements drawn N(0, 0.02); two codes per byte, the even element in the low nibble.

Requests. Token ids are uniform over the non-special ids [1, vocab - 512) (id 0 and the top 512 ids are treated as
special since no tokenizer is present), drawn from numpy's default_rng(seed).
"""

import zlib

import numpy as np
import torch

from .config import LINEAR, SHAPES, ModelShape
from .packing import Question, pack_listwise, pack_tree

LORA_TARGETS = ("q_proj", "k_proj", "v_proj", "o_proj", "in_proj_qkv", "in_proj_z", "in_proj_b", "in_proj_a", "out_proj")
INT4_GROUP = 128


def _gen(seed, name, device):
    g = torch.Generator(device=device)
    g.manual_seed((seed * 1_000_003 + zlib.crc32(name.encode())) % (2 ** 63))
    return g


def _normal(shape, std, seed, name, device):
    return torch.randn(shape, generator=_gen(seed, name, device), device=device, dtype=torch.float32) * std


def parameter_shapes(shape: ModelShape, head="pointer", layers=None):
    """(name, shape, init) of every parameter, HF Qwen3_5TextModel names plus `head.*`."""
    H = shape.hidden
    out = [("embed_tokens.weight", (shape.vocab, H), "normal")]
    for i in (range(shape.layers) if layers is None else layers):
        p = f"layers.{i}."
        out += [(p + "input_layernorm.weight", (H,), "zeros"), (p + "post_attention_layernorm.weight", (H,), "zeros")]
        if shape.layer_types[i] == LINEAR:
            a = p + "linear_attn."
            out += [(a + "in_proj_qkv.weight", (shape.conv_dim, H), "normal"),
                    (a + "in_proj_z.weight", (shape.value_dim, H), "normal"),
                    (a + "in_proj_b.weight", (shape.lin_v_heads, H), "normal"),
                    (a + "in_proj_a.weight", (shape.lin_v_heads, H), "normal"),
                    (a + "conv1d.weight", (shape.conv_dim, 1, shape.conv_kernel), "normal"),
                    (a + "dt_bias", (shape.lin_v_heads,), "ones"),
                    (a + "A_log", (shape.lin_v_heads,), "a_log"),
                    (a + "norm.weight", (shape.lin_v_dim,), "ones"),
                    (a + "out_proj.weight", (H, shape.value_dim), "normal")]
        else:
            a = p + "self_attn."
            D = shape.head_dim
            out += [(a + "q_proj.weight", (2 * shape.heads * D, H), "normal"),
                    (a + "k_proj.weight", (shape.kv_heads * D, H), "normal"),
                    (a + "v_proj.weight", (shape.kv_heads * D, H), "normal"),
                    (a + "o_proj.weight", (H, shape.heads * D), "normal"),
                    (a + "q_norm.weight", (D,), "zeros"), (a + "k_norm.weight", (D,), "zeros")]
        m = p + "mlp."
        if shape.moe:
            E, I, S = shape.experts, shape.moe_intermediate, shape.shared_intermediate
            out += [(m + "gate.weight", (E, H), "normal"),
                    (m + "experts.gate_up_proj", (E, 2 * I, H), "int4"),
                    (m + "experts.down_proj", (E, H, I), "int4"),
                    (m + "shared_expert.gate_proj.weight", (S, H), "normal"),
                    (m + "shared_expert.up_proj.weight", (S, H), "normal"),
                    (m + "shared_expert.down_proj.weight", (H, S), "normal"),
                    (m + "shared_expert_gate.weight", (1, H), "normal")]
        else:
            out += [(m + "gate_proj.weight", (shape.intermediate, H), "normal"),
                    (m + "up_proj.weight", (shape.intermediate, H), "normal"),
                    (m + "down_proj.weight", (H, shape.intermediate), "normal")]
    out.append(("norm.weight", (H,), "zeros"))
    if head == "pointer":
        out += [("head.norm.weight", (H,), "ones32"), ("head.norm.bias", (H,), "zeros32"),
                ("head.query.weight", (shape.head_rank, H), "normal32"), ("head.key.weight", (shape.head_rank, H), "normal32")]
    else:
        out += [("head.norm.weight", (H,), "ones32"), ("head.norm.bias", (H,), "zeros32"),
                ("head.out.weight", (1, H), "normal32"), ("head.out.bias", (1,), "zeros32")]
    return out


def int4_quantized(shape, seed, name, device):
    """(codes uint8 [..., K/2] two per byte with the even element low, scales bf16 [..., K/128]) of one expert stack."""
    *lead, K = shape
    if K % INT4_GROUP:
        raise ValueError(f"{name}: K={K} is not a multiple of the int4 group {INT4_GROUP}")
    g = _gen(seed, name + "#codes", device)
    codes = torch.randint(-8, 8, (*lead, K), generator=g, device=device, dtype=torch.int16)
    nib = (codes & 15).to(torch.uint8)
    packed = (nib[..., 0::2] | (nib[..., 1::2] << 4)).contiguous()
    scales = _normal((*lead, K // INT4_GROUP), 0.02, seed, name + "#scales", device).to(torch.bfloat16)
    return packed, scales


E2M1_VALUES = (0.0, 0.5, 1.0, 1.5, 2.0, 3.0, 4.0, 6.0)
FP4_BLOCK = 16


def e2m1_encode(x):
    """fp32 -> 4-bit e2m1 codes (bit 3 the sign), nearest value with ties to the even code."""
    vals = torch.tensor(E2M1_VALUES, device=x.device)
    mids = (vals[1:] + vals[:-1]) / 2
    mag = x.abs()
    code = torch.bucketize(mag, mids)  # a magnitude equal to a midpoint goes to the lower code
    tie = (code < 7) & (mag == mids[code.clamp(max=6)]) & (code % 2 == 1)
    code = (code + tie.to(code.dtype)).to(torch.uint8)
    return code | ((x < 0).to(torch.uint8) << 3)


def nvfp4_quantize(w, rows_global=None):
    """A weight [..., rows, K] in the reference's NVFP4 layout (janus/hybrid.py:427-440, ModelOpt's rule): a global
    fp32 scale amax / (6 * 448) over each [rows, K] matrix (or over each slice of rows given by `rows_global`, e.g.
    the gate and up halves of a gate/up stack), per 16 inputs an e4m3 block scale block_amax / 6 / global (1 for an
    all-zero block), codes the e2m1 rounding of w / (block scale * global), two per byte with the even element in
    the low nibble. Returns (codes uint8 [..., rows, K/2], block scales e4m3 [..., rows, K/16], global fp32
    [..., rows])."""
    w = w.float()
    *lead, R, K = w.shape
    bounds = rows_global or [(0, R)]
    glob = torch.empty(*lead, R, device=w.device)
    for a, b in bounds:
        amax = w[..., a:b, :].abs().amax(dim=(-1, -2))
        glob[..., a:b] = (amax / (6.0 * 448.0)).clamp(min=torch.finfo(torch.float32).tiny)[..., None]
    blocks = w.view(*lead, R, K // FP4_BLOCK, FP4_BLOCK)
    bs = blocks.abs().amax(-1) / 6.0 / glob[..., None]
    bs = torch.where(bs == 0, torch.ones_like(bs), bs).to(torch.float8_e4m3fn)
    codes = e2m1_encode(blocks / (bs.float() * glob[..., None])[..., None]).reshape(w.shape)
    return (codes[..., 0::2] | (codes[..., 1::2] << 4)).contiguous(), bs.contiguous(), glob.contiguous()


def nvfp4_quantized(shape, seed, name, device, halves=False):
    """A seeded NVFP4 expert stack: N(0, 0.02) weights of `shape` [E, rows, K] quantised by `nvfp4_quantize` (with
    `halves`, the gate and up halves of a gate/up stack get their own global scales, as ModelOpt stores them)."""
    w = _normal(shape, 0.02, seed, name, device)
    R = shape[-2]
    return nvfp4_quantize(w, [(0, R // 2), (R // 2, R)] if halves else None)


def int4_dequantize(packed, scales, dtype=torch.bfloat16):
    """code * scale in fp32 (exact: a 4-bit integer times a bf16 value), rounded once to `dtype`."""
    lo = (packed & 15).to(torch.int16)
    hi = (packed >> 4).to(torch.int16)
    codes = torch.stack([lo, hi], dim=-1).flatten(-2)
    codes = torch.where(codes >= 8, codes - 16, codes).float()
    K = codes.shape[-1]
    w = codes.view(*codes.shape[:-1], K // INT4_GROUP, INT4_GROUP) * scales.float()[..., None]
    return w.reshape(codes.shape).to(dtype)


def make_weights(shape: ModelShape, seed=0, head="pointer", device="cpu", layers=None, lora=True, std=None,
                 experts="int4"):
    """Name -> tensor. Matrices bf16 (int4 experts as (codes, scales) pairs under `<name>` and `<name>.scales`),
    head fp32. `layers` restricts the decoder layers generated (default all). `std`: {name suffix: standard deviation}
    replacing the 0.02 of the matrices whose names end with the suffix (test variants only: e.g. a sharper router).
    `experts`: "int4" (group 128, bf16 scales: `<name>`, `<name>.scales`) or "nvfp4" (the reference's format: codes,
    e4m3 block scales `<name>.scales`, fp32 global scales per row `<name>.global`)."""
    out = {}
    r = shape.lora_rank if lora else 0
    for name, shp, init in parameter_shapes(shape, head, layers):
        if init == "int4":
            if experts == "nvfp4":
                packed, scales, glob = nvfp4_quantized(shp, seed, name, device, halves=name.endswith("gate_up_proj"))
                out[name + ".global"] = glob
            else:
                packed, scales = int4_quantized(shp, seed, name, device)
            out[name] = packed
            out[name + ".scales"] = scales
            continue
        if init in ("normal", "normal32"):
            sd = next((v for k, v in (std or {}).items() if name.endswith(k)), 0.02)
            t = _normal(shp, sd, seed, name, device)
            leaf = name.split(".")[-2] if name.endswith(".weight") else ""
            if r and init == "normal" and leaf in LORA_TARGETS:
                a = _normal((r, shp[1]), 1.0 / r, seed, name + "#lora_A", device)
                b = _normal((shp[0], r), 0.02, seed, name + "#lora_B", device)
                t = t + 2.0 * (b @ a)
        elif init in ("zeros", "zeros32"):
            t = torch.zeros(shp, device=device)
        elif init in ("ones", "ones32"):
            t = torch.ones(shp, device=device)
        elif init == "a_log":
            u = torch.rand(shp, generator=_gen(seed, name, device), device=device) * 16.0
            t = torch.log(u.clamp(min=1e-6))
        else:
            raise AssertionError(init)
        out[name] = t if init.endswith("32") else t.to(torch.bfloat16)
    return out


def weight_checksum(weights):
    """Order-independent float64 checksum of a weight dict (detects generator drift between machines)."""
    total = 0.0
    for name in sorted(weights):
        t = weights[name]
        v = t.double() if t.is_floating_point() else t.to(torch.float64)
        total += float((v * (1 + (zlib.crc32(name.encode()) % 97))).sum()) + float(v.abs().sum())
    return total


# ----------------------------------------------------------------------------------------------------------- requests

class Tokens:
    def __init__(self, vocab, seed):
        self.rng = np.random.default_rng(seed)
        self.hi = max(2, vocab - 512)

    def __call__(self, n):
        return tuple(int(t) for t in self.rng.integers(1, self.hi, size=n))


def tiny_request(vocab=4096, seed=0, state_tokens=256, mode="listwise"):
    """Workload 1: a 256-token state and 3 questions of 16 question tokens: a choice with 4 options of 3 tokens,
    a score with 3 levels of 3 tokens and a noul (false/true, 3 tokens each); 3 "Decision:" tokens per listwise
    branch. Tree mode: the 16 tokens are the block; the choice and score leaves are the option tokens; the noul has
    one 3-token decision leaf."""
    tok = Tokens(vocab, seed)
    state = tok(state_tokens)
    qs = []
    for kind, n in (("choice", 4), ("score", 3), ("noul", 2)):
        header = tok(16)
        if mode == "tree" and kind == "noul":
            qs.append(Question(kind, header, (tok(3),)))
        else:
            qs.append(Question(kind, header, tuple(tok(3) for _ in range(n)), tok(3)))
    return (pack_tree if mode == "tree" else pack_listwise)(state, qs)


def q08b_request(vocab=248320, seed=0, state_tokens=2048):
    """Workload 2: a 2048-token state, one choice question of 24 tokens (9 header tokens, 3 options of 4 tokens,
    3 "Decision:" tokens), listwise."""
    tok = Tokens(vocab, seed)
    state = tok(state_tokens)
    q = Question("choice", tok(9), tuple(tok(4) for _ in range(3)), tok(3))
    return pack_listwise(state, [q])


def q4b_request(vocab=248320, seed=0, state_tokens=8192, questions=8, block_tokens=32, mode="tree"):
    """Workload 3: an 8192-token state, 8 choice questions of 32 block tokens with U{2..20} options of U{2..6}
    tokens each, tree layout (the listwise variant puts the block, the options and 3 decision tokens in one branch)."""
    tok = Tokens(vocab, seed)
    state = tok(state_tokens)
    qs = []
    for _ in range(questions):
        n = int(tok.rng.integers(2, 21))
        header = tok(block_tokens)
        options = tuple(tok(int(tok.rng.integers(2, 7))) for _ in range(n))
        qs.append(Question("choice", header, options, tok(3)))
    return (pack_tree if mode == "tree" else pack_listwise)(state, qs)


def stress_request(vocab=248320, seed=0, state_tokens=4096, block_tokens=32):
    """Workload 4: a 4096-token state, one choice with 255 options of 3 tokens, 15 choices with 8 options (3 tokens),
    8 scores with 5 levels (4 tokens) and 8 nouls (one 3-token leaf); 32-token blocks; tree layout."""
    tok = Tokens(vocab, seed)
    state = tok(state_tokens)
    qs = [Question("choice", tok(block_tokens), tuple(tok(3) for _ in range(255)))]
    qs += [Question("choice", tok(block_tokens), tuple(tok(3) for _ in range(8))) for _ in range(15)]
    qs += [Question("score", tok(block_tokens), tuple(tok(4) for _ in range(5))) for _ in range(8)]
    qs += [Question("noul", tok(block_tokens), (tok(3),)) for _ in range(8)]
    return pack_tree(state, qs)


def a3b_request(vocab=248320, seed=0, state_tokens=16384, block_tokens=32):
    """Workload 5: a 16384-token state, 8 choice questions of 32 block tokens and 4 options of 3 tokens, tree."""
    tok = Tokens(vocab, seed)
    state = tok(state_tokens)
    qs = [Question("choice", tok(block_tokens), tuple(tok(3) for _ in range(4))) for _ in range(8)]
    return pack_tree(state, qs)


WORKLOADS = {
    # id: (shape name, readout mode, request builder, batch)
    1: ("tiny", "listwise", tiny_request, 1),
    2: ("0.8b", "listwise", q08b_request, 64),
    3: ("4b", "tree", q4b_request, 16),
    4: ("0.8b", "tree", stress_request, 1),
    5: ("35b-a3b", "tree", a3b_request, 8),
}


def workload_requests(wid, seed=0, batch=None, **overrides):
    """The packed requests of workload `wid` (request j uses seed + j)."""
    shape_name, mode, builder, default_batch = WORKLOADS[wid]
    shape = SHAPES[shape_name]
    n = default_batch if batch is None else batch
    kwargs = dict(overrides)
    kwargs.setdefault("vocab", shape.vocab)
    return [builder(seed=seed + j, **kwargs) for j in range(n)]
