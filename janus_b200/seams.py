"""Drop-in seams with the reference's own signatures, over the packed-level ops of libjanus_b200.

The reference's hybrid runner reaches its hot ops through four replaceable points, and each function here keeps the
signature, argument meaning and result layout of the one it replaces, so the reference's `HybridBackbone`,
`LevelGraphs`, buckets and `Worker` stay as they are:

1. the chunked gated delta rule `rule(q, k, v, *, g, beta, initial_state, output_final_state,
   use_qk_l2norm_in_kernel[, chunk_size])` (fla's `chunk_gated_delta_rule`, selected by `chunk_rule`,
   janus/hybrid.py:100-125, called at :771-772 and :1061-1069): `chunk_gated_delta_rule`;
2. the HF experts call `experts(hidden_states [S, H], top_k_index [S, k], top_k_weights [S, k]) -> [S, H]`
   (janus/hybrid.py:551-572): `W4A16Experts`;
3. the attention of a level, `state_attention(m, h, cos, sin, mask, state, fused)` and
   `branch_attention(m, h, cos, sin, valid, plan, states, flex, fused)` -> (out [B, L, d], k, v)
   (janus/hybrid.py:943-989): `state_attention`, `branch_attention`;
4. the heads `PointerHead.forward(decision [d], options [n, d]) -> [n]` and `ScalarHead.forward(rows [n, d]) -> [n]`
   (janus/model.py:71-92): `PointerHead`, `ScalarHead`.

Each adapter maps the reference's padded [B, L, ...] level tensors onto this library's packed rows (row b = tokens
[b L, (b + 1) L)) and calls the C ABI ops (janus_b200.ops); none of them reads a device value on the host, so they
can run inside the reference's CUDA-graph capture. Level batches of the reference are right-padded
(janus/hybrid.py:1721-1741): a row's valid keys are a prefix of its row, so a causal query never sees a pad key and
an ancestor row's keys are the range [g L_l, g L_l + valid_l[g]). Pad queries get finite outputs the caller ignores.

`install(hybrid, model=None)` patches 1 and 3 into the reference's `janus.hybrid` module by attribute, the way
janus/latency.py:48-50 patches its timers, and swaps the head module of a `DecisionModel`; `uninstall` restores.
Experts are per layer: `W4A16Experts.replace(layer.mlp, codes...)`.
"""

import math

import torch
import torch.nn.functional as F

from . import ops

BF16, F32, I32 = torch.bfloat16, torch.float32, torch.int32
CHUNK = 64  # tokens per chunk of the chunk scan


def _rows(B, L, device):
    """row_start [B + 1] and row_of_token [B L] of B padded rows of L tokens (device arange: capture-safe)."""
    rs = (torch.arange(B + 1, device=device, dtype=I32) * L).contiguous()
    rot = torch.arange(B, device=device, dtype=I32).repeat_interleave(L).contiguous()
    return rs, rot


def _l2norm(x, eps=1e-6):
    x = x.float()
    return x * torch.rsqrt((x * x).sum(-1, keepdim=True) + eps)


# ------------------------------------------------------------------------------------------------ 1. the chunk rule

def chunk_gated_delta_rule(q, k, v, g=None, beta=None, scale=None, initial_state=None, output_final_state=False,
                           use_qk_l2norm_in_kernel=False, chunk_size=64, cu_seqlens=None, **_):
    """fla's chunk_gated_delta_rule: q, k [B, T, Hk, Dk], v [B, T, Hv, Dv] (Hk divides Hv: value head h reads qk head
    h // (Hv / Hk) in place), g (log decay) and beta [B, T, Hv], initial_state [B, Hv, Dk, Dv] fp32 or None. Returns
    (o [B, T, Hv, Dv] in q's dtype, final state [B, Hv, Dk, Dv] fp32 or None). `cu_seqlens` (int [N + 1], B = 1)
    gives packed rows instead of B rows of T tokens. `chunk_size` is accepted and ignored: the rule runs in 64-token
    chunks (other chunk sizes differ by fp32 accumulation order only, janus/hybrid.py:113-118). Rows with
    Dk = Dv = 128 run the tcgen05 chunk scan, other head dims the token-by-token kernel."""
    B, T, Hk, Dk = q.shape
    Hv, Dv = v.shape[2], v.shape[3]
    if k.shape != q.shape or v.shape[:2] != (B, T) or Hv % Hk:
        raise ValueError("chunk_gated_delta_rule: q, k [B, T, Hk, Dk] and v [B, T, Hv, Dv] with Hk dividing Hv")
    dev = q.device
    if use_qk_l2norm_in_kernel:
        q, k = _l2norm(q), _l2norm(k)
    qp = q.reshape(B * T, Hk, Dk).to(BF16).contiguous()
    kp = k.reshape(B * T, Hk, Dk).to(BF16).contiguous()
    vp = v.reshape(B * T, Hv, Dv).to(BF16).contiguous()
    gp = g.reshape(B * T, Hv).to(F32).contiguous()
    bp = beta.reshape(B * T, Hv).to(F32).contiguous()
    if cu_seqlens is not None:
        if B != 1:
            raise ValueError("chunk_gated_delta_rule: cu_seqlens needs B = 1")
        rs = cu_seqlens.to(dev, I32).contiguous()
        n_rows = rs.shape[0] - 1
        lengths = rs[1:] - rs[:-1]
        # chunk_start needs the row lengths: a host read, so packed rows (cu_seqlens) are not capture-safe
        n_chunk = ((lengths + CHUNK - 1) // CHUNK).cpu()
        cs = torch.cat([torch.zeros(1, dtype=torch.int64), n_chunk.cumsum(0)]).to(dev, I32)
        n_chunks = int(n_chunk.sum())
    else:
        n_rows = B
        rs, _ = _rows(B, T, dev)
        per = (T + CHUNK - 1) // CHUNK
        cs = (torch.arange(B + 1, device=dev, dtype=I32) * per).contiguous()
        n_chunks = B * per
    state = None if initial_state is None else initial_state.to(F32).contiguous()
    if state is not None and state.shape != (n_rows, Hv, Dk, Dv):
        raise ValueError(f"initial_state must be [{n_rows}, {Hv}, {Dk}, {Dv}]")
    scale = Dk ** -0.5 if scale is None else float(scale)
    if Dk == 128 and Dv == 128:
        own = torch.arange(n_rows, device=dev, dtype=I32) if state is not None else None
        o, S = ops.gdn_chunk_scan(qp, kp, vp, gp, bp, rs, cs, n_chunks, state, own, bool(output_final_state), scale)
    else:
        o, S = ops.gdn_fork_recurrent(qp, kp, vp, gp, bp, rs, torch.arange(n_rows + 1, device=dev, dtype=I32),
                                      state, bool(output_final_state), scale)
    return o.view(B, T, Hv, Dv).to(q.dtype if q.dtype in (BF16, torch.float16, F32) else BF16), S


# ------------------------------------------------------------------------------------------------ 2. the experts

class W4A16Experts(torch.nn.Module):
    """The HF experts module of a Qwen3.5-MoE layer on int4 weights (group 128, bf16 scales; codes two per byte, the
    even element in the low nibble): `forward(hidden_states [S, H], top_k_index [S, k], top_k_weights [S, k])` is
    sum_j w_j * down_e(silu(gate_e(x)) * up_e(x)) over the k routed experts e = top_k_index[s, j] (transformers
    qwen3_5_moe experts, janus/hybrid.py:551-572), the expert weights decoded to bf16 in registers inside the
    tcgen05 grouped GEMMs. gate_up codes [E, 2I, H/2] (rows 0..I-1 gate, I..2I-1 up), down codes [E, H, I/2]."""

    def __init__(self, gate_up_codes, gate_up_scales, down_codes, down_scales):
        super().__init__()
        self.gate_up_codes, self.gate_up_scales = gate_up_codes, gate_up_scales
        self.down_codes, self.down_scales = down_codes, down_scales
        self.num_experts = gate_up_codes.shape[0]

    @classmethod
    def replace(cls, moe_block, gate_up_codes, gate_up_scales, down_codes, down_scales):
        """Swap the experts module of a reference MoE block (`layer.mlp.experts`) for this one; returns it."""
        dev = next(iter(moe_block.parameters())).device
        mod = cls(*(t.to(dev).contiguous() for t in (gate_up_codes, gate_up_scales, down_codes, down_scales)))
        moe_block.experts = mod
        return mod

    def forward(self, hidden_states, top_k_index, top_k_weights):
        S, H = hidden_states.shape
        k = top_k_index.shape[1]
        x = hidden_states.to(BF16).contiguous()
        ids = top_k_index.to(I32).contiguous()
        plan = ops.moe_plan(ids, self.num_experts)
        h = ops.moe_grouped_w4a16(x, self.gate_up_codes, self.gate_up_scales, plan, True, k)
        y2 = ops.moe_grouped_w4a16(h, self.down_codes, self.down_scales, plan, False, k,
                                  topk_w=top_k_weights.to(F32).reshape(-1).contiguous())
        return ops.moe_reduce_slots(y2, k, ids).to(hidden_states.dtype)


# ------------------------------------------------------------------------------------------------ 3. attention

def _rope(x, cos, sin):
    """Rotary on the first R dims of x [B, L, H, D] (cos/sin [B, L, R], rotate_half; transformers qwen3_5
    apply_rotary_pos_emb with the partial rotary factor), fp32."""
    R = cos.shape[-1]
    c, s = cos.float()[:, :, None], sin.float()[:, :, None]
    xr, xp = x[..., :R], x[..., R:]
    half = torch.cat([-xr[..., R // 2:], xr[..., :R // 2]], dim=-1)
    return torch.cat([xr * c + half * s, xp], dim=-1)


def _qkv(m, h, cos, sin):
    """q [B L, Hq, D] (RMSNorm(1 + w) per head, rotary; fp32 math, rounded once to bf16), k, v [B, L, Hkv, D] and the
    gate view [B L, Hq, D] of one Qwen3_5Attention layer `m` (its merged `serve_qkv` weight when enable_fast made one,
    janus/hybrid.py:919-940)."""
    B, L, _ = h.shape
    D = m.head_dim
    if hasattr(m, "serve_qkv"):
        qg, k, v = F.linear(h, m.serve_qkv).split(m.serve_split, dim=-1)
    else:
        qg, k, v = m.q_proj(h), m.k_proj(h), m.v_proj(h)
    qg = qg.reshape(B, L, -1, 2 * D).to(BF16)
    Hq = qg.shape[2]
    norm = lambda t, w, eps: t.float() * torch.rsqrt(t.float().pow(2).mean(-1, keepdim=True) + eps) * (1.0 + w.float())
    q = _rope(norm(qg[..., :D], m.q_norm.weight, m.q_norm.eps), cos, sin).to(BF16).reshape(B * L, Hq, D)
    k = _rope(norm(k.reshape(B, L, -1, D), m.k_norm.weight, m.k_norm.eps), cos, sin).to(BF16)
    v = v.reshape(B, L, -1, D).to(BF16)
    gate = qg.reshape(B * L, Hq, 2 * D)[:, :, D:]
    return q, k, v, gate


def _tiles(B, L, tq, device):
    """Query tiles of at most tq tokens that never leave a row (B padded rows of L tokens), int32 [n, 2]."""
    per = (L + tq - 1) // tq
    starts = (torch.arange(B, device=device, dtype=I32)[:, None] * L
              + torch.arange(per, device=device, dtype=I32)[None, :] * tq).reshape(-1)
    ends = torch.minimum(starts + tq, (starts // L + 1) * L)
    return torch.stack([starts, ends], 1).contiguous()


def _token_major(t):
    """[B, Hkv, L, D] (the reference's key/value layout) -> [B L, Hkv, D] bf16."""
    return t.transpose(1, 2).reshape(-1, t.shape[1], t.shape[3]).to(BF16).contiguous()


def _head_major(t, B, L):
    """[B, L, Hkv, D] -> [B, Hkv, L, D]."""
    return t.reshape(B, L, t.shape[-2], t.shape[-1]).transpose(1, 2)


def _attend(m, h, q, k, v, gate, ancestors):
    """The tree attention of B padded rows of L own tokens over `ancestors` (a list of (keys [T_l, Hkv, D], values,
    lo [B], hi [B]) per ancestor level), output gate in the epilogue, then o_proj. Returns [B, L, d]."""
    B, L, _ = h.shape
    Hq, D = q.shape[1], q.shape[2]
    Hkv = k.shape[2]
    dev = h.device
    rs, rot = _rows(B, L, dev)
    tiles = _tiles(B, L, ops.tree_attention_tile_tokens(D, Hq, Hkv), dev)
    keys = [a[0] for a in ancestors] + [k.reshape(B * L, Hkv, D).contiguous()]
    values = [a[1] for a in ancestors] + [v.reshape(B * L, Hkv, D).contiguous()]
    out = ops.tree_attention(q, keys, values, [a[2] for a in ancestors], [a[3] for a in ancestors], rs, rot, tiles,
                             gate, m.scaling)
    return m.o_proj(out.view(B, L, Hq * D).to(h.dtype))


def state_attention(m, h, cos, sin, mask, state, fused=None):
    """The level-0 attention (janus/hybrid.py:943-955): each row's queries over its accumulated keys (`state`: the
    keys and values [B, Hkv, S0, D] of the row's earlier state chunks, or empty) and its own keys causally; `mask`
    (the padding mask of right-padded rows) changes nothing for the valid queries and is not read. Returns
    (out [B, L, d], keys [B, Hkv, S0 + L, D], values)."""
    B, L, _ = h.shape
    q, k, v, gate = _qkv(m, h, cos, sin)
    ancestors = []
    if state:
        k0, v0 = state
        S0 = k0.shape[2]
        lo = torch.arange(B, device=h.device, dtype=I32) * S0
        ancestors.append((_token_major(k0), _token_major(v0), lo, (lo + S0).contiguous()))
    out = _attend(m, h, q, k, v, gate, ancestors)
    kh, vh = _head_major(k, B, L), _head_major(v, B, L)
    if state:
        kh, vh = torch.cat([state[0].to(kh.dtype), kh], dim=2), torch.cat([state[1].to(vh.dtype), vh], dim=2)
    return out, kh, vh


def branch_attention(m, h, cos, sin, valid, plan, states, flex=False, fused=None):
    """A branch level (janus/hybrid.py:958-989): every row attends to its ancestors' valid keys and its own causally,
    one softmax over their union. plan = (kv_valid_0 [B_0, L_0], slots_0 [G_0, R_0], back_0 [B], ...) per ancestor
    level, back = group * R + slot (group = the ancestor row); states = (k_0, v_0, ...) [B_l, Hkv, L_l, D]. Returns
    (out [B, L, d], k [B, Hkv, L, D], v)."""
    B, L, _ = h.shape
    q, k, v, gate = _qkv(m, h, cos, sin)
    ancestors = []
    for level, (kv_valid, slots, back) in enumerate(zip(plan[0::3], plan[1::3], plan[2::3])):
        k_a, v_a = states[2 * level], states[2 * level + 1]
        L_a = k_a.shape[2]
        group = back.long() // slots.shape[1]
        lo = group * L_a
        hi = lo + kv_valid.long().sum(1)[group]
        ancestors.append((_token_major(k_a), _token_major(v_a), lo.to(I32).contiguous(), hi.to(I32).contiguous()))
    out = _attend(m, h, q, k, v, gate, ancestors)
    return out, _head_major(k, B, L), _head_major(v, B, L)


# ------------------------------------------------------------------------------------------------ 4. the heads

class ScalarHead(torch.nn.Module):
    """ScalarHead (janus/model.py:85-92): LayerNorm(rows) . w + b in fp32, rows [n, d] final-normed hidden states."""

    def __init__(self, ln_w, ln_b, ln_eps, w_out, b_out):
        super().__init__()
        self.ln_w, self.ln_b, self.ln_eps = ln_w.float().contiguous(), ln_b.float().contiguous(), float(ln_eps)
        self.w_out, self.b_out = w_out.float().reshape(-1).contiguous(), b_out.float().reshape(1).contiguous()

    @classmethod
    def from_module(cls, head):
        return cls(head.norm.weight.data, head.norm.bias.data, head.norm.eps, head.out.weight.data, head.out.bias.data)

    def forward(self, reps):
        x = reps.float().contiguous()
        rows = torch.arange(x.shape[0], device=x.device, dtype=I32)
        return ops.head_scalar(x, rows, None, 0.0, self.ln_w, self.ln_b, self.ln_eps, self.w_out, self.b_out)


class PointerHead(torch.nn.Module):
    """PointerHead (janus/model.py:71-82): (LN(options) Wk) . (LN(decision) Wq) / sqrt(rank), fp32."""

    def __init__(self, ln_w, ln_b, ln_eps, wq, wk):
        super().__init__()
        self.ln_w, self.ln_b, self.ln_eps = ln_w.float().contiguous(), ln_b.float().contiguous(), float(ln_eps)
        self.wq, self.wk = wq.float().contiguous(), wk.float().contiguous()
        self.scale = math.sqrt(wq.shape[0])

    @classmethod
    def from_module(cls, head):
        return cls(head.norm.weight.data, head.norm.bias.data, head.norm.eps, head.query.weight.data,
                   head.key.weight.data)

    def forward(self, decision, options):
        x = torch.cat([options.float().reshape(-1, options.shape[-1]), decision.float().reshape(1, -1)]).contiguous()
        n = x.shape[0] - 1
        dev = x.device
        rows = torch.arange(n, device=dev, dtype=I32)
        return ops.head_pointer(x, rows, torch.zeros(n, device=dev, dtype=I32),
                                torch.full((1,), n, device=dev, dtype=I32), None, 0.0, self.ln_w, self.ln_b,
                                self.ln_eps, self.wq, self.wk)


# ------------------------------------------------------------------------------------------------ install

_SAVED = {}


def install(hybrid, model=None):
    """Patch the chunk rule and the two attention functions into the reference's `janus.hybrid` module (passed in:
    this package never imports the reference) and, with `model` (a janus.model.DecisionModel), its head. The rule
    replaces fla's in both of its roles (FLA_CHUNK_RULE, and FLA_RECURRENT_RULE for the short rows): this one
    takes rows of any length."""
    _SAVED.setdefault(id(hybrid), (hybrid, {n: getattr(hybrid, n) for n in
                                            ("FLA_CHUNK_RULE", "FLA_RECURRENT_RULE", "state_attention", "branch_attention")}))
    hybrid.FLA_CHUNK_RULE = chunk_gated_delta_rule
    hybrid.FLA_RECURRENT_RULE = chunk_gated_delta_rule
    hybrid.state_attention = state_attention
    hybrid.branch_attention = branch_attention
    if model is not None:
        _SAVED.setdefault(id(model), (model, {"head": model.head}))
        cls = PointerHead if hasattr(model.head, "query") else ScalarHead
        model.head = cls.from_module(model.head)


def uninstall(*targets):
    """Undo `install` on the given modules / models (all of them by default)."""
    keys = [id(t) for t in targets] if targets else list(_SAVED)
    for key in keys:
        obj, attrs = _SAVED.pop(key)
        for name, value in attrs.items():
            setattr(obj, name, value)
