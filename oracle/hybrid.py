"""CPU oracle of the decision readout: a plain fp32 restatement of the reference's forward pass.

TEST INFRASTRUCTURE ONLY. Nothing in the `janus_b200` package imports this module; the tests, the smoke check of
`__graft_entry__` and the CPU-baseline leg of `bench.py` call it as the checker (and as the timed CPU baseline),
never as the product path.

What it restates (reference files cited per function; transformers 5.5.0 for the HF modules the reference reuses):
the Qwen3.5 hybrid decoder (Gated DeltaNet + gated full attention, dense SwiGLU or sparse MoE feed-forward) run as a
tree of segments (janus/hybrid.py:1-62): the state segment first, then every branch segment continuing from its
parent segment's DeltaNet states (conv tail + recurrent matrix, janus/hybrid.py:1082-1083) and attending to its
ancestors' keys plus its own tokens causally (janus/attention.py:10-23 restricted to one root-to-leaf path),
then the readout heads (janus/model.py:71-92, 319-366) and the temperature softmax (janus/server.py:277-282).
Everything runs in fp32 on the weights as given (bf16-rounded values); one segment at a time, no padding.

Pinned against the reference itself: tests/golden/make_golden.py runs janus.hybrid.HybridBackbone + janus.model
heads on the same seeded weights and requests and stores the probabilities; tests/test_oracle.py checks this
module against them.
"""

import math
import time

import torch
import torch.nn.functional as F

LINEAR = "linear_attention"


# ------------------------------------------------------------------------------------------------------------ ops

def rmsnorm(x, w, eps):
    """Qwen3_5RMSNorm: x * rsqrt(mean(x^2) + eps) * (1 + w) (transformers qwen3_5 :711-725; janus/hybrid.py:250-254)."""
    x = x.float()
    return x * torch.rsqrt(x.pow(2).mean(-1, keepdim=True) + eps) * (1.0 + w.float())


def gated_rmsnorm(core, z, w, eps):
    """Qwen3_5RMSNormGated over the value head: rmsnorm(core) * w * silu(z) (transformers :175-190;
    janus/hybrid.py:241-247)."""
    h = core.float()
    h = h * torch.rsqrt(h.pow(2).mean(-1, keepdim=True) + eps)
    return w.float() * h * F.silu(z.float())


def l2norm(x, eps=1e-6):
    """fla's l2norm: x * rsqrt(sum(x^2) + eps) (transformers :228-231)."""
    return x * torch.rsqrt((x * x).sum(-1, keepdim=True) + eps)


def _keep(x):
    return x


def bf16_round(x):
    """x rounded to bf16 (nearest even) and back to fp32: a tensor the B200 path stores in bf16."""
    return x.to(torch.bfloat16).float()


def delta_prologue(mixed, b, a, tail, conv_w, A_log, dt_bias, key_dim, k_dim, v_dim, rnd=_keep):
    """The glue between a DeltaNet layer's projections and its recurrence (janus/hybrid.py:220-238, 276-301) for one
    unpadded row: causal depthwise conv (K taps) over [tail || mixed], silu, head split, l2-normalised q and k,
    beta = sigmoid(b), g = -exp(A_log) * softplus(a + dt_bias). mixed [L, C], tail [C, K-1] or None.
    Returns q [L, Hk, Dk], k, v [L, Hv, Dv], g [L, Hv], beta [L, Hv], new tail [C, K-1] (the last K-1 conv inputs);
    `rnd` is applied to q, k and v (the tensors the next op reads)."""
    L, C = mixed.shape
    K = conv_w.shape[-1]
    if tail is None:
        tail = mixed.new_zeros(C, K - 1)
    ext = torch.cat([tail.t().float(), mixed.float()], dim=0)  # [K-1+L, C]
    new_tail = ext[L:].t().contiguous()
    w = conv_w.reshape(C, K).float()
    conv = sum(ext[j:j + L] * w[:, j] for j in range(K))
    act = F.silu(conv)
    q, k, v = torch.split(act, [key_dim, key_dim, C - 2 * key_dim], dim=-1)
    q = l2norm(q.reshape(L, -1, k_dim))
    k = l2norm(k.reshape(L, -1, k_dim))
    v = v.reshape(L, -1, v_dim)
    beta = torch.sigmoid(b.float())
    g = -A_log.float().exp() * F.softplus(a.float() + dt_bias.float())
    return rnd(q), rnd(k), rnd(v), g, beta, new_tail


def _expand_heads(x, hv):
    """GQA of the DeltaNet: value head h reads qk head h // (Hv / Hk) (repeat_interleave, janus/hybrid.py:369-371)."""
    return x.repeat_interleave(hv // x.shape[1], dim=1) if x.shape[1] != hv else x


def delta_recurrent(q, k, v, g, beta, state=None):
    """The gated delta rule token by token (transformers torch_recurrent_gated_delta_rule :314-354), one row:
    S <- S * exp(g_t);  S <- S + k_t (beta_t (v_t - S^T k_t))^T;  o_t = S^T q_t / sqrt(Dk).
    q, k [L, Hk, Dk] (already l2-normalised), v [L, Hv, Dv], g, beta [L, Hv], state [Hv, Dk, Dv] or None.
    Returns o [L, Hv, Dv], final state [Hv, Dk, Dv]."""
    L, Hv, Dv = v.shape
    q, k = _expand_heads(q.float(), Hv), _expand_heads(k.float(), Hv)
    Dk = q.shape[-1]
    q = q / math.sqrt(Dk)
    S = q.new_zeros(Hv, Dk, Dv) if state is None else state.float().clone()
    out = q.new_zeros(L, Hv, Dv)
    for t in range(L):
        S = S * g[t].float().exp()[:, None, None]
        kv = (S * k[t][:, :, None]).sum(1)
        delta = (v[t].float() - kv) * beta[t].float()[:, None]
        S = S + k[t][:, :, None] * delta[:, None, :]
        out[t] = (S * q[t][:, :, None]).sum(1)
    return out, S


def delta_chunked(q, k, v, g, beta, state=None, chunk=64):
    """The same rule in chunks (transformers torch_chunk_gated_delta_rule :234-311), one row: within a chunk the
    WY form (I - tril(diag(beta) K K^T * decay))^-1 by forward substitution, across chunks the state recurrence.
    Same arguments and results as `delta_recurrent`; differs from it by fp32 accumulation order only."""
    L, Hv, Dv = v.shape
    q, k = _expand_heads(q.float(), Hv), _expand_heads(k.float(), Hv)
    Dk = q.shape[-1]
    pad = (-L) % chunk
    tr = lambda x: F.pad(x.float().transpose(0, 1), (0, 0, 0, pad)) if x.dim() == 3 else F.pad(x.float().t(), (0, pad))
    q, k, v, beta, g = tr(q) / math.sqrt(Dk), tr(k), tr(v), tr(beta), tr(g)  # [Hv, T, D] / [Hv, T]
    n = q.shape[1] // chunk
    q, k, v = (x.reshape(Hv, n, chunk, -1) for x in (q, k, v))
    beta, g = beta.reshape(Hv, n, chunk), g.reshape(Hv, n, chunk).cumsum(-1)
    k_beta, v_beta = k * beta[..., None], v * beta[..., None]
    decay = (g[..., :, None] - g[..., None, :]).tril().exp().tril()
    upper = torch.triu(torch.ones(chunk, chunk, dtype=torch.bool), 0)
    A = -((k_beta @ k.transpose(-1, -2)) * decay).masked_fill(upper, 0)
    for i in range(1, chunk):
        A[..., i, :i] = A[..., i, :i] + (A[..., i, :i, None] * A[..., :i, :i]).sum(-2)
    A = A + torch.eye(chunk)
    u = A @ v_beta
    w = A @ (k_beta * g.exp()[..., None])
    S = q.new_zeros(Hv, Dk, Dv) if state is None else state.float().clone()
    out = torch.zeros_like(u)
    strict = torch.triu(torch.ones(chunk, chunk, dtype=torch.bool), 1)
    for c in range(n):
        qc, kc = q[:, c], k[:, c]
        attn = (qc @ kc.transpose(-1, -2) * decay[:, c]).masked_fill(strict, 0)
        v_new = u[:, c] - w[:, c] @ S
        out[:, c] = (qc * g[:, c, :, None].exp()) @ S + attn @ v_new
        S = S * g[:, c, -1, None, None].exp() + (kc * (g[:, c, -1, None] - g[:, c]).exp()[..., None]).transpose(-1, -2) @ v_new
    out = out.reshape(Hv, n * chunk, Dv)[:, :L].transpose(0, 1)
    return out, S


def rope_tables(positions, rotary_dim, theta):
    """cos, sin [L, rotary_dim] of Qwen3_5TextRotaryEmbedding for text positions (identical on the three M-RoPE axes,
    so the interleave is the identity; transformers :85-173)."""
    inv = 1.0 / (theta ** (torch.arange(0, rotary_dim, 2, dtype=torch.int64).float() / rotary_dim))
    freqs = positions.float()[:, None] * inv[None]
    emb = torch.cat([freqs, freqs], dim=-1)
    return emb.cos(), emb.sin()


def apply_rope(x, cos, sin):
    """Rotary on the first rotary_dim dims of x [L, H, D] with rotate_half (transformers :536-579)."""
    r = cos.shape[-1]
    xr, xp = x[..., :r], x[..., r:]
    half = torch.cat([-xr[..., r // 2:], xr[..., :r // 2]], dim=-1)
    return torch.cat([xr * cos[:, None] + half * sin[:, None], xp], dim=-1)


def attention(q, k_all, v_all, n_prefix, scale):
    """Softmax attention of the L own queries q [L, Hq, D] over keys [n_prefix + L, Hkv, D]: every prefix (ancestor)
    key and the own keys causally, the tree rule along one root-to-leaf path (janus/attention.py:10-23). GQA: query
    head h reads kv head h // (Hq / Hkv), folded without repeating the keys. Query chunks bound the score matrix.
    Returns [L, Hq, D]."""
    L, Hq, D = q.shape
    T, Hkv, _ = k_all.shape
    grp = Hq // Hkv
    kt = k_all.float().permute(1, 2, 0)            # [Hkv, D, T]
    vt = v_all.float().transpose(0, 1)             # [Hkv, T, D]
    qt = q.float().view(L, Hkv, grp, D).permute(1, 2, 0, 3)  # [Hkv, G, L, D]
    out = torch.empty(Hkv, grp, L, D)
    step = max(1, (256 << 20) // (4 * Hq * max(T, 1)))
    keys = torch.arange(T)
    for a in range(0, L, step):
        b = min(L, a + step)
        s = torch.matmul(qt[:, :, a:b].reshape(Hkv, grp * (b - a), D), kt).view(Hkv, grp, b - a, T) * scale
        allowed = keys[None, :] <= (n_prefix + torch.arange(a, b))[:, None]
        s = s.masked_fill(~allowed, float("-inf"))
        p = torch.softmax(s, dim=-1).view(Hkv, grp * (b - a), T)
        out[:, :, a:b] = torch.matmul(p, vt).view(Hkv, grp, b - a, D)
    return out.permute(2, 0, 1, 3).reshape(L, Hq, D)


def moe_block(x, p, shape, rnd=_keep):
    """Qwen3_5MoeSparseMoeBlock (transformers qwen3_5_moe :754-791): router softmax (fp32) -> top-k -> renormalise;
    routed SwiGLU experts weighted by the routing weights; the shared expert times sigmoid(x . w_gate). `rnd` marks
    the tensors stored between ops: silu(gate) * up per assignment, each expert's weighted output row, the shared
    expert's projections, and the block output."""
    logits = x @ p["gate.weight"].t()
    probs = torch.softmax(logits, dim=-1)
    top, idx = torch.topk(probs, shape.top_k, dim=-1)
    top = top / top.sum(-1, keepdim=True)
    out = torch.zeros_like(x)
    gu, dn = p["experts.gate_up_proj"], p["experts.down_proj"]
    I = shape.moe_intermediate
    for e in torch.unique(idx).tolist():
        tok, slot = torch.where(idx == e)
        h = x[tok] @ gu[e].t()
        h = rnd(F.silu(h[:, :I]) * h[:, I:])
        out.index_add_(0, tok, rnd((h @ dn[e].t()) * top[tok, slot, None]))
    sh = rnd(F.silu(rnd(x @ p["shared_expert.gate_proj.weight"].t())) * rnd(x @ p["shared_expert.up_proj.weight"].t()))
    sh = rnd(sh @ p["shared_expert.down_proj.weight"].t())
    return rnd(out + torch.sigmoid(x @ p["shared_expert_gate.weight"].t()) * sh)


def mlp(x, p, rnd=_keep):
    """Qwen3_5MLP: down(silu(gate(x)) * up(x)) (transformers :695-708); `rnd` marks the stored tensors (the gate and
    up projections, their SwiGLU product, the output)."""
    h = rnd(F.silu(rnd(x @ p["gate_proj.weight"].t())) * rnd(x @ p["up_proj.weight"].t()))
    return rnd(h @ p["down_proj.weight"].t())


def layer_norm(x, w, b, eps=1e-5):
    return F.layer_norm(x.float(), (x.shape[-1],), w.float(), b.float(), eps)


def pointer_head(decision, options, p):
    """PointerHead (janus/model.py:71-82): LN(decision) Wq . LN(options) Wk / sqrt(rank), fp32."""
    w, b = p["head.norm.weight"], p["head.norm.bias"]
    query = layer_norm(decision, w, b) @ p["head.query.weight"].float().t()
    keys = layer_norm(options, w, b) @ p["head.key.weight"].float().t()
    return (keys * query).sum(-1) / math.sqrt(p["head.query.weight"].shape[0])


def scalar_head(rows, p):
    """ScalarHead (janus/model.py:85-92): LN(rows) w + b, fp32."""
    return (layer_norm(rows, p["head.norm.weight"], p["head.norm.bias"]) @ p["head.out.weight"].float().t() + p["head.out.bias"].float())[:, 0]


def int4_dequantize(packed, scales, group=128):
    """W4A16 int4 expert weights: two's-complement codes two per byte (even element in the low nibble) times one bf16
    scale per `group` consecutive input elements, exact in fp32 and rounded once to bf16 (the rounding convention
    of janus/moe_w4a16.py:9-11 for its NVFP4 codes)."""
    lo, hi = (packed & 15).long(), (packed >> 4).long()
    codes = torch.stack([lo, hi], dim=-1).flatten(-2)
    codes = torch.where(codes >= 8, codes - 16, codes).float()
    K = codes.shape[-1]
    w = codes.view(*codes.shape[:-1], K // group, group) * scales.float()[..., None]
    return w.reshape(codes.shape).to(torch.bfloat16)


def e2m1_decode(codes):
    """4-bit e2m1 codes (bit 3 sign, bits 2-1 exponent, bit 0 mantissa) to fp32: 0, 0.5, 1, 1.5, 2, 3, 4, 6 and their
    negatives (janus/hybrid.py:400-405)."""
    m = (codes & 1).float()
    e = ((codes >> 1) & 3).float()
    mag = torch.where(e == 0, 0.5 * m, (1.0 + 0.5 * m) * torch.exp2(e - 1.0))
    return torch.where((codes & 8) != 0, -mag, mag)


def nvfp4_dequantize(packed, block_scales, global_scale, block=16):
    """NVFP4 expert weights (the reference's own MoE format, janus/hybrid.py:418-425): e2m1 codes two per byte (the
    even element in the low nibble), one e4m3 scale per `block` consecutive inputs, an fp32 global scale per row
    ([..., rows] or broadcastable). The value is e2m1 * (scale * global) in fp32 (the scale product first, as the
    reference computes it), rounded once to bf16."""
    codes = torch.stack([packed & 15, packed >> 4], dim=-1).flatten(-2)
    s = block_scales.float() * global_scale.float()[..., None]
    K = codes.shape[-1]
    v = e2m1_decode(codes).view(*codes.shape[:-1], K // block, block) * s[..., None]
    return v.reshape(codes.shape).to(torch.bfloat16)


def tree_levels(segment_ids, parents):
    """Segments grouped by depth (janus/hybrid.py:128-153): [(segment, start, end)] per level."""
    seg = segment_ids.tolist()
    par = parents.tolist()
    spans = {}
    for i, s in enumerate(seg):
        a, b = spans.get(s, (i, i))
        if s in spans and b != i:
            raise ValueError(f"segment {s} is not contiguous")
        spans[s] = (a, i + 1)
    depth, levels = {}, []
    for s in range(len(par)):
        if s not in spans:
            raise ValueError(f"segment {s} has no tokens")
        depth[s] = 0 if s == 0 else depth[par[s]] + 1
        while len(levels) <= depth[s]:
            levels.append([])
        levels[depth[s]].append((s, *spans[s]))
    return levels


# ----------------------------------------------------------------------------------------------------------- model

class Oracle:
    """The fp32 tree forward of one model. `weights`: the name -> tensor dict of janus_b200.synthetic.make_weights
    (int4 expert stacks are dequantised here to their bf16 values).

    `storage`: "fp32" computes and keeps every tensor in fp32 (the reference's fp32 readout). "bf16" rounds to bf16
    exactly the tensors the B200 path stores in bf16 between its kernels (the normed GEMM inputs, every projection
    output, q/k/v after the DeltaNet prologue and after the attention q/k preparation, the delta rule's and the
    attention's outputs, the gated norm's output, the SwiGLU product, the MoE rows) while the residual stream, the
    DeltaNet g/beta and states, the router logits and the heads stay fp32 as there: the reference's algorithm at the
    storage precision of the B200 path, so the two differ only by what happens inside the kernels (accumulation
    order, the kernels' internal bf16 operands)."""

    def __init__(self, shape, weights, chunk_threshold=64, storage="fp32"):
        if storage not in ("fp32", "bf16"):
            raise ValueError("storage must be fp32 or bf16")
        self.shape = shape
        self.rnd = bf16_round if storage == "bf16" else _keep
        w = {}
        for name, t in weights.items():
            if name.endswith(".scales") or name.endswith(".global"):
                continue
            if name + ".global" in weights:  # NVFP4 experts: codes, e4m3 block scales, fp32 global per row
                t = nvfp4_dequantize(t, weights[name + ".scales"], weights[name + ".global"])
            elif name + ".scales" in weights:
                t = int4_dequantize(t, weights[name + ".scales"])
            w[name] = t.float()
        self.w = w
        self.chunk_threshold = chunk_threshold
        self.layer_seconds = {}  # wall seconds spent per layer kind (the CPU baseline scales a slice by these)

    def _p(self, prefix):
        n = len(prefix)
        return {k[n:]: v for k, v in self.w.items() if k.startswith(prefix)}

    def run_segment(self, ids, positions, parent_states, ancestor_kv):
        """All layers over one segment's tokens. parent_states: per DeltaNet layer (tail, S) or None; ancestor_kv:
        per attention layer (K, V) of the ancestors' tokens (concatenated root first) or None. Returns (final-norm
        hidden [L, H], per-layer own states: DeltaNet (tail, S) after the last token, attention (K, V) of the
        ancestors and this segment together)."""
        s = self.shape
        x = self.w["embed_tokens.weight"][ids]
        L = x.shape[0]
        cos, sin = rope_tables(positions, s.rotary_dim, s.rope_theta)
        states = []
        r = self.rnd
        for i, kind in enumerate(s.layer_types):
            t0 = time.perf_counter()
            p = self._p(f"layers.{i}.")
            h = r(rmsnorm(x, p["input_layernorm.weight"], s.rms_eps))
            if kind == LINEAR:
                a = {k[len("linear_attn."):]: v for k, v in p.items() if k.startswith("linear_attn.")}
                mixed = r(h @ a["in_proj_qkv.weight"].t())
                z = r(h @ a["in_proj_z.weight"].t()).reshape(L, s.lin_v_heads, s.lin_v_dim)
                b = r(h @ a["in_proj_b.weight"].t())
                aa = r(h @ a["in_proj_a.weight"].t())
                tail, S0 = parent_states[i] if parent_states is not None else (None, None)
                q, k, v, g, beta, new_tail = delta_prologue(mixed, b, aa, tail, a["conv1d.weight"], a["A_log"],
                                                            a["dt_bias"], s.key_dim, s.lin_k_dim, s.lin_v_dim, r)
                rule = delta_chunked if L > self.chunk_threshold else delta_recurrent
                core, S = rule(q, k, v, g, beta, S0)
                core = r(gated_rmsnorm(r(core), z, a["norm.weight"], s.rms_eps)).reshape(L, -1)
                h = r(core @ a["out_proj.weight"].t())
                states.append((new_tail, S))
            else:
                a = {k[len("self_attn."):]: v for k, v in p.items() if k.startswith("self_attn.")}
                D = s.head_dim
                qg = r(h @ a["q_proj.weight"].t()).reshape(L, s.heads, 2 * D)
                q, gate = qg[..., :D], qg[..., D:].reshape(L, -1)
                k = r(h @ a["k_proj.weight"].t()).reshape(L, s.kv_heads, D)
                v = r(h @ a["v_proj.weight"].t()).reshape(L, s.kv_heads, D)
                q = r(apply_rope(rmsnorm(q, a["q_norm.weight"], s.rms_eps), cos, sin))
                k = r(apply_rope(rmsnorm(k, a["k_norm.weight"], s.rms_eps), cos, sin))
                if ancestor_kv is not None and ancestor_kv[i] is not None:
                    k_all = torch.cat([ancestor_kv[i][0], k]); v_all = torch.cat([ancestor_kv[i][1], v])
                else:
                    k_all, v_all = k, v
                o = attention(q, k_all, v_all, k_all.shape[0] - L, D ** -0.5).reshape(L, -1)
                h = r(r(o * torch.sigmoid(gate)) @ a["o_proj.weight"].t())
                states.append((k_all, v_all))
            x = x + h
            h = r(rmsnorm(x, p["post_attention_layernorm.weight"], s.rms_eps))
            x = x + (moe_block(h, self._p(f"layers.{i}.mlp."), s, r) if s.moe else mlp(h, self._p(f"layers.{i}.mlp."), r))
            self.layer_seconds[kind] = self.layer_seconds.get(kind, 0.0) + time.perf_counter() - t0
        return rmsnorm(x, self.w["norm.weight"], s.rms_eps), states

    def encode(self, packed):
        """Final-norm hidden states [n, H] at the packed positions (janus/hybrid.py:1804-1807): every segment run
        from its parent's states, level by level."""
        ids = packed.input_ids[0]
        pos = packed.position_ids[0]
        parents = packed.parents.tolist()
        hidden = torch.zeros(ids.shape[0], self.shape.hidden)
        seg_states = {}
        has_children = set(parents[1:])  # only these segments' states are read again (a leaf's are dropped at once)
        for level in tree_levels(packed.segment_ids, packed.parents):
            for seg, start, end in level:
                if seg == 0:
                    parent_states = ancestor_kv = None
                else:
                    ps = seg_states[parents[seg]]
                    parent_states = [st if kind == LINEAR else None for st, kind in zip(ps, self.shape.layer_types)]
                    ancestor_kv = [st if kind != LINEAR else None for st, kind in zip(ps, self.shape.layer_types)]
                h, states = self.run_segment(ids[start:end], pos[start:end], parent_states, ancestor_kv)
                hidden[start:end] = h
                if seg in has_children:
                    seg_states[seg] = states
        return hidden

    def logits(self, packed, mode):
        """Per question the option logits (janus/model.py:319-366): tree mode reads every leaf's last token through
        the ScalarHead (noul: [0, z]); listwise scores the options against the decision row through the PointerHead."""
        hidden = self.encode(packed)
        out = [[None] * k for k in packed.option_counts]
        for br in packed.branches:
            if mode == "tree":
                z = scalar_head(hidden[list(br.option_positions)], self.w)
                if br.kind == "noul":
                    out[br.question_index] = [torch.zeros(()), z[0]]
                else:
                    for i, val in zip(br.option_indices, z):
                        out[br.question_index][i] = val
            else:
                z = pointer_head(hidden[br.decision_position], hidden[list(br.option_positions)], self.w)
                for i, val in zip(br.option_indices, z):
                    out[br.question_index][i] = val
        return [torch.stack(v) for v in out]


def probabilities(logits, temperatures=None):
    """Worker.probabilities (janus/server.py:277-282): per question softmax(logits / T), T = 1 without calibration."""
    temperatures = temperatures or [1.0] * len(logits)
    return [torch.softmax(z.float() / t, dim=-1) for z, t in zip(logits, temperatures)]
