"""The drop-in seams (janus_b200/seams.py) on the GPU against the CPU oracle, with the reference's argument layouts:
padded [B, L, ...] level tensors, fla's chunk-rule signature, the reference's branch plan (kv_valid, slots, back per
ancestor level) and head-major [B, Hkv, L, D] key/value states, the HF experts call, the head modules' forwards.
Inside the reference's runner itself the seams are checked on CPU (tests/test_seams.py).

bf16 outputs against fp32 restatements: 2e-2 absolute + relative on O(1) values (bf16 inputs and one output
rounding); fp32 states and logits as stated per test."""

import math

import numpy as np
import pytest
import torch

from oracle import hybrid as oracle

pytestmark = pytest.mark.gpu
BF = torch.bfloat16


def close(a, b, atol=2e-2, rtol=2e-2):
    np.testing.assert_allclose(a.detach().float().cpu().numpy(), b.detach().float().cpu().numpy(), atol=atol, rtol=rtol)


@pytest.mark.parametrize("dims", [(16, 32, 128, 200), (2, 4, 32, 40)])
def test_chunk_rule_with_the_fla_signature(dims):
    """B rows of T tokens, Hk qk heads read in place by Hv value heads, an initial and a final state; q/k normalised
    inside (use_qk_l2norm_in_kernel). Dk = 128 runs the tcgen05 chunk scan, Dk = 32 the token-by-token kernel."""
    from janus_b200.seams import chunk_gated_delta_rule
    Hk, Hv, D, T = dims
    B = 3
    g = torch.Generator().manual_seed(31)
    q = torch.randn(B, T, Hk, D, generator=g).to(BF)
    k = torch.randn(B, T, Hk, D, generator=g).to(BF)
    v = torch.randn(B, T, Hv, D, generator=g).to(BF)
    gg = -torch.rand(B, T, Hv, generator=g) * 0.3
    beta = torch.sigmoid(torch.randn(B, T, Hv, generator=g))
    s0 = torch.randn(B, Hv, D, D, generator=g) * 0.1
    o, S = chunk_gated_delta_rule(q.cuda(), k.cuda(), v.cuda(), g=gg.cuda(), beta=beta.cuda(), initial_state=s0.cuda(),
                                  output_final_state=True, use_qk_l2norm_in_kernel=True)
    assert o.shape == (B, T, Hv, D) and S.shape == (B, Hv, D, D)
    for b in range(B):
        qn = oracle.l2norm(q[b].float()).to(BF).float()
        kn = oracle.l2norm(k[b].float()).to(BF).float()
        ro, rS = oracle.delta_chunked(qn, kn, v[b].float(), gg[b], beta[b], s0[b])
        close(o[b], ro, atol=3e-2, rtol=3e-2)
        close(S[b], rS, atol=3e-2, rtol=3e-2)
    o2, S2 = chunk_gated_delta_rule(q.cuda(), k.cuda(), v.cuda(), g=gg.cuda(), beta=beta.cuda(),
                                    use_qk_l2norm_in_kernel=True)
    assert S2 is None
    ro, _ = oracle.delta_chunked(oracle.l2norm(q[1].float()).to(BF).float(), oracle.l2norm(k[1].float()).to(BF).float(),
                                 v[1].float(), gg[1], beta[1], None)
    close(o2[1], ro, atol=3e-2, rtol=3e-2)


class _Norm(torch.nn.Module):
    def __init__(self, D, g):
        super().__init__()
        self.weight = torch.nn.Parameter((0.1 * torch.randn(D, generator=g)).to(BF))
        self.eps = 1e-6


class _Attn(torch.nn.Module):
    """A Qwen3_5Attention-shaped module: q_proj (query and gate per head), k_proj, v_proj, o_proj, q/k norms."""

    def __init__(self, d, Hq, Hkv, D, g):
        super().__init__()
        lin = lambda i, o: torch.nn.Parameter((torch.randn(o, i, generator=g) * 0.05).to(BF))
        self.head_dim, self.scaling = D, D ** -0.5
        self.q_proj, self.k_proj = torch.nn.Linear(d, 2 * Hq * D, bias=False), torch.nn.Linear(d, Hkv * D, bias=False)
        self.v_proj, self.o_proj = torch.nn.Linear(d, Hkv * D, bias=False), torch.nn.Linear(Hq * D, d, bias=False)
        for m, (i, o) in ((self.q_proj, (d, 2 * Hq * D)), (self.k_proj, (d, Hkv * D)), (self.v_proj, (d, Hkv * D)),
                          (self.o_proj, (Hq * D, d))):
            m.weight = lin(i, o)
        self.q_norm, self.k_norm = _Norm(D, g), _Norm(D, g)


def _ref_qkv(m, h, cos, sin):
    """fp32 q [B, L, Hq, D], k, v [B, L, Hkv, D], gate [B, L, Hq, D] of the module (the oracle's formulas)."""
    B, L, _ = h.shape
    D = m.head_dim
    f = lambda lin: h.float() @ lin.weight.float().t()
    qg = f(m.q_proj).view(B, L, -1, 2 * D)
    q = oracle.rmsnorm(qg[..., :D], m.q_norm.weight, 1e-6)
    k = oracle.rmsnorm(f(m.k_proj).view(B, L, -1, D), m.k_norm.weight, 1e-6)
    v = f(m.v_proj).view(B, L, -1, D)
    rope = lambda x: torch.stack([oracle.apply_rope(x[b], cos[b], sin[b]) for b in range(B)])
    return rope(q), rope(k), v, qg[..., D:]


def _rope_tables(B, L, R, g, start=0):
    pos = torch.arange(start, start + L)[None].repeat(B, 1) + torch.randint(0, 50, (B, 1), generator=g)
    cs = [oracle.rope_tables(pos[b], R, 10000.0) for b in range(B)]
    return torch.stack([c for c, _ in cs]), torch.stack([s for _, s in cs])


@pytest.mark.parametrize("heads", [(16, 4, 256), (4, 2, 32)])
def test_branch_and_state_attention_with_the_reference_plan(heads):
    """A state level of 3 right-padded rows (level 0, through state_attention with an earlier state chunk), then a
    branch level of 5 padded rows under those 3 states (branch_attention with the reference's kv_valid / slots /
    back plan and head-major states). Every valid query against the oracle's attention over its ancestors' valid
    keys and its own keys causally, gate and o_proj applied."""
    from janus_b200.seams import branch_attention, state_attention
    Hq, Hkv, D = heads
    d, R = 256, D // 4
    g = torch.Generator().manual_seed(32)
    m = _Attn(d, Hq, Hkv, D, g).cuda()
    m_cpu = _Attn(d, Hq, Hkv, D, torch.Generator().manual_seed(32))
    # level 0: an earlier chunk of 40 keys per row, then 60 new tokens (row 2 has 47 valid)
    B0, S0, L0 = 3, 40, 60
    k_prev = torch.randn(B0, Hkv, S0, D, generator=g).to(BF)
    v_prev = torch.randn(B0, Hkv, S0, D, generator=g).to(BF)
    h0 = torch.randn(B0, L0, d, generator=g).to(BF)
    cos0, sin0 = _rope_tables(B0, L0, R, g, start=S0)
    out0, K0, V0 = state_attention(m, h0.cuda(), cos0.cuda(), sin0.cuda(), None, (k_prev.cuda(), v_prev.cuda()))
    assert K0.shape == (B0, Hkv, S0 + L0, D)
    q, k, v, gate = _ref_qkv(m_cpu, h0, cos0, sin0)
    for b in range(B0):
        k_all = torch.cat([k_prev[b].transpose(0, 1).float(), k[b].to(BF).float()])
        v_all = torch.cat([v_prev[b].transpose(0, 1).float(), v[b].to(BF).float()])
        o = oracle.attention(q[b].to(BF).float(), k_all, v_all, S0, m.scaling) * torch.sigmoid(gate[b].to(BF).float())
        ref = o.reshape(L0, -1).to(BF).float() @ m_cpu.o_proj.weight.float().t()
        close(out0[b], ref, atol=3e-2, rtol=3e-2)
        close(K0[b, :, S0:].transpose(0, 1), k[b])
    # level 1: 5 rows under ancestors [0, 0, 1, 2, 2] of level 0 (valid keys: 100, 100, 87)
    valid0 = torch.ones(B0, S0 + L0, dtype=torch.bool)
    valid0[2, S0 + 47:] = False
    anc = [0, 0, 1, 2, 2]
    slots = torch.tensor([[0, 1], [2, 0], [3, 4]])
    back = torch.tensor([0, 1, 2, 4, 5])
    B1, L1 = 5, 12
    valid1 = torch.ones(B1, L1, dtype=torch.bool)
    valid1[3, 9:] = False
    h1 = torch.randn(B1, L1, d, generator=g).to(BF)
    cos1, sin1 = _rope_tables(B1, L1, R, g, start=200)
    plan = (valid0.cuda(), slots.cuda(), back.cuda())
    out1, K1, V1 = branch_attention(m, h1.cuda(), cos1.cuda(), sin1.cuda(), valid1.cuda(), plan, (K0, V0), False, None)
    assert K1.shape == (B1, Hkv, L1, D)
    q, k, v, gate = _ref_qkv(m_cpu, h1, cos1, sin1)
    Kc, Vc = K0.cpu().float(), V0.cpu().float()
    for r in range(B1):
        a = anc[r]
        n = int(valid0[a].sum())
        n_own = int(valid1[r].sum())
        k_all = torch.cat([Kc[a, :, :n].transpose(0, 1), k[r, :n_own].to(BF).float()])
        v_all = torch.cat([Vc[a, :, :n].transpose(0, 1), v[r, :n_own].to(BF).float()])
        o = oracle.attention(q[r, :n_own].to(BF).float(), k_all, v_all, n, m.scaling)
        o = o * torch.sigmoid(gate[r, :n_own].to(BF).float())
        ref = o.reshape(n_own, -1).to(BF).float() @ m_cpu.o_proj.weight.float().t()
        close(out1[r, :n_own], ref, atol=3e-2, rtol=3e-2)


def test_experts_with_the_hf_signature():
    """experts(hidden [S, H], top_k_index [S, k], top_k_weights [S, k]) against the oracle's dequantised experts."""
    from janus_b200 import synthetic
    from janus_b200.seams import W4A16Experts
    E, k, H, I, S = 16, 4, 256, 128, 300
    gu_c, gu_s = synthetic.int4_quantized((E, 2 * I, H), 33, "gu", "cpu")
    dn_c, dn_s = synthetic.int4_quantized((E, H, I), 33, "dn", "cpu")
    g = torch.Generator().manual_seed(33)
    x = torch.randn(S, H, generator=g).to(BF)
    idx = torch.stack([torch.randperm(E, generator=g)[:k] for _ in range(S)])
    w = torch.softmax(torch.randn(S, k, generator=g), -1)
    mod = W4A16Experts(gu_c.cuda(), gu_s.cuda(), dn_c.cuda(), dn_s.cuda())
    out = mod(x.cuda(), idx.cuda(), w.cuda())
    assert out.dtype == BF and out.shape == (S, H)
    gu = oracle.int4_dequantize(gu_c, gu_s).float()
    dn = oracle.int4_dequantize(dn_c, dn_s).float()
    ref = torch.zeros(S, H)
    for s in range(S):
        for j in range(k):
            e = int(idx[s, j])
            hh = x[s].float() @ gu[e].t()
            hh = (torch.nn.functional.silu(hh[:I]) * hh[I:]).to(BF).float()
            ref[s] += ((hh @ dn[e].t()) * w[s, j]).to(BF).float()
    close(out, ref, atol=3e-2, rtol=3e-2)


def test_heads_with_the_module_signatures():
    from janus_b200.seams import PointerHead, ScalarHead
    g = torch.Generator().manual_seed(34)
    H, R, n = 512, 128, 9
    p = {"head.norm.weight": 1 + 0.1 * torch.randn(H, generator=g), "head.norm.bias": 0.1 * torch.randn(H, generator=g),
         "head.out.weight": 0.02 * torch.randn(1, H, generator=g), "head.out.bias": torch.tensor([0.2]),
         "head.query.weight": 0.02 * torch.randn(R, H, generator=g), "head.key.weight": 0.02 * torch.randn(R, H, generator=g)}
    rows = torch.randn(n, H, generator=g) * 2
    dec = torch.randn(H, generator=g)
    sh = ScalarHead(p["head.norm.weight"].cuda(), p["head.norm.bias"].cuda(), 1e-5, p["head.out.weight"].cuda(),
                    p["head.out.bias"].cuda())
    close(sh(rows.cuda().to(BF)), oracle.scalar_head(rows.to(BF).float(), p), atol=2e-4, rtol=2e-4)
    ph = PointerHead(p["head.norm.weight"].cuda(), p["head.norm.bias"].cuda(), 1e-5, p["head.query.weight"].cuda(),
                     p["head.key.weight"].cuda())
    close(ph(dec.cuda(), rows.cuda()), oracle.pointer_head(dec, rows, p), atol=2e-4, rtol=2e-4)
    assert math.isclose(ph.scale, math.sqrt(R))
