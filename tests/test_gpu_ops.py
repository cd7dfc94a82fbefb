"""Each libjanus_b200 op on the GPU against the CPU oracle's fp32 restatement (seeded inputs, small sizes).

bf16 outputs are compared with a tolerance of 2e-2 absolute + 2e-2 relative on O(1) values (one bf16 rounding of
the output plus bf16 operands inside the kernels); fp32 outputs (states, logits) with 2e-3."""

import math

import numpy as np
import pytest
import torch

from oracle import hybrid as oracle

pytestmark = pytest.mark.gpu
BF = torch.bfloat16


def _ops():
    from janus_b200 import ops
    return ops


def close(a, b, atol=2e-2, rtol=2e-2):
    np.testing.assert_allclose(a.detach().float().cpu().numpy(), b.detach().float().cpu().numpy(), atol=atol, rtol=rtol)


def test_embed_and_add_rmsnorm():
    ops = _ops()
    g = torch.Generator().manual_seed(0)
    V, H, T = 50, 2560, 33
    table = (torch.randn(V, H, generator=g)).to(BF)
    ids = torch.randint(0, V, (T,), generator=g, dtype=torch.int32)
    w = (torch.randn(H, generator=g) * 0.1).to(BF)
    x, y = ops.embed_rmsnorm(table.cuda(), ids.cuda(), w.cuda(), 1e-6)
    ref_x = table.float()[ids.long()]
    close(x, ref_x, atol=0, rtol=0)
    close(y, oracle.rmsnorm(ref_x, w, 1e-6))
    delta = torch.randn(T, H, generator=g).to(BF)
    w2 = (torch.randn(H, generator=g) * 0.1).to(BF)
    y2 = ops.add_rmsnorm(x, delta.cuda(), w2.cuda(), 1e-6)
    close(x, ref_x + delta.float(), atol=1e-6, rtol=1e-6)
    close(y2, oracle.rmsnorm(ref_x + delta.float(), w2, 1e-6))
    # a residual 16- but not 32-byte aligned takes the 16-byte accesses; same results bit for bit
    buf = torch.zeros(T * H + 4, device="cuda")
    x16 = buf[4:].view(T, H)
    x16.copy_(ref_x.cuda())
    xw = ref_x.cuda().clone()
    y16 = ops.add_rmsnorm(x16, delta.cuda(), w2.cuda(), 1e-6)
    yw = ops.add_rmsnorm(xw, delta.cuda(), w2.cuda(), 1e-6)
    assert torch.equal(x16, xw) and torch.equal(y16, yw)


def test_silu_mul_and_gated_rmsnorm():
    ops = _ops()
    g = torch.Generator().manual_seed(1)
    gu = torch.randn(17, 2 * 96, generator=g).to(BF)
    out = ops.silu_mul(gu.cuda())
    close(out, torch.nn.functional.silu(gu.float()[:, :96]) * gu.float()[:, 96:])
    # many units per CTA, a ragged last column block (9216 = 4.5 x 2048); I = 104 is not a multiple of 16 and
    # takes the 16-byte kernel, the others the 32-byte one
    for T, I in ((3001, 9216), (700, 2048), (513, 104)):
        gu = torch.randn(T, 2 * I, generator=g).to(BF).cuda()
        out = ops.silu_mul(gu)
        ref = torch.nn.functional.silu(gu.float()[:, :I]) * gu.float()[:, I:]
        close(out, ref)
        assert torch.equal(ops.silu_mul(gu), out)
    for Dv in (32, 128):
        T, Hv = 9, 4
        core = torch.randn(T, Hv, Dv, generator=g).to(BF)
        zbuf = torch.randn(T, Hv * Dv + 40, generator=g).to(BF)
        w = (1 + 0.1 * torch.randn(Dv, generator=g)).to(BF)
        out = ops.gated_rmsnorm(core.cuda(), zbuf.cuda()[:, 8:8 + Hv * Dv], w.cuda(), 1e-6)
        ref = oracle.gated_rmsnorm(core.float(), zbuf.float()[:, 8:8 + Hv * Dv].reshape(T, Hv, Dv), w, 1e-6)
        close(out, ref.reshape(T, -1))
    # 32-byte aligned z (the 32-byte kernel), many units per thread
    for T, Hv, Dv in ((5000, 32, 128), (37, 3, 64)):
        core = torch.randn(T, Hv, Dv, generator=g).to(BF)
        zbuf = torch.randn(T, Hv * Dv + 48, generator=g).to(BF)
        w = (1 + 0.1 * torch.randn(Dv, generator=g)).to(BF)
        out = ops.gated_rmsnorm(core.cuda(), zbuf.cuda()[:, 16:16 + Hv * Dv], w.cuda(), 1e-6)
        ref = oracle.gated_rmsnorm(core.float(), zbuf.float()[:, 16:16 + Hv * Dv].reshape(T, Hv, Dv), w, 1e-6)
        close(out, ref.reshape(T, -1))


def _level(lengths):
    rs = np.concatenate([[0], np.cumsum(lengths)]).astype(np.int32)
    rot = np.repeat(np.arange(len(lengths)), lengths).astype(np.int32)
    return torch.from_numpy(rs), torch.from_numpy(rot)


@pytest.mark.parametrize("dims", [(2, 32, 4, 32), (16, 128, 32, 128)])
def test_gdn_prologue_with_parent_tails(dims):
    ops = _ops()
    Hk, Dk, Hv, Dv = dims
    K = 4
    C = 2 * Hk * Dk + Hv * Dv
    g = torch.Generator().manual_seed(2)
    lengths = [5, 1, 2, 70, 300, 3]  # rows across the 96-token tiles, a last tile of an odd token count
    parent = torch.tensor([1, 0, 1, 2, 0, 2], dtype=torch.int32)
    rs, rot = _level(lengths)
    T = int(rs[-1])
    stride = C + Hv * Dv + 2 * Hv + 8
    proj = torch.randn(T, stride, generator=g).to(BF)
    tails = torch.randn(3, K - 1, C, generator=g).to(BF)
    conv = (torch.randn(C, K, generator=g) * 0.3).to(BF)
    A_log = torch.log(torch.rand(Hv, generator=g) * 16).to(BF)
    dt = torch.ones(Hv).to(BF)
    q, k, v, gg, beta, tail_out = ops.gdn_prologue(proj.cuda(), rs.cuda(), rot.cuda(), parent.cuda(), tails.cuda(), True,
                                                    conv.cuda(), A_log.cuda(), dt.cuda(), Hk, Dk, Hv, Dv)
    for r, L in enumerate(lengths):
        a, b = int(rs[r]), int(rs[r + 1])
        mixed = proj.float()[a:b, :C]
        bb = proj.float()[a:b, C + Hv * Dv:C + Hv * Dv + Hv]
        aa = proj.float()[a:b, C + Hv * Dv + Hv:C + Hv * Dv + 2 * Hv]
        tail = tails.float()[int(parent[r])].t()  # [C, K-1]
        rq, rk, rv, rg, rb, rt = oracle.delta_prologue(mixed, bb, aa, tail, conv.float(), A_log, dt, Hk * Dk, Dk, Dv)
        # one rounding of the fp32 result: within a bf16 unit in the last place (2^-7 relative)
        close(q[a:b], rq, atol=1e-6, rtol=2.0 ** -7)
        close(k[a:b], rk, atol=1e-6, rtol=2.0 ** -7)
        close(v[a:b], rv, atol=1e-6, rtol=2.0 ** -7)
        close(gg[a:b], rg, atol=1e-4, rtol=1e-4)
        close(beta[a:b], rb, atol=1e-5, rtol=1e-5)
        close(tail_out[r].float().t(), rt, atol=0, rtol=0)


@pytest.mark.parametrize("dims", [(2, 32, 4, 32), (16, 128, 32, 128)])
def test_gdn_fork_recurrent_reads_parent_states(dims):
    ops = _ops()
    Hk, Dk, Hv, Dv = dims
    g = torch.Generator().manual_seed(3)
    lengths = [3, 6, 1, 4, 2]
    child_start = torch.tensor([0, 2, 2, 5], dtype=torch.int32)  # parent 0: rows 0-1, parent 1: none, parent 2: rows 2-4
    rs, _ = _level(lengths)
    T = int(rs[-1])
    q = oracle.l2norm(torch.randn(T, Hk, Dk, generator=g)).to(BF)
    k = oracle.l2norm(torch.randn(T, Hk, Dk, generator=g)).to(BF)
    v = torch.randn(T, Hv, Dv, generator=g).to(BF)
    gg = -torch.rand(T, Hv, generator=g) * 0.5
    beta = torch.rand(T, Hv, generator=g)
    S0 = torch.randn(3, Hv, Dk, Dv, generator=g) * 0.2
    scale = 1 / math.sqrt(Dk)
    o, S = ops.gdn_fork_recurrent(q.cuda(), k.cuda(), v.cuda(), gg.cuda(), beta.cuda(), rs.cuda(), child_start.cuda(),
                                  S0.cuda(), True, scale)
    parent_of = [0, 0, 2, 2, 2]
    for r in range(5):
        a, b = int(rs[r]), int(rs[r + 1])
        ro, rS = oracle.delta_recurrent(q[a:b].float(), k[a:b].float(), v[a:b].float(), gg[a:b], beta[a:b], S0[parent_of[r]])
        close(o[a:b], ro)
        close(S[r], rS, atol=2e-4, rtol=2e-4)
    # no parent state: zeros
    o2, _ = ops.gdn_fork_recurrent(q.cuda(), k.cuda(), v.cuda(), gg.cuda(), beta.cuda(), rs.cuda(),
                                   torch.arange(6, dtype=torch.int32).cuda(), None, False, scale)
    ro, _ = oracle.delta_recurrent(q[3:9].float(), k[3:9].float(), v[3:9].float(), gg[3:9], beta[3:9], None)
    close(o2[3:9], ro)


@pytest.mark.parametrize("shape", [(4, 2, 32, 8), (16, 4, 256, 64), (8, 2, 256, 64), (16, 2, 128, 32)])
def test_attn_qk_prep(shape):
    ops = _ops()
    Hq, Hkv, D, rot = shape
    g = torch.Generator().manual_seed(4)
    T = 21
    stride = Hq * 2 * D + 2 * Hkv * D
    qkv = torch.randn(T, stride, generator=g).to(BF)
    pos = torch.randint(0, 9000, (T,), generator=g, dtype=torch.int32)
    qw = (0.1 * torch.randn(D, generator=g)).to(BF)
    kw = (0.1 * torch.randn(D, generator=g)).to(BF)
    inv = 1.0 / (10000.0 ** (torch.arange(0, rot, 2, dtype=torch.int64).float() / rot))
    q, k, v = ops.attn_qk_prep(qkv.cuda(), pos.cuda(), inv.cuda(), qw.cuda(), kw.cuda(), 1e-6, Hq, Hkv, D)
    cos, sin = oracle.rope_tables(pos.long(), rot, 10000.0)
    f = qkv.float()
    rq = oracle.apply_rope(oracle.rmsnorm(f[:, :Hq * 2 * D].view(T, Hq, 2 * D)[..., :D], qw, 1e-6), cos, sin)
    rk = oracle.apply_rope(oracle.rmsnorm(f[:, Hq * 2 * D:Hq * 2 * D + Hkv * D].view(T, Hkv, D), kw, 1e-6), cos, sin)
    close(q, rq)
    close(k, rk)
    close(v, f[:, Hq * 2 * D + Hkv * D:].view(T, Hkv, D), atol=0, rtol=0)


@pytest.mark.parametrize("form", ["pairs", "single"])
@pytest.mark.parametrize("heads", [(4, 2, 32), (16, 4, 256), (8, 2, 256), (16, 2, 256), (4, 4, 128), (8, 8, 256),
                                   (2, 1, 64)])
def test_tree_attention_three_levels(heads, form, monkeypatch):
    """A state level (2 requests), a block level and a leaf level; every query of the leaf level sees its state,
    its block and its own leaf causally (janus/attention.py:10-23 along the path). Head dims 128 and 256 run on
    single CTAs by default and on CTA pairs with JANUS_B200_ATTN=pairs; both are checked."""
    monkeypatch.setenv("JANUS_B200_ATTN", form)
    ops = _ops()
    from janus_b200.plan import build_levels
    from janus_b200 import synthetic
    Hq, Hkv, D = heads
    G = Hq // Hkv
    packs = [synthetic.q4b_request(vocab=4096, seed=s, state_tokens=n, questions=3, block_tokens=9)
             for s, n in ((0, 150), (1, 70))]
    levels, _ = build_levels(packs)
    g = torch.Generator().manual_seed(5)
    K = [torch.randn(lv.T, Hkv, D, generator=g).to(BF) for lv in levels]
    V = [torch.randn(lv.T, Hkv, D, generator=g).to(BF) for lv in levels]
    for d, lv in enumerate(levels):
        T = lv.T
        q = torch.randn(T, Hq, D, generator=g).to(BF)
        gate_buf = torch.randn(T, Hq, 2 * D, generator=g).to(BF)
        gate = gate_buf[:, :, D:]
        cuda = lambda a: torch.from_numpy(np.ascontiguousarray(a)).cuda()
        status = torch.zeros(1, dtype=torch.int32, device="cuda")
        tiles = lv.attention_tiles(ops.tree_attention_tile_tokens(D, Hq, Hkv))
        out = ops.tree_attention(q.cuda(), [k.cuda() for k in K[:d + 1]], [v.cuda() for v in V[:d + 1]],
                                 [cuda(x) for x in lv.anc_lo], [cuda(x) for x in lv.anc_hi], cuda(lv.row_start),
                                 cuda(lv.row_of_token), cuda(tiles), gate_buf.cuda()[:, :, D:], D ** -0.5,
                                 status=status)
        assert int(status.item()) == 0
        out = out.view(T, Hq, D).float().cpu()
        for r in range(lv.B):
            a, b = int(lv.row_start[r]), int(lv.row_start[r + 1])
            pk = [K[l][int(lv.anc_lo[l][r]):int(lv.anc_hi[l][r])] for l in range(d)]
            pv = [V[l][int(lv.anc_lo[l][r]):int(lv.anc_hi[l][r])] for l in range(d)]
            k_all = torch.cat(pk + [K[d][a:b]]).float()
            v_all = torch.cat(pv + [V[d][a:b]]).float()
            ref = oracle.attention(q[a:b].float(), k_all, v_all, k_all.shape[0] - (b - a), D ** -0.5)
            ref = ref * torch.sigmoid(gate[a:b].float())
            close(out[a:b], ref)


@pytest.mark.parametrize("heads", [(16, 4, 256), (8, 8, 128), (16, 2, 128), (4, 4, 256)])
def test_tree_attention_cta_pairs_match_single_ctas(heads, monkeypatch):
    """The CTA-pair form against the single-CTA form on a three-level tree whose state rows have odd tile counts
    (pairs that straddle two requests) and whose branch tiles pair blocks of different questions. A pair walks each
    tile's keys plus blocks fully masked for it, and on the branch levels it may walk the union of two ancestor
    ranges from an earlier first key, which groups the same keys into other blocks (fp32 sums in another order)."""
    ops = _ops()
    from janus_b200.plan import build_levels
    from janus_b200 import synthetic
    Hq, Hkv, D = heads
    packs = [synthetic.q4b_request(vocab=4096, seed=s, state_tokens=n, questions=5, block_tokens=23)
             for s, n in ((10, 1501), (11, 777), (12, 64))]
    levels, _ = build_levels(packs)
    g = torch.Generator().manual_seed(15)
    K = [torch.randn(lv.T, Hkv, D, generator=g).to(BF).cuda() for lv in levels]
    V = [torch.randn(lv.T, Hkv, D, generator=g).to(BF).cuda() for lv in levels]
    cuda = lambda a: torch.from_numpy(np.ascontiguousarray(a)).cuda()
    for d, lv in enumerate(levels):
        q = torch.randn(lv.T, Hq, D, generator=g).to(BF).cuda()
        gate_buf = torch.randn(lv.T, Hq, 2 * D, generator=g).to(BF).cuda()
        tiles = lv.attention_tiles(ops.tree_attention_tile_tokens(D, Hq, Hkv))
        outs = {}
        for form in ("pairs", "single"):
            monkeypatch.setenv("JANUS_B200_ATTN", form)
            status = torch.zeros(1, dtype=torch.int32, device="cuda")
            outs[form] = ops.tree_attention(q, K[:d + 1], V[:d + 1], [cuda(x) for x in lv.anc_lo],
                                            [cuda(x) for x in lv.anc_hi], cuda(lv.row_start), cuda(lv.row_of_token),
                                            cuda(tiles), gate_buf[:, :, D:], D ** -0.5, status=status)
            torch.cuda.synchronize()
            assert int(status.item()) == 0, form
        a, b = outs["pairs"].float(), outs["single"].float()
        diff = (a - b).abs()
        print(f"\nlevel {d}: max |pairs - single| {float(diff.max()):.2e}, equal {float((diff == 0).float().mean()):.4f}")
        close(a, b, atol=1e-2, rtol=1e-2)


def test_heads_match_oracle():
    ops = _ops()
    g = torch.Generator().manual_seed(6)
    T, H, R = 40, 1024, 128
    x = torch.randn(T, H, generator=g) * 3
    fw = (0.1 * torch.randn(H, generator=g)).to(BF)
    lw, lb = 1 + 0.1 * torch.randn(H, generator=g), 0.1 * torch.randn(H, generator=g)
    w_out, b_out = 0.02 * torch.randn(1, H, generator=g), torch.tensor([0.3])
    rows = torch.tensor([3, 7, 39, 0], dtype=torch.int32)
    z = ops.head_scalar(x.cuda(), rows.cuda(), fw.cuda(), 1e-6, lw.cuda(), lb.cuda(), 1e-5, w_out.reshape(-1).cuda(),
                        b_out.cuda())
    hidden = oracle.rmsnorm(x, fw, 1e-6)
    p = {"head.norm.weight": lw, "head.norm.bias": lb, "head.out.weight": w_out, "head.out.bias": b_out}
    close(z, oracle.scalar_head(hidden[rows.long()], p), atol=2e-4, rtol=2e-4)
    wq, wk = 0.02 * torch.randn(R, H, generator=g), 0.02 * torch.randn(R, H, generator=g)
    orows = torch.tensor([1, 2, 3, 10, 11], dtype=torch.int32)
    oq = torch.tensor([0, 0, 0, 1, 1], dtype=torch.int32)
    drows = torch.tensor([5, 12], dtype=torch.int32)
    z = ops.head_pointer(x.cuda(), orows.cuda(), oq.cuda(), drows.cuda(), fw.cuda(), 1e-6, lw.cuda(), lb.cuda(), 1e-5,
                         wq.cuda(), wk.cuda())
    p = {"head.norm.weight": lw, "head.norm.bias": lb, "head.query.weight": wq, "head.key.weight": wk}
    ref = torch.cat([oracle.pointer_head(hidden[5], hidden[[1, 2, 3]], p), oracle.pointer_head(hidden[12], hidden[[10, 11]], p)])
    close(z, ref, atol=2e-4, rtol=2e-4)


def test_bad_arguments_raise_before_launch():
    ops = _ops()
    x = torch.zeros(4, 12, device="cuda")
    with pytest.raises(ValueError):
        ops.add_rmsnorm(x, None, torch.zeros(12, dtype=BF, device="cuda"), 1e-6)  # hidden not a multiple of 8
    with pytest.raises(ValueError):
        ops.silu_mul(torch.zeros(3, 10, dtype=BF, device="cuda"))


def test_gdn_chunk_scan_matches_recurrent_oracle():
    """Rows of 1, 63, 64, 65 and 300 tokens (ragged last chunks), GQA 32:16, an initial state per row read through
    state_row; outputs and final states against the oracle's token-by-token rule."""
    ops = _ops()
    Hk, Hv, D = 16, 32, 128
    g = torch.Generator().manual_seed(7)
    lengths = [1, 63, 64, 65, 300]
    rs, _ = _level(lengths)
    T = int(rs[-1])
    q = oracle.l2norm(torch.randn(T, Hk, D, generator=g)).to(BF)
    k = oracle.l2norm(torch.randn(T, Hk, D, generator=g)).to(BF)
    v = torch.randn(T, Hv, D, generator=g).to(BF)
    A = torch.rand(Hv, generator=g) * 8
    gg = -A * torch.nn.functional.softplus(torch.randn(T, Hv, generator=g) + 1.0) * 0.1
    beta = torch.sigmoid(torch.randn(T, Hv, generator=g))
    S0 = torch.randn(2, Hv, D, D, generator=g) * 0.1
    state_row = torch.tensor([1, 0, 1, 1, 0], dtype=torch.int32)
    scale = D ** -0.5
    cs = torch.from_numpy(np.concatenate([[0], np.cumsum([(n + 63) // 64 for n in lengths])]).astype(np.int32))
    nc = int(cs[-1])
    status = torch.zeros(1, dtype=torch.int32, device="cuda")
    o, S = ops.gdn_chunk_scan(q.cuda(), k.cuda(), v.cuda(), gg.cuda(), beta.cuda(), rs.cuda(), cs.cuda(), nc,
                              S0.cuda(), state_row.cuda(), True, scale, status=status)
    assert int(status.item()) == 0
    for r in range(len(lengths)):
        a, b = int(rs[r]), int(rs[r + 1])
        ro, rS = oracle.delta_recurrent(q[a:b].float(), k[a:b].float(), v[a:b].float(), gg[a:b], beta[a:b],
                                        S0[int(state_row[r])])
        close(o[a:b], ro, atol=3e-2, rtol=3e-2)
        close(S[r], rS, atol=3e-2, rtol=3e-2)
    o2, _ = ops.gdn_chunk_scan(q.cuda(), k.cuda(), v.cuda(), gg.cuda(), beta.cuda(), rs.cuda(), cs.cuda(), nc, None,
                               None, False, scale)
    a, b = int(rs[4]), int(rs[5])
    ro, _ = oracle.delta_chunked(q[a:b].float(), k[a:b].float(), v[a:b].float(), gg[a:b], beta[a:b], None)
    close(o2[a:b], ro, atol=3e-2, rtol=3e-2)


def test_gdn_chunk_scan_one_launch_equals_two_launch():
    """The one-launch chunk scan (prep of chunk c+1 under the state pass of chunk c, hand-over in shared memory) and
    the two-launch form (prep into an HBM workspace, then the state pass) compute the same products with the same
    roundings: outputs and kept states bit-identical. Rows of 0, 1, 63, 64, 65, 129, 300 and 2000 tokens, initial
    states through state_row, fast- and slow-forgetting heads; then the same without initial states."""
    ops = _ops()
    Hk, Hv, D = 16, 32, 128
    g = torch.Generator().manual_seed(17)
    lengths = [0, 1, 63, 64, 65, 129, 300, 2000, 0, 77]
    rs = torch.tensor(np.concatenate([[0], np.cumsum(lengths)]).astype(np.int32))
    T = int(rs[-1])
    q = oracle.l2norm(torch.randn(T, Hk, D, generator=g)).to(BF).cuda()
    k = oracle.l2norm(torch.randn(T, Hk, D, generator=g)).to(BF).cuda()
    v = torch.randn(T, Hv, D, generator=g).to(BF).cuda()
    A = torch.exp(torch.linspace(np.log(1e-3), np.log(16.0), Hv))
    gg = (-A * torch.nn.functional.softplus(torch.randn(T, Hv, generator=g) + 1.0)).cuda()
    beta = torch.sigmoid(torch.randn(T, Hv, generator=g)).cuda()
    S0 = (torch.randn(3, Hv, D, D, generator=g) * 0.1).cuda()
    state_row = torch.tensor([2, 1, 0, 1, 2, 0, 1, 2, 0, 1], dtype=torch.int32).cuda()
    cs = torch.tensor(np.concatenate([[0], np.cumsum([(n + 63) // 64 for n in lengths])]).astype(np.int32)).cuda()
    nc = int(cs[-1].item())
    for s_in, s_row in ((S0, state_row), (None, None)):
        status = torch.zeros(1, dtype=torch.int32, device="cuda")
        o1, S1 = ops.gdn_chunk_scan(q, k, v, gg, beta, rs.cuda(), cs, nc, s_in, s_row, True, D ** -0.5,
                                    status=status, fused=True)
        o2, S2 = ops.gdn_chunk_scan(q, k, v, gg, beta, rs.cuda(), cs, nc, s_in, s_row, True, D ** -0.5,
                                    status=status, fused=False)
        torch.cuda.synchronize()
        assert int(status.item()) == 0
        assert torch.equal(o1, o2), float((o1.float() - o2.float()).abs().max())
        assert torch.equal(S1, S2), float((S1 - S2).abs().max())
        for r, n in enumerate(lengths):  # empty rows keep their initial state
            if n == 0:
                assert torch.equal(S1[r], s_in[int(s_row[r])] if s_in is not None else torch.zeros_like(S1[r]))


def test_device_wait_that_runs_out_is_reported_and_the_context_survives():
    """The bounded mbarrier wait of the tcgen05 kernels: a phase nothing completes ends in status 1 after ~1 s,
    not in a hang or a fault, and the next launch on the same context works."""
    import time
    from janus_b200 import ops
    t0 = time.perf_counter()
    assert ops.selftest_wait_timeout() == 1
    assert time.perf_counter() - t0 < 30
    x = torch.randn(4, 128, device="cuda")
    y = ops.silu_mul(torch.randn(4, 256, device="cuda").to(torch.bfloat16))
    torch.cuda.synchronize()
    assert torch.isfinite(y.float()).all() and torch.isfinite(x).all()


def test_tcgen05_kernels_run_to_run_identical():
    """Tree attention and the chunk scan on many CTAs at once: repeated launches agree bit for bit (their
    accumulation orders are fixed, so any difference is a race between pipeline stages)."""
    ops = _ops()
    from janus_b200.plan import build_levels
    from janus_b200 import synthetic
    g = torch.Generator().manual_seed(11)
    packs = [synthetic.q4b_request(vocab=4096, seed=s, state_tokens=1500 + 300 * s, questions=4, block_tokens=16)
             for s in range(4)]
    levels, _ = build_levels(packs)
    Hq, Hkv, D = 16, 4, 256
    K = [torch.randn(lv.T, Hkv, D, generator=g).to(BF).cuda() for lv in levels]
    V = [torch.randn(lv.T, Hkv, D, generator=g).to(BF).cuda() for lv in levels]
    cuda = lambda a: torch.from_numpy(np.ascontiguousarray(a)).cuda()
    for d, lv in enumerate(levels):
        q = torch.randn(lv.T, Hq, D, generator=g).to(BF).cuda()
        gate_buf = torch.randn(lv.T, Hq, 2 * D, generator=g).to(BF).cuda()
        tiles = cuda(lv.attention_tiles(ops.tree_attention_tile_tokens(D, Hq, Hkv)))
        args = (q, K[:d + 1], V[:d + 1], [cuda(x) for x in lv.anc_lo], [cuda(x) for x in lv.anc_hi],
                cuda(lv.row_start), cuda(lv.row_of_token), tiles, gate_buf[:, :, D:], D ** -0.5)
        status = torch.zeros(1, dtype=torch.int32, device="cuda")
        first = ops.tree_attention(*args, status=status).clone()
        for _ in range(4):
            assert torch.equal(ops.tree_attention(*args, status=status), first)
        assert int(status.item()) == 0
    Hk, Hv, Dk = 16, 32, 128
    lengths = [700 + 37 * i for i in range(24)]
    rs, _ = _level(lengths)
    T = int(rs[-1])
    qq = oracle.l2norm(torch.randn(T, Hk, Dk, generator=g)).to(BF).cuda()
    kk = oracle.l2norm(torch.randn(T, Hk, Dk, generator=g)).to(BF).cuda()
    vv = torch.randn(T, Hv, Dk, generator=g).to(BF).cuda()
    gg = (-torch.rand(T, Hv, generator=g) * 0.2).cuda()
    beta = torch.sigmoid(torch.randn(T, Hv, generator=g)).cuda()
    cs = torch.from_numpy(np.concatenate([[0], np.cumsum([(n + 63) // 64 for n in lengths])]).astype(np.int32))
    nc = int(cs[-1])
    status = torch.zeros(1, dtype=torch.int32, device="cuda")
    o0, S0 = ops.gdn_chunk_scan(qq, kk, vv, gg, beta, rs.cuda(), cs.cuda(), nc, None, None, True, Dk ** -0.5,
                                status=status)
    o0, S0 = o0.clone(), S0.clone()
    for _ in range(4):
        o, S = ops.gdn_chunk_scan(qq, kk, vv, gg, beta, rs.cuda(), cs.cuda(), nc, None, None, True, Dk ** -0.5,
                                  status=status)
        assert torch.equal(o, o0) and torch.equal(S, S0)
    assert int(status.item()) == 0


def test_segmented_chunk_scan_is_the_state_fork():
    """Sibling rows packed into 64-token runs (the segmented chunk scan) equal the fork: every child row runs the
    token-by-token rule from its parent's state (oracle), rows of 1..20 tokens, several runs per parent."""
    ops = _ops()
    from janus_b200.plan import Level
    Hk, Hv, D = 16, 32, 128
    g = torch.Generator().manual_seed(21)
    rng = np.random.default_rng(21)
    children = [list(rng.integers(1, 21, size=n)) for n in (1, 7, 12, 3)]  # per parent: child row lengths
    lengths = [int(x) for c in children for x in c]
    child_start = np.concatenate([[0], np.cumsum([len(c) for c in children])]).astype(np.int32)
    parent = np.repeat(np.arange(len(children)), [len(c) for c in children]).astype(np.int32)
    rs, rot = _level(lengths)
    T = int(rs[-1])
    lv = Level(1, np.zeros(T, np.int32), np.zeros(T, np.int32), rs.numpy(), rot.numpy(), parent, [], [], child_start,
               np.zeros(len(lengths) + 1, np.int32), [])
    starts, parents = lv.fork_chunks()
    q = oracle.l2norm(torch.randn(T, Hk, D, generator=g)).to(BF)
    k = oracle.l2norm(torch.randn(T, Hk, D, generator=g)).to(BF)
    v = torch.randn(T, Hv, D, generator=g).to(BF)
    gg = -torch.rand(T, Hv, generator=g) * 0.5
    beta = torch.sigmoid(torch.randn(T, Hv, generator=g))
    S0 = torch.randn(len(children), Hv, D, D, generator=g) * 0.1
    status = torch.zeros(1, dtype=torch.int32, device="cuda")
    n = int(parents.shape[0])
    cuda = lambda a: torch.from_numpy(np.ascontiguousarray(a)).cuda()
    o, S = ops.gdn_chunk_scan(q.cuda(), k.cuda(), v.cuda(), gg.cuda(), beta.cuda(), cuda(starts),
                              cuda(np.arange(n + 1, dtype=np.int32)), n, S0.cuda(), cuda(parents), False, D ** -0.5,
                              status=status, segment=rot.cuda())
    assert S is None and int(status.item()) == 0
    for r in range(len(lengths)):
        a, b = int(rs[r]), int(rs[r + 1])
        ro, _ = oracle.delta_recurrent(q[a:b].float(), k[a:b].float(), v[a:b].float(), gg[a:b], beta[a:b],
                                       S0[int(parent[r])])
        close(o[a:b], ro, atol=3e-2, rtol=3e-2)
