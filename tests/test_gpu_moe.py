"""The MoE path (routing plan, W4A16 grouped GEMMs, combine) against fp32 restatements on seeded inputs."""

import numpy as np
import pytest
import torch
import torch.nn.functional as F

from oracle import hybrid as oracle

pytestmark = pytest.mark.gpu
BF = torch.bfloat16


def _ops():
    from janus_b200 import ops
    return ops


def _experts(E, NW, K, seed):
    from janus_b200.synthetic import int4_quantized
    codes, scales = int4_quantized((E, NW, K), seed, "experts", "cpu")
    return codes, scales


@pytest.mark.parametrize("S,E,k", [(1, 8, 2), (37, 8, 2), (300, 32, 8), (1000, 256, 8)])
def test_route_topk_and_plan(S, E, k):
    ops = _ops()
    g = torch.Generator().manual_seed(S)
    logits = torch.randn(S, E, generator=g) * 2
    idx, w, sorted_ids, tile_expert, n_tiles = ops.moe_route(logits.cuda(), k)
    probs = torch.softmax(logits, -1)
    top, ref_idx = torch.topk(probs, k, dim=-1)
    np.testing.assert_array_equal(idx.cpu().numpy(), ref_idx.numpy())
    np.testing.assert_allclose(w.cpu().numpy(), (top / top.sum(-1, keepdim=True)).numpy(), atol=1e-6, rtol=1e-5)
    n = int(n_tiles.item())
    T = ops.MOE_TILE
    ids = sorted_ids.cpu().numpy()[: n * T]
    te = tile_expert.cpu().numpy()[:n]
    live = ids[ids >= 0]
    assert sorted(live.tolist()) == list(range(S * k))  # every assignment exactly once
    flat = idx.cpu().numpy().reshape(-1)
    for t in range(n):  # every row of a tile belongs to the tile's expert
        rows = ids[t * T:(t + 1) * T]
        assert (flat[rows[rows >= 0]] == te[t]).all()
    counts = np.bincount(flat, minlength=E)
    assert n == sum((c + T - 1) // T for c in counts)


@pytest.mark.parametrize("S,E,k,H", [(1, 8, 2, 128), (37, 8, 2, 128), (300, 256, 8, 2048), (1000, 256, 8, 2048),
                                     (130, 40, 4, 256)])
def test_fused_router_matches_router_gemm_and_route(S, E, k, H):
    """The router GEMM fused with the routing against the fp32 logits x W_r^T fed to moe_route (the same top-k
    arithmetic): the same experts wherever the logits do not tie at the k-th place within fp32 rounding, the same
    weights for those, the shared gate logit to fp32 rounding, and a consistent tile plan."""
    ops = _ops()
    g = torch.Generator().manual_seed(S + E)
    x = torch.randn(S, H, generator=g).to(BF)
    wr = (0.05 * torch.randn(E, H, generator=g)).to(BF)
    wg = (0.05 * torch.randn(1, H, generator=g)).to(BF)
    status = torch.zeros(1, dtype=torch.int32, device="cuda")
    (idx, w, sorted_ids, tile_expert, n_tiles), gate = ops.moe_route_fused(x.cuda(), wr.cuda(), k, w_gate=wg.cuda(),
                                                                          status=status)
    logits = x.double() @ wr.double().t()
    ref_idx, ref_w, *_ = ops.moe_route(logits.float().cuda(), k)
    torch.cuda.synchronize()
    assert int(status.item()) == 0
    idx, ref_idx = idx.cpu(), ref_idx.cpu()
    same = (idx == ref_idx).all(1)
    assert float(same.float().mean()) >= 0.995, float(same.float().mean())
    np.testing.assert_allclose(w.cpu()[same].numpy(), ref_w.cpu()[same].numpy(), atol=2e-6, rtol=2e-5)
    np.testing.assert_allclose(gate.cpu().numpy(), (x.double() @ wg.double().t()).reshape(-1).numpy(),
                               atol=1e-5, rtol=1e-5)
    n = int(n_tiles.item())
    T = ops.MOE_TILE
    ids = sorted_ids.cpu().numpy()[: n * T]
    te = tile_expert.cpu().numpy()[:n]
    assert sorted(ids[ids >= 0].tolist()) == list(range(S * k))
    flat = idx.numpy().reshape(-1)
    for t in range(n):
        rows = ids[t * T:(t + 1) * T]
        assert (flat[rows[rows >= 0]] == te[t]).all()


@pytest.mark.parametrize("S,E,k,H,I", [(5, 8, 2, 128, 128), (700, 16, 4, 2048, 512), (300, 256, 8, 2048, 512)])
def test_grouped_w4a16_gemms_and_combine(S, E, k, H, I):
    ops = _ops()
    g = torch.Generator().manual_seed(H + S)
    x = (torch.randn(S, H, generator=g)).to(torch.bfloat16)
    logits = torch.randn(S, E, generator=g)
    logits[:, 0] += 3.0  # skewed routing: expert 0 takes most tokens
    gu_codes, gu_scales = _experts(E, 2 * I, H, 11)
    dn_codes, dn_scales = _experts(E, H, I, 12)
    plan = ops.moe_route(logits.cuda(), k)
    h = ops.moe_grouped_w4a16(x.cuda(), gu_codes.cuda(), gu_scales.cuda(), plan, True, k)
    y2 = ops.moe_grouped_w4a16(h, dn_codes.cuda(), dn_scales.cuda(), plan, False, k, topk_w=plan[1])
    shared = torch.randn(S, H, generator=g).to(torch.bfloat16)
    sg = torch.randn(S, generator=g)
    out = ops.moe_combine(y2, k, shared.cuda(), sg.cuda())
    torch.cuda.synchronize()
    # reference: dequantised experts, fp32 math on the same routing
    gu = oracle.int4_dequantize(gu_codes, gu_scales).float()
    dn = oracle.int4_dequantize(dn_codes, dn_scales).float()
    idx = plan[0].cpu().long()
    wts = plan[1].cpu()
    ref = torch.zeros(S, H)
    xf = x.float()
    for t in range(S):
        for j in range(k):
            e = int(idx[t, j])
            hh = xf[t] @ gu[e].t()
            hh = (F.silu(hh[:I]) * hh[I:]).to(torch.bfloat16).float()  # the kernel stores h in bf16
            ref[t] += wts[t, j] * (hh @ dn[e].t())
    ref += torch.sigmoid(sg)[:, None] * shared.float()
    scale = ref.abs().max().item()
    np.testing.assert_allclose(out.float().cpu().numpy(), ref.numpy(), atol=2e-2 * scale, rtol=2e-2)


@pytest.mark.parametrize("S,E,k,W", [(5, 8, 2, 2), (300, 32, 8, 4), (256, 256, 8, 8)])
def test_expert_parallel_kernels_emulated_on_one_gpu(S, E, k, W):
    """moe_plan / moe_reduce_slots / moe_combine_ep as W ranks would run them (every token sent to every rank,
    each rank holding E/W experts), on one GPU: equal to the single-device route + GEMMs + combine."""
    ops = _ops()
    H, I = 256, 128
    g = torch.Generator().manual_seed(S + W)
    x = torch.randn(S, H, generator=g).to(torch.bfloat16).cuda()
    logits = torch.randn(S, E, generator=g).cuda()
    gu_codes, gu_scales = (t.cuda() for t in _experts(E, 2 * I, H, 21))
    dn_codes, dn_scales = (t.cuda() for t in _experts(E, H, I, 22))
    shared = torch.randn(S, H, generator=g).to(torch.bfloat16).cuda()
    sg = torch.randn(S, generator=g).cuda()
    plan = ops.moe_route(logits, k)
    y2 = ops.moe_grouped_w4a16(ops.moe_grouped_w4a16(x, gu_codes, gu_scales, plan, True, k), dn_codes, dn_scales,
                               plan, False, k, topk_w=plan[1])
    ref = ops.moe_combine(y2, k, shared, sg)
    idx, wts = plan[0], plan[1]
    L = E // W
    parts = []
    for r in range(W):
        local = idx - r * L
        slot_e = torch.where((local >= 0) & (local < L), local, torch.full_like(local, -1)).to(torch.int32)
        rp = ops.moe_plan(slot_e.contiguous(), L)
        sl = slice(r * L, (r + 1) * L)
        hh = ops.moe_grouped_w4a16(x, gu_codes[sl].contiguous(), gu_scales[sl].contiguous(), rp, True, k)
        yy = ops.moe_grouped_w4a16(hh, dn_codes[sl].contiguous(), dn_scales[sl].contiguous(), rp, False, k,
                                   topk_w=wts.reshape(-1))
        parts.append(ops.moe_reduce_slots(yy, k, slot_e))
    partials = torch.cat(parts)
    row_index = (torch.arange(S, device="cuda")[:, None] + S * torch.arange(W, device="cuda")[None, :]).to(torch.int32)
    got = ops.moe_combine_ep(partials, row_index.contiguous(), shared, sg)
    torch.cuda.synchronize()
    # the same bf16 expert rows summed in another fp32 order: equal up to the final bf16 rounding
    np.testing.assert_allclose(got.float().cpu().numpy(), ref.float().cpu().numpy(), atol=2e-2, rtol=1e-2)
    # plan of explicit ids: every slot with an expert exactly once, -1 slots never
    n = int(rp[4].item())
    ids = rp[2].cpu().numpy()[: n * ops.MOE_TILE]
    live = np.sort(ids[ids >= 0])
    expect = np.nonzero(slot_e.cpu().numpy().reshape(-1) >= 0)[0]
    np.testing.assert_array_equal(live, expect)


@pytest.mark.parametrize("S,E,k", [(300, 256, 8), (4096, 64, 8)])
def test_grouped_w4a16_run_to_run_identical(S, E, k):
    """The grouped GEMMs accumulate in a fixed order, so repeated launches must agree bit for bit; a difference is a
    race between the pipeline stages (a tolerance check alone can miss one that corrupts a few tiles)."""
    ops = _ops()
    H, I = 2048, 512
    g = torch.Generator().manual_seed(S + E)
    x = torch.randn(S, H, generator=g).to(torch.bfloat16).cuda()
    logits = torch.randn(S, E, generator=g).cuda()
    gu_codes, gu_scales = (t.cuda() for t in _experts(E, 2 * I, H, 31))
    dn_codes, dn_scales = (t.cuda() for t in _experts(E, H, I, 32))
    plan = ops.moe_route(logits, k)
    st = torch.zeros(1, dtype=torch.int32, device="cuda")
    valid = plan[2] >= 0
    h0 = ops.moe_grouped_w4a16(x, gu_codes, gu_scales, plan, True, k, status=st)
    y0 = ops.moe_grouped_w4a16(h0, dn_codes, dn_scales, plan, False, k, topk_w=plan[1], status=st)
    for _ in range(6):
        h = ops.moe_grouped_w4a16(x, gu_codes, gu_scales, plan, True, k, status=st)
        y = ops.moe_grouped_w4a16(h0, dn_codes, dn_scales, plan, False, k, topk_w=plan[1], status=st)
        assert torch.equal(h[valid], h0[valid])
        assert torch.equal(y, y0)
    assert int(st.item()) == 0


@pytest.mark.parametrize("fmt", ["int4", "nvfp4"])
def test_decoded_weights_are_the_reference_values_bit_for_bit(fmt):
    """The down GEMM of one expert on identity rows returns the decoded weight matrix itself (1 x w accumulated in
    fp32 and rounded to bf16 is w): every decoded element equals the oracle's dequantised bf16 weight."""
    from janus_b200 import synthetic
    ops = _ops()
    E, H, I = 3, 256, 512
    if fmt == "int4":
        codes, scales = synthetic.int4_quantized((E, H, I), 21, "dn", "cpu")
        ref = oracle.int4_dequantize(codes, scales)
    else:
        codes, bs, gl = synthetic.nvfp4_quantized((E, H, I), 21, "dn", "cpu")
        ref = oracle.nvfp4_dequantize(codes, bs, gl)
    e = 2
    slot = torch.full((I, 1), e, dtype=torch.int32)
    plan = ops.moe_plan(slot.cuda(), E)
    # the down GEMM reads sorted row r and writes assignment ids[r]: put e_a in the sorted row of assignment a
    ids = plan[2].cpu().long()
    pos = torch.nonzero(ids >= 0).reshape(-1)
    assert sorted(ids[pos].tolist()) == list(range(I))
    x = torch.zeros(ids.shape[0], I, dtype=torch.bfloat16)
    x[pos, ids[pos]] = 1.0
    x = x.cuda()
    w1 = torch.ones(I, dtype=torch.float32).cuda()
    if fmt == "int4":
        out = ops.moe_grouped_w4a16(x, codes.cuda(), scales.cuda(), plan, False, 1, topk_w=w1)
    else:
        out = ops.moe_grouped_nvfp4(x, codes.cuda(), bs.cuda(), gl.cuda(), plan, False, 1, topk_w=w1)
    np.testing.assert_array_equal(out.cpu().float().numpy(), ref[e].t().float().numpy())


def test_grouped_nvfp4_gemms_and_combine():
    """The A3B expert shapes in the reference's NVFP4 format (gate and up with their own global scales): both grouped
    GEMMs and the combine against fp32 math on the oracle's dequantised weights."""
    from janus_b200 import synthetic
    ops = _ops()
    S, E, k, H, I = 400, 64, 8, 2048, 512
    g = torch.Generator().manual_seed(9)
    x = torch.randn(S, H, generator=g).to(torch.bfloat16)
    logits = torch.randn(S, E, generator=g)
    gu = synthetic.nvfp4_quantized((E, 2 * I, H), 31, "gu", "cpu", halves=True)
    dn = synthetic.nvfp4_quantized((E, H, I), 32, "dn", "cpu")
    plan = ops.moe_route(logits.cuda(), k)
    h = ops.moe_grouped_nvfp4(x.cuda(), *(t.cuda() for t in gu), plan, True, k)
    y2 = ops.moe_grouped_nvfp4(h, *(t.cuda() for t in dn), plan, False, k, topk_w=plan[1])
    out = ops.moe_combine(y2, k, None, None)
    torch.cuda.synchronize()
    guw = oracle.nvfp4_dequantize(*gu).float()
    dnw = oracle.nvfp4_dequantize(*dn).float()
    idx, wts = plan[0].cpu().long(), plan[1].cpu()
    ref = torch.zeros(S, H)
    for t in range(S):
        for j in range(k):
            e = int(idx[t, j])
            hh = x[t].float() @ guw[e].t()
            hh = (F.silu(hh[:I]) * hh[I:]).to(torch.bfloat16).float()
            ref[t] += (wts[t, j] * (hh @ dnw[e].t())).to(torch.bfloat16).float()
    scale = ref.abs().max().item()
    np.testing.assert_allclose(out.float().cpu().numpy(), ref.numpy(), atol=1e-2 * scale, rtol=2e-2)


def test_nvfp4_experts_in_the_readout():
    """A tiny MoE readout whose experts are in the reference's NVFP4 format, against the oracle at the B200 path's
    storage precision (the same weights dequantised)."""
    from janus_b200 import synthetic
    from janus_b200.config import SHAPES
    from janus_b200.model import DecisionReadout
    shape = SHAPES["tiny-moe"]
    weights = synthetic.make_weights(shape, seed=8, head="scalar", experts="nvfp4")
    packs = [synthetic.tiny_request(vocab=shape.vocab, seed=s, mode="tree") for s in (3, 4)]
    got = DecisionReadout(shape, weights, "tree").probabilities(packs)
    model16 = oracle.Oracle(shape, weights, storage="bf16")
    worst = 0.0
    for pack, per in zip(packs, got):
        for a, b in zip(per, oracle.probabilities(model16.logits(pack, "tree"))):
            worst = max(worst, float((a - b).abs().max()))
    print(f"\nNVFP4 tiny MoE readout: max |p - p_oracle_bf16| {worst:.2e}")
    assert worst <= 5e-3
