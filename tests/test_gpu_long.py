"""The two heavy ops at the headline length (8192-token states) against the CPU oracle's fp32 restatement.

The short op tests (tests/test_gpu_ops.py) cover the edge cases; these cover what only a long row shows: error that
builds up in the chunk scan's fp32 state over 128 chunks (the state is carried in fp32, but each chunk's products
read a bf16 copy of it), and the softmax of an attention row over 8192 keys (level 0 causally, and a block level
whose rows see the whole state). Inputs follow the model's value ranges: l2-normalised q/k, g = -A softplus(a + 1)
with A spread over [0.001, 16] (some heads keep their state over the whole row, others forget within a few tokens),
beta = sigmoid(b). Every test prints the max and RMS error next to the scale of the compared values.
"""

import numpy as np
import pytest
import torch

from oracle import hybrid as oracle

pytestmark = pytest.mark.gpu
BF = torch.bfloat16


def _stats(got, ref):
    got, ref = got.detach().float().cpu(), ref.detach().float().cpu()
    err = (got - ref).abs()
    return float(err.max()), float(err.pow(2).mean().sqrt()), float(ref.pow(2).mean().sqrt())


def test_chunk_scan_over_8192_token_rows():
    from janus_b200 import ops
    Hk, Hv, D = 16, 32, 128
    lengths = [8192, 8192 - 37]
    g = torch.Generator().manual_seed(81)
    rs = torch.tensor(np.concatenate([[0], np.cumsum(lengths)]).astype(np.int32))
    T = int(rs[-1])
    q = oracle.l2norm(torch.randn(T, Hk, D, generator=g)).to(BF)
    k = oracle.l2norm(torch.randn(T, Hk, D, generator=g)).to(BF)
    v = torch.randn(T, Hv, D, generator=g).to(BF)
    A = torch.exp(torch.linspace(np.log(1e-3), np.log(16.0), Hv))  # per head, slow to fast decay
    gg = -A * torch.nn.functional.softplus(torch.randn(T, Hv, generator=g) * 0.5 + 1.0)
    beta = torch.sigmoid(torch.randn(T, Hv, generator=g))
    cs = torch.tensor(np.concatenate([[0], np.cumsum([(n + 63) // 64 for n in lengths])]).astype(np.int32))
    status = torch.zeros(1, dtype=torch.int32, device="cuda")
    o, S = ops.gdn_chunk_scan(q.cuda(), k.cuda(), v.cuda(), gg.cuda(), beta.cuda(), rs.cuda(), cs.cuda(), int(cs[-1]),
                              None, None, True, D ** -0.5, status=status)
    assert int(status.item()) == 0
    for r in range(len(lengths)):
        a, b = int(rs[r]), int(rs[r + 1])
        ro, rS = oracle.delta_chunked(q[a:b].float(), k[a:b].float(), v[a:b].float(), gg[a:b], beta[a:b], None)
        om, orms, oscale = _stats(o[a:b], ro)
        sm, srms, sscale = _stats(S[r], rS)
        # the last 64 tokens see the state after the longest carry
        tm, trms, _ = _stats(o[b - 64:b], ro[-64:])
        print(f"\nrow {r} ({b - a} tokens): o max {om:.2e} rms {orms:.2e} (rms of o {oscale:.2e}); last chunk max {tm:.2e} "
              f"rms {trms:.2e}; final state max {sm:.2e} rms {srms:.2e} (rms of S {sscale:.2e})")
        # bf16 output rounding is 2^-9 relative; the kernel's bf16 state operands add the same order per chunk
        assert orms <= 1e-2 * oscale and om <= 3e-2 * max(1.0, float(ro.abs().max()))
        assert trms <= 1e-2 * oscale
        assert srms <= 1e-2 * sscale and sm <= 2e-2 * max(1.0, float(rS.abs().max()))


def _attention_ref(q, k_all, v_all, n_prefix, gate, D):
    ref = oracle.attention(q.float(), k_all.float(), v_all.float(), n_prefix, D ** -0.5)
    return ref * torch.sigmoid(gate.float())


def test_tree_attention_over_8192_key_states():
    """Level 0: one 8192-token state causally (queries near the end see ~8k keys); level 1: 8 blocks of 32 tokens
    that each see the 8192 state keys plus their own keys causally. 4B attention heads (16 q, 4 kv, dim 256)."""
    from janus_b200 import ops, synthetic
    from janus_b200.plan import build_levels
    Hq, Hkv, D = 16, 4, 256
    pack = synthetic.q4b_request(vocab=4096, seed=82, state_tokens=8192, questions=8, block_tokens=32)
    levels, _ = build_levels([pack])
    g = torch.Generator().manual_seed(82)
    K = [oracle.l2norm(torch.randn(lv.T, Hkv, D, generator=g)).mul(16.0).to(BF) for lv in levels[:2]]
    V = [torch.randn(lv.T, Hkv, D, generator=g).to(BF) for lv in levels[:2]]
    cuda = lambda a: torch.from_numpy(np.ascontiguousarray(a)).cuda()
    for d, lv in enumerate(levels[:2]):
        T = lv.T
        # queries of norm 16 like the keys: scores up to 256 / 16 = 16 (sharp rows next to flat ones)
        q = oracle.l2norm(torch.randn(T, Hq, D, generator=g)).mul(16.0).to(BF)
        gate_buf = torch.randn(T, Hq, 2 * D, generator=g).to(BF)
        status = torch.zeros(1, dtype=torch.int32, device="cuda")
        tiles = lv.attention_tiles(ops.tree_attention_tile_tokens(D, Hq, Hkv))
        out = ops.tree_attention(q.cuda(), [x.cuda() for x in K[:d + 1]], [x.cuda() for x in V[:d + 1]],
                                 [cuda(x) for x in lv.anc_lo], [cuda(x) for x in lv.anc_hi], cuda(lv.row_start),
                                 cuda(lv.row_of_token), cuda(tiles), gate_buf.cuda()[:, :, D:], D ** -0.5,
                                 status=status)
        assert int(status.item()) == 0
        out = out.view(T, Hq, D).float().cpu()
        gate = gate_buf[:, :, D:]
        if d == 0:
            # the last 512 queries of the state (8k visible keys each) and the first 64
            for a, b in ((T - 512, T), (0, 64)):
                ref = _attention_ref(q[a:b], K[0][:b], V[0][:b], a, gate[a:b], D)
                m, rms, scale = _stats(out[a:b], ref)
                print(f"\nlevel 0 queries {a}..{b}: max {m:.2e} rms {rms:.2e} (rms of o {scale:.2e})")
                assert m <= 2e-2 and rms <= 1e-2 * max(scale, 1e-3) + 1e-4
        else:
            worst = 0.0
            for r in range(lv.B):
                a, b = int(lv.row_start[r]), int(lv.row_start[r + 1])
                lo, hi = int(lv.anc_lo[0][r]), int(lv.anc_hi[0][r])
                k_all = torch.cat([K[0][lo:hi], K[1][a:b]])
                v_all = torch.cat([V[0][lo:hi], V[1][a:b]])
                ref = _attention_ref(q[a:b], k_all, v_all, hi - lo, gate[a:b], D)
                m, rms, scale = _stats(out[a:b], ref)
                worst = max(worst, m)
                assert m <= 2e-2 and rms <= 1e-2 * max(scale, 1e-3) + 1e-4
            print(f"\nlevel 1 ({lv.B} blocks over 8192 state keys): max {worst:.2e}")
