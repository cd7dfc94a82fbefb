"""Expert-parallel dispatch / combine (janus_b200/ep.py) on CPU: world-size-2 gloo ranks.

Each rank routes its own tokens, holds half of the experts, runs its received rows through its experts (a dense
fp32 restatement of the W4A16 experts stands in for the CUDA grouped GEMMs, which need a GPU) and combines; the
result must equal the single-process MoE block of the oracle on the same tokens with all experts. The failure
cases make a rank leave before its collective and check that the other one gets an error instead of waiting.
"""

import datetime
import multiprocessing as mproc
import os
import socket
import traceback
from types import SimpleNamespace

import pytest
import torch
import torch.nn.functional as F

E, K, H, I = 8, 4, 64, 32


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _weights():
    g = torch.Generator().manual_seed(7)
    r = lambda *shape: torch.randn(*shape, generator=g) * 0.1
    return {
        "gate.weight": r(E, H),
        "experts.gate_up_proj": r(E, 2 * I, H),
        "experts.down_proj": r(E, H, I),
        "shared_expert.gate_proj.weight": r(I, H),
        "shared_expert.up_proj.weight": r(I, H),
        "shared_expert.down_proj.weight": r(H, I),
        "shared_expert_gate.weight": r(1, H),
    }


def _route(x, p):
    probs = torch.softmax(x @ p["gate.weight"].t(), dim=-1)
    top, idx = torch.topk(probs, K, dim=-1)
    return idx.to(torch.int32), top / top.sum(-1, keepdim=True)


def _local_experts(rows, slot_e, slot_w, gu, dn):
    """fp32 partial per received row: the sum over its slots with a local expert, in slot order."""
    out = torch.zeros(rows.shape[0], H)
    for j in range(slot_e.shape[1]):
        for e in torch.unique(slot_e[:, j]).tolist():
            if e < 0:
                continue
            sel = slot_e[:, j] == e
            h = rows[sel] @ gu[e].t()
            h = F.silu(h[:, :I]) * h[:, I:]
            out[sel] += (h @ dn[e].t()) * slot_w[sel, j, None]
    return out


def _rank_main(rank, world, port, scenario, queue):
    try:
        os.environ["MASTER_ADDR"], os.environ["MASTER_PORT"] = "127.0.0.1", str(port)
        import torch.distributed as dist
        from janus_b200.ep import ExpertParallel, sum_partials
        from oracle.hybrid import moe_block
        dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=5))
        p = _weights()
        static = scenario.startswith("static")
        ep = ExpertParallel(E, static=static)
        gu, dn = ep.shard(p["experts.gate_up_proj"]), ep.shard(p["experts.down_proj"])
        n_tok = {"basic": 37 + 11 * rank, "empty": 0 if rank == 1 else 23, "one_rank": 19,
                 "static": 37 + 11 * rank, "static_empty": 0 if rank == 1 else 23}.get(scenario, 16)
        x = torch.randn(n_tok, H, generator=torch.Generator().manual_seed(100 + rank))
        idx, w = _route(x, p)
        if scenario == "one_rank":  # every slot of rank 0's tokens on rank 1's experts and the reverse
            idx = (idx % (E // world)) + (1 - rank) * (E // world)
        if scenario == "dead_peer" and rank == 1:
            queue.put((rank, "left"))
            return  # leaves before the collective; the process group is never joined again
        if static:
            cap = ep.agree_capacity(n_tok, "cpu")  # the same block size on both ranks
            (rows, se, sw), row_index = ep.dispatch_static(x, idx, w, cap)
            assert rows.shape[0] == ep.world * cap
            part = _local_experts(rows, se, sw, gu, dn)
            back, row_index = ep.combine_static(part, row_index)
            routed = sum_partials(back, row_index)
            sent = int((row_index >= 0).sum())
        else:
            (rows, se, sw), handle = ep.dispatch(x, idx, w)
            part = _local_experts(rows, se, sw, gu, dn)
            back, row_index = ep.combine(part, handle)
            routed = sum_partials(back, row_index)
            sent = sum(handle[0])
        if scenario == "one_rank":
            ref = torch.zeros(n_tok, H)
            for j in range(K):
                for t in range(n_tok):
                    e = int(idx[t, j])
                    h = x[t] @ p["experts.gate_up_proj"][e].t()
                    h = F.silu(h[:I]) * h[I:]
                    ref[t] += (h @ p["experts.down_proj"][e].t()) * w[t, j]
            err = float((routed - ref).abs().max()) if n_tok else 0.0
        else:
            shared = F.silu(x @ p["shared_expert.gate_proj.weight"].t()) * (x @ p["shared_expert.up_proj.weight"].t())
            shared = shared @ p["shared_expert.down_proj.weight"].t()
            got = routed + torch.sigmoid(x @ p["shared_expert_gate.weight"].t()) * shared
            ref = moe_block(x, p, SimpleNamespace(top_k=K, moe_intermediate=I))
            err = float((got - ref).abs().max()) if n_tok else 0.0
        # one row per (token, rank owning any of its experts): deduplicated per rank, not per expert
        pairs = {(t, int(e) // ep.local) for t in range(n_tok) for e in idx[t].tolist()}
        queue.put((rank, ("ok", err, sent, len(pairs))))
        dist.destroy_process_group()
    except Exception as e:  # reported to the parent, which asserts on it
        queue.put((rank, ("error", type(e).__name__, str(e)[:200], traceback.format_exc()[-400:])))


def _run(scenario, world=2, timeout=60):
    ctx = mproc.get_context("spawn")
    queue = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_rank_main, args=(r, world, port, scenario, queue)) for r in range(world)]
    for pr in procs:
        pr.start()
    results = {}
    try:
        for _ in range(world):
            rank, res = queue.get(timeout=timeout)
            results[rank] = res
    finally:
        for pr in procs:
            pr.join(timeout=10)
            if pr.is_alive():
                pr.kill()
    return results


@pytest.mark.parametrize("scenario", ["basic", "empty", "one_rank", "static", "static_empty"])
def test_expert_parallel_matches_single_process(scenario):
    """Equal to the oracle's MoE block with all experts; a token is sent once per rank owning any of its experts."""
    res = _run(scenario)
    for rank, r in res.items():
        assert r[0] == "ok", r
        assert r[1] < 1e-5, f"rank {rank}: max |ep - oracle| = {r[1]:.2e}"
        assert r[2] == r[3], f"rank {rank}: sent {r[2]} rows, expected {r[3]} (token, rank) pairs"


def test_dead_peer_ends_in_an_error_not_a_hang():
    """Rank 1 leaves before the dispatch; rank 0's collective must fail within the process-group timeout."""
    res = _run("dead_peer", timeout=90)
    assert res[1] == "left"
    assert res[0][0] == "error", res[0]
