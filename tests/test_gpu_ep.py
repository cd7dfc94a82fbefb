"""Expert-parallel readout on 2 GPUs (NCCL all-to-all): each rank keeps half of the experts, runs the golden MoE
cases through janus_b200.model.DecisionReadout(ep=...) and must match the reference's probabilities like the
single-GPU path, and the single-GPU path itself up to the reordered fp32 expert sum. Skipped below 2 GPUs."""

import datetime
import multiprocessing as mproc
import os
import socket
import traceback

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu
CASES = ("tiny_moe_tree", "wa3b_tree")


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rank_main(rank, world, port, queue):
    try:
        os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
        import torch.distributed as dist
        from janus_b200.ep import ExpertParallel
        from janus_b200.model import DecisionReadout
        from tests.golden_cases import case_model, load_cases
        torch.cuda.set_device(rank)
        dev = torch.device("cuda", rank)
        dist.init_process_group("nccl", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60),
                                device_id=dev)
        cases = load_cases()
        out = {}
        for name in CASES:
            case = cases[name]
            shape, weights, mode, packs = case_model(case)
            # each rank serves its own requests (rank 1 a shorter batch): the level sizes differ across ranks
            mine = packs if rank == 0 else packs[:1]
            single = DecisionReadout(shape, weights, mode, device=dev).probabilities(mine)
            for static in (False, True):
                ep = ExpertParallel(shape.experts, static=static)
                probs = DecisionReadout(shape, weights, mode, device=dev, ep=ep).probabilities(mine)
                ref_dev = max(float(np.abs(g.numpy() - np.array(r)).max())
                              for gp, rp in zip(probs, case["probs"]) for g, r in zip(gp, rp))
                single_dev = max(float((g - s).abs().max()) for gp, sp in zip(probs, single) for g, s in zip(gp, sp))
                out[(name, static)] = (ref_dev, single_dev, case["bf16_max_dev"])
        queue.put((rank, ("ok", out)))
        dist.barrier()
        dist.destroy_process_group()
    except Exception as e:
        queue.put((rank, ("error", type(e).__name__, str(e)[:300], traceback.format_exc()[-600:])))


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs 2 GPUs")
def test_expert_parallel_readout_matches_reference_and_single_gpu():
    ctx = mproc.get_context("spawn")
    queue = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_rank_main, args=(r, 2, port, queue)) for r in range(2)]
    for pr in procs:
        pr.start()
    res = {}
    try:
        for _ in range(2):
            rank, r = queue.get(timeout=600)
            res[rank] = r
    finally:
        for pr in procs:
            pr.join(timeout=60)
            if pr.is_alive():
                pr.kill()
    for rank, r in res.items():
        assert r[0] == "ok", r
        for name, (ref_dev, single_dev, floor) in r[1].items():
            print(f"rank {rank} {name}: |p_ep - p_ref| {ref_dev:.2e} (tolerance {max(2e-3, 1.5 * floor):.2e}), "
                  f"|p_ep - p_1gpu| {single_dev:.2e}")
            assert ref_dev <= max(2e-3, 1.5 * floor), (rank, name, ref_dev)
            assert single_dev <= 2e-3, (rank, name, single_dev)
