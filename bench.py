"""Benchmark of the B200 decision readout (workload 3: the 4B shape, 16 requests of an 8192-token state and 8 tree
questions per GPU).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl b200|reference]

One step is one forward readout of a batch of 16 requests (every level, every layer, heads): `value` is decision
requests per second over all ranks with the level tables already on the device; `e2e` is the same metric through
the public API (DecisionReadout.probabilities: host planning, one host-to-device copy, the device pass, one
device-to-host copy of the logits and the softmax) per step. Weights are random (seeded) and generated on the
device; requests are seeded synthetic token ids (no dataset). Multi-GPU: one process per GPU (torchrun), each rank a
replica serving its own 16 requests (requests are independent: weak scaling, no collective on the data path); the
step time is the max over ranks.

`--op moe` times the W4A16 MoE block of the 35B-A3B shape instead (hidden 2048, 256 experts of FFN 512, top-8;
`--moe-tokens` rows, default 131072 = a level-0 pass of 8 requests of 16384 tokens): routing, the two grouped GEMMs
and the combine per step, each timed with CUDA events, TFLOP/s of the grouped GEMMs against the measured bf16 peak.

`--op prefix` times the same batch with every state a prefix-cache hit: the states are encoded once into
snapshots (DecisionReadout.encode_prefixes) and each step runs the branch levels only.

`--op a3b [--ep]` runs workload 5 (the 35B-A3B shape, 40 layers, 8 requests of a 16384-token state per GPU), as
replicas or expert parallel over the torchrun group.

`--impl reference` times the reference algorithm on the host cores instead: the CPU oracle (oracle/hybrid.py, a
restatement of the reference's readout pinned to its golden outputs) on one request of the same workload, each
step through one 4-layer block of the model (3 DeltaNet + 1 attention layer, every level; the model is 8 such
blocks), plus one measured pass of the same request through all 32 layers as a check of that factor.

Besides the batch step, the line carries `request_latency_ms`: p50/p90 over single requests of the workload run one
at a time (batch 1), device time and end to end through the public API.
"""

import argparse
import json
import os
import statistics
import subprocess
import sys
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

import numpy as np  # noqa: E402
import torch  # noqa: E402

WORKLOAD = 3
REQUESTS_PER_GPU = 16
METRIC = "decision requests/s (4B shape, 8K state, 8 questions)"
UNIT = "requests/s"
PEAKS_FALLBACK = {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0}


def ncu_traffic():
    """DRAM bytes (dram__bytes_read.sum + dram__bytes_write.sum) of one level-0 launch per kernel, as the ncu
    summaries under profiles/ state them on a line `bench-traffic: kernel=<name> bytes=<B> requests=<R>` (the
    capture's request count; each request reads only its own state, so the traffic scales with the requests)."""
    import glob
    import re
    out = {}
    for path in sorted(glob.glob(os.path.join(ROOT, "profiles", "*.md"))):
        with open(path) as f:
            for line in f:
                m = re.match(r"\s*bench-traffic:\s*kernel=(\w+)\s+bytes=([0-9.eE+]+)\s+requests=(\d+)", line)
                if m:
                    out[m.group(1)] = (float(m.group(2)), int(m.group(3)), os.path.basename(path))
    return out


def peaks():
    path = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(path):
        with open(path) as f:
            p = json.load(f)
        return p, "measured"
    return PEAKS_FALLBACK, "fallback"


def nearest_rank(values, q):
    """The q-quantile by nearest rank (janus/loadtest.py:33-35); None for no values."""
    if not values:
        return None
    v = sorted(values)
    return v[min(len(v) - 1, max(0, int(np.ceil(q * len(v))) - 1))]


def dist_env():
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    return world, rank, local


class Clocks:
    """nvidia-smi samples of SM clock and throttle reasons while running (start before, stop after the timed region)."""

    def __init__(self, index, out):
        self.out = out
        q = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,clocks_event_reasons.hw_slowdown,"
             "clocks_event_reasons.hw_thermal_slowdown,clocks_event_reasons.sw_thermal_slowdown,"
             "clocks_event_reasons.sw_power_cap")
        try:
            self.proc = subprocess.Popen(["nvidia-smi", f"--id={index}", f"--query-gpu={q}", "--format=csv,noheader,nounits",
                                          "-lms", "200"], stdout=open(out, "w"), stderr=subprocess.DEVNULL)
        except OSError:
            self.proc = None

    def stop(self):
        if self.proc is None:
            return None
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
        rows = []
        with open(self.out) as f:
            for line in f:
                parts = [p.strip() for p in line.split(",")]
                if len(parts) >= 9:
                    rows.append(parts)
        if not rows:
            return None
        sm = [float(r[1]) for r in rows if r[1].replace(".", "").isdigit()]
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({n for r in rows for n, v in zip(names, r[5:9]) if v.lower() == "active"})
        return {"sm_mhz": statistics.median(sm) if sm else None,
                "sm_max_mhz": float(rows[0][2]) if rows[0][2].replace(".", "").isdigit() else None,
                "reasons": reasons, "samples": len(rows)}


def attention_flops(levels, shape):
    """4 * D * Hq * sum over query tokens of their visible keys (tree rule), per attention layer, per level."""
    per = []
    for lv in levels:
        lengths = np.diff(lv.row_start.astype(np.int64))
        own = float((lengths * (lengths + 1) // 2).sum())
        anc = float(sum(((hi - lo).astype(np.int64) * lengths).sum() for lo, hi in zip(lv.anc_lo, lv.anc_hi)))
        per.append(4.0 * shape.head_dim * shape.heads * (own + anc))
    return per


def chunk_algorithmic(levels, shape, which):
    """DeltaNet rule FLOPs and bytes per launch (per DeltaNet layer) at each level the kernel `which` runs (a
    bool per level): FLOPs per token per value head 6*Dk*Dv + 2*C*(3*Dk + 2*Dv) (C = 64); bytes = q, k, v (bf16) +
    g, beta (fp32) in, o out (bf16), the final fp32 state out when kept."""
    Dk, Dv, Hk, Hv = shape.lin_k_dim, shape.lin_v_dim, shape.lin_k_heads, shape.lin_v_heads
    out = []
    for lv, use in zip(levels, which):
        if not use:
            continue
        T = lv.T
        flops = T * Hv * (6 * Dk * Dv + 2 * 64 * (3 * Dk + 2 * Dv))
        byts = T * (2 * Hk * Dk * 2 + Hv * Dv * 2 + Hv * 8 + Hv * Dv * 2) + (lv.B * Hv * Dk * Dv * 4 if lv.keep else 0)
        out.append((flops, byts))
    return out


def run_reference(args):
    """The reference arm: the reference's CPU readout (or the oracle's restatement of it when the reference does
    not import) on a bounded sample of the workload, all host threads."""
    world, rank, _ = dist_env()
    if rank != 0:
        return
    cores = os.cpu_count() or 1
    torch.set_num_threads(cores)
    value, sample, detail = cpu_reference_rate(args.steps, min(args.warmup, 1), full_request=True)
    line = {"metric": METRIC, "value": value, "unit": UNIT, "n_gpus": args.gpus, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": detail["block_s"] * 1000.0, "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
            "impl": "reference",
            "config": {"workload": "4b-tree-8k-state-8q", "requests_per_gpu": 1, "sample": sample,
                       "same_config": False},
            "cpu_baseline": {"value": value, "unit": UNIT, "cores": cores, "sample": sample, **detail},
            "e2e": {"value": value, "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


def cpu_reference_rate(steps=1, warmup=0, full_request=False, kind=None):
    """The reference's CPU readout (fp32, all host threads) on one full request of the workload (8192-token state, 8
    tree questions). kind "reference": the reference's own code, its HybridBackbone plain CPU path over a
    transformers Qwen3.5 model read out by its DecisionModel (oracle/reference_cpu.py; the reference installed under
    baseline/_ref travels with the checkout); kind "port": the CPU oracle's restatement of it (oracle/hybrid.py),
    used when the reference or transformers does not import. Default: the reference when it imports. A timed step
    runs the request through one 4-layer block of the 4B shape (3 DeltaNet + 1 attention layer, every level,
    embedding and head included): the model is 8 repeats of that block, so a request costs 8 blocks (the embedding
    gather and the head, a few ms, are counted 8 times). With `full_request` the whole 32-layer model (full
    vocabulary) also runs the same request once, measured, as a check of that factor.
    Returns (requests/s from the block steps, description, details with the kind)."""
    from janus_b200 import synthetic
    from janus_b200.config import SHAPES
    from oracle import reference_cpu
    if kind is None:
        kind = "reference" if reference_cpu.available() else "port"
    full = SHAPES["4b"]
    blocks = full.layers // 4

    def readout(shape):
        weights = synthetic.make_weights(shape, seed=0, head="scalar", device="cpu")
        if kind == "reference":
            model = reference_cpu.reference_readout(shape, weights, "tree", grouped_branches=True)
            return lambda pack: model.forward_many(reference_cpu.reference_packs([pack]))
        from oracle import hybrid as oracle
        model = oracle.Oracle(shape, weights)
        return lambda pack: oracle.probabilities(model.logits(pack, "tree"))

    run = readout(full.with_layers(4, vocab=4096))
    pack = synthetic.q4b_request(vocab=4096, seed=0)
    times = []
    with torch.no_grad():
        for i in range(max(0, warmup) + max(1, steps)):
            t0 = time.perf_counter()
            run(pack)
            if i >= warmup:
                times.append(time.perf_counter() - t0)
    block_s = statistics.median(times)
    detail = {"block_s": block_s, "blocks_per_request": blocks, "block_steps": len(times), "kind": kind}
    what = ("the reference's own CPU readout (janus HybridBackbone + DecisionModel over transformers Qwen3.5)"
            if kind == "reference" else "the CPU oracle (a restatement of the reference)")
    sample = (f"one 4B-shape request ({pack.token_count} tokens: 8192-token state, 8 questions) through one 4-layer "
              f"block (3 DeltaNet + 1 attention) of {what} per step, fp32, {torch.get_num_threads()} threads, "
              f"median of {len(times)} steps; requests/s = 1 / ({blocks} x block seconds)")
    if full_request:
        del run
        run = readout(full)
        pack = synthetic.q4b_request(seed=0)
        t0 = time.perf_counter()
        with torch.no_grad():
            run(pack)
        detail["full_request_s"] = time.perf_counter() - t0
        detail["full_request"] = "the same request through all 32 layers (vocab 248320), measured once"
        detail["block_extrapolation_error"] = blocks * block_s / detail["full_request_s"] - 1.0
    return 1.0 / (blocks * block_s), sample, detail


def run_moe(args):
    """The MoE block of the A3B shape on one GPU: route -> gate/up GEMM -> down GEMM -> combine, experts in the
    BASELINE's int4 group-128 format or (`--moe-format nvfp4`) the reference's NVFP4. With `--vs-reference` and the
    reference installed under baseline/_ref, the reference's own Triton kernels (`fused_moe`,
    janus/moe_w4a16.py:122-140, NVFP4 only) run on the same routing and weights and are timed the same way, and the
    two outputs are compared."""
    from janus_b200 import ops
    from janus_b200.synthetic import int4_quantized, nvfp4_quantized
    device = torch.device("cuda", 0)
    S, E, k, H, I = args.moe_tokens, 256, 8, 2048, 512
    fp4 = args.moe_format == "nvfp4"
    g = torch.Generator(device=device).manual_seed(0)
    x = (torch.randn(S, H, generator=g, device=device) * 0.5).to(torch.bfloat16)
    logits = torch.randn(S, E, generator=g, device=device)
    shared = torch.randn(S, H, generator=g, device=device).to(torch.bfloat16)
    sgate = torch.randn(S, generator=g, device=device)
    if fp4:
        gu = nvfp4_quantized((E, 2 * I, H), 11, "experts", device, halves=True)
        dn = nvfp4_quantized((E, H, I), 12, "experts", device)
        gemm = lambda a, w, plan, gated, **kw: ops.moe_grouped_nvfp4(a, *w, plan, gated, k, **kw)
    else:
        gu = int4_quantized((E, 2 * I, H), 11, "experts", device)
        dn = int4_quantized((E, H, I), 12, "experts", device)
        gemm = lambda a, w, plan, gated, **kw: ops.moe_grouped_w4a16(a, *w, plan, gated, k, **kw)
    status = torch.zeros(1, dtype=torch.int32, device=device)
    flush = torch.empty(256 << 20, dtype=torch.uint8, device=device)  # > L2 between steps
    names = ["moe_route", "gemm_gate_up", "gemm_down", "moe_combine"]
    times = {n: [] for n in names}
    for step in range(args.warmup + args.steps):
        flush.zero_()
        ev = [torch.cuda.Event(enable_timing=True) for _ in range(5)]
        ev[0].record()
        plan = ops.moe_route(logits, k)
        ev[1].record()
        h = gemm(x, gu, plan, True, status=status)
        ev[2].record()
        y2 = gemm(h, dn, plan, False, topk_w=plan[1], status=status)
        ev[3].record()
        ops.moe_combine(y2, k, shared, sgate)
        ev[4].record()
        torch.cuda.synchronize()
        if step >= args.warmup:
            for i, n in enumerate(names):
                times[n].append(ev[i].elapsed_time(ev[i + 1]))
    if int(status.item()) != 0:
        raise RuntimeError("moe bench: a device-side wait ran out")
    ms = {n: statistics.median(v) for n, v in times.items()}
    A = S * k
    flops = {"gemm_gate_up": 2.0 * A * 2 * I * H, "gemm_down": 2.0 * A * H * I}
    pk, kind = peaks()
    gemm_ms = ms["gemm_gate_up"] + ms["gemm_down"]
    achieved = (flops["gemm_gate_up"] + flops["gemm_down"]) / (gemm_ms * 1e-3) / 1e12
    line = {
        "metric": "MoE W4A16 grouped GEMMs, A3B shape (hidden 2048, 256 experts x FFN 512, top-8)",
        "value": achieved, "unit": "TFLOP/s", "steps": args.steps, "warmup": args.warmup,
        "config": {"tokens": S, "assignments": A, "experts": E, "top_k": k, "format": args.moe_format,
                   "l2": "256 MiB written between steps"},
        "ms": ms, "tflops": {n: flops[n] / (ms[n] * 1e-3) / 1e12 for n in flops},
        "roofline": {"bound": "tensor", "achieved": achieved, "peak": pk["bf16_tflops"], "unit": "TFLOP/s",
                     "frac": achieved / pk["bf16_tflops"], "peak_kind": kind + " (burst bf16)"},
    }
    if args.vs_reference:
        line["reference_fused_moe"] = reference_fused_moe(args, x, plan, gu, dn, gemm, k, flush) if fp4 else \
            "the reference's fused kernel reads NVFP4 only (--moe-format nvfp4)"
    print(json.dumps(line))


def reference_fused_moe(args, x, plan, gu, dn, gemm, k, flush):
    """The reference's Triton NVFP4 MoE (`fused_moe` from baseline/_ref, its plan `align` included) against this
    library's plan + two grouped GEMMs + per-token sum, on the same routing (ids and weights) and weights: device
    milliseconds of each and the largest difference of their outputs."""
    ref_root = os.path.join(ROOT, "baseline", "_ref")
    if not os.path.isdir(os.path.join(ref_root, "janus")):
        return {"unavailable": "the reference is not installed under baseline/_ref"}
    sys.path.insert(0, ref_root)
    try:
        from janus.moe_w4a16 import fused_moe
    except Exception as e:  # triton or the package missing on this box
        return {"unavailable": f"import failed: {type(e).__name__}: {e}"}
    from janus_b200 import ops
    idx, w = plan[0], plan[1]
    E = gu[0].shape[0]
    ref_args = (gu[0], gu[1], gu[2][..., None], dn[0], dn[1], dn[2][..., None])

    def ours():
        p = ops.moe_plan(idx, E)
        hh = gemm(x, gu, p, True)
        y2 = gemm(hh, dn, p, False, topk_w=w.reshape(-1))
        return ops.moe_combine(y2, k, None, None)

    def theirs():
        return fused_moe(x, idx.long(), w, *ref_args)

    out = {}
    for name, fn in (("janus_b200", ours), ("reference_triton", theirs)):
        for _ in range(args.warmup):
            fn()
        ts = []
        for _ in range(args.steps):
            flush.zero_()
            a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            a.record()
            res = fn()
            b.record()
            torch.cuda.synchronize()
            ts.append(a.elapsed_time(b))
        out[name] = {"ms": statistics.median(ts)}
        out[name + "_result"] = res
    d = (out.pop("janus_b200_result").float() - out.pop("reference_triton_result").float()).abs()
    out["max_abs_diff"] = float(d.max())
    out["speedup"] = out["reference_triton"]["ms"] / out["janus_b200"]["ms"]
    return out


def run_gemm(args):
    """The dense projections of the 4B shape at a level-0 pass of `--gemm-tokens` rows: the tcgen05 GEMM
    (janus_b200_gemm_bf16) against cuBLAS (torch F.linear) on the same operands, each timed with CUDA events over
    `--steps` launches after `--warmup`; the MLP gate/up also as the SwiGLU epilogue against cuBLAS + silu_mul."""
    import torch.nn.functional as F
    from janus_b200 import ops
    from janus_b200.config import SHAPES
    device = torch.device("cuda", 0)
    s = SHAPES["4b"]
    T, H = args.gemm_tokens, s.hidden
    g = torch.Generator(device=device).manual_seed(0)
    x = {k: torch.randn(T, k, generator=g, device=device).to(torch.bfloat16) for k in (H, s.value_dim, s.intermediate)}
    shapes = {"deltanet_proj": (s.conv_dim + s.value_dim + 2 * s.lin_v_heads, H),
              "attn_qkv": (2 * s.heads * s.head_dim + 2 * s.kv_heads * s.head_dim, H),
              "out_proj": (H, s.value_dim), "gate_up": (2 * s.intermediate, H), "down": (H, s.intermediate)}
    flush = torch.empty(256 << 20, dtype=torch.uint8, device=device)

    def timed(*fns):
        """Median ms of each of `fns`, the calls interleaved step by step so that they see the same clocks."""
        for _ in range(args.warmup):
            for fn in fns:
                fn()
        ms = [[] for _ in fns]
        for _ in range(args.steps):
            for fn, out in zip(fns, ms):
                flush.zero_()
                a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                a.record()
                fn()
                b.record()
                torch.cuda.synchronize()
                out.append(a.elapsed_time(b))
        return [statistics.median(m) for m in ms]

    pk, kind = peaks()
    rows = {}
    for name, (N, K) in shapes.items():
        w = (torch.randn(N, K, generator=g, device=device) * 0.02).to(torch.bfloat16)
        a = x[K]
        flops = 2.0 * T * N * K
        t_ours, t_cublas = timed(lambda: ops.gemm_bf16(a, w), lambda: F.linear(a, w))
        rows[name] = {"N": N, "K": K, "ms_tcgen05": t_ours, "ms_cublas": t_cublas,
                      "tflops_tcgen05": flops / t_ours / 1e9, "tflops_cublas": flops / t_cublas / 1e9}
        if name == "gate_up":
            wi = ops.swiglu_weight(w[:s.intermediate], w[s.intermediate:])
            t_fused, t_sep = timed(lambda: ops.gemm_bf16(a, wi, swiglu=True), lambda: ops.silu_mul(F.linear(a, w)))
            rows["gate_up+swiglu"] = {"ms_tcgen05_fused": t_fused, "ms_cublas_plus_silu_mul": t_sep,
                                      "tflops_tcgen05_fused": flops / t_fused / 1e9}
        del w
    total_ours = sum(r["ms_tcgen05"] for n, r in rows.items() if "ms_tcgen05" in r)
    total_cublas = sum(r["ms_cublas"] for n, r in rows.items() if "ms_cublas" in r)
    print(json.dumps({"metric": "dense projection GEMMs of one 4B layer group at a level-0 pass", "unit": "ms",
                      "tokens": T, "steps": args.steps, "warmup": args.warmup, "per_gemm": rows,
                      "ms_tcgen05": total_ours, "ms_cublas": total_cublas,
                      "peak": {"bf16_tflops": pk["bf16_tflops"], "kind": kind},
                      "l2": "256 MiB written between launches"}))


def run_a3b(args):
    """Workload 5: the 35B-A3B shape at full depth (40 layers, 256 experts of FFN 512, top-8, int4 group-128 experts),
    8 requests of a 16384-token state with 8 questions of 4 options per GPU. `--ep`: expert parallel over the
    torchrun group (each rank keeps 256 / N experts; the capturable static exchange, `janus_b200/ep.py`), otherwise
    one replica per GPU (all experts on every GPU: 16.6 GB of int4). One step = one readout of the rank's batch;
    `value` = requests/s over all ranks, the step time the max over ranks; weights random (seeded, generated on the
    device), requests seeded synthetic token ids."""
    import datetime
    import torch.distributed as dist
    from janus_b200 import synthetic
    from janus_b200.config import SHAPES
    from janus_b200.ep import ExpertParallel
    from janus_b200.model import DecisionReadout
    world, rank, local = dist_env()
    torch.cuda.set_device(local)
    device = torch.device("cuda", local)
    if world > 1:
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=600), device_id=device)
    shape = SHAPES["35b-a3b"]
    if args.layers:
        shape = shape.with_layers(args.layers)
    ep = ExpertParallel(shape.experts, static=True) if (args.ep and world > 1) else None
    weights = synthetic.make_weights(shape, seed=0, head="scalar", device=device)
    model = DecisionReadout(shape, weights, "tree", device=device, ep=ep)
    del weights
    torch.cuda.empty_cache()
    n_req = args.requests if args.requests != REQUESTS_PER_GPU else 8
    packs = [synthetic.a3b_request(seed=1000 * rank + j) for j in range(n_req)]
    prepared = model.prepare(packs)
    for _ in range(args.warmup):
        model.run(prepared)
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier(device_ids=[local])
    ev = []
    for _ in range(args.steps):
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record()
        model.run(prepared)
        b.record()
        ev.append((a, b))
    torch.cuda.synchronize()
    model.check_status()
    total = sum(a.elapsed_time(b) for a, b in ev)
    if world > 1:
        t = torch.tensor([total], dtype=torch.float64, device=device)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        total = float(t.item())
    ms = total / args.steps
    if rank == 0:
        print(json.dumps({
            "metric": "decision requests/s (35B-A3B shape, 16K state, 8 questions)", "value": world * n_req / (ms / 1e3),
            "unit": "requests/s", "n_gpus": world, "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms,
            "config": {"workload": "a3b-tree-16k-state-8q" + (f"-{args.layers}layers-INVALID" if args.layers else ""),
                       "requests_per_gpu": n_req, "tokens_per_gpu": sum(p.token_count for p in packs),
                       "parallelism": f"ep{world} (static exchange)" if ep is not None else f"dp{world} (replicas)",
                       "experts": "int4 group 128"}}), flush=True)
    if world > 1:
        dist.destroy_process_group()


def run_workload(args):
    """A BASELINE configuration other than the headline (`--workload 2`: the 0.8B shape, listwise + PointerHead, a
    2048-token state and one choice question, batch 64; `--workload 4`: the 0.8B cardinality stress pack, a 4096-token
    state with 32 questions, one of them 255 options, batch 1), on one GPU: requests/s at the workload's batch, then
    per-request latency p50/p90 at batch 1 (device time and end to end through DecisionReadout.probabilities).
    Weights random (seeded), requests seeded synthetic token ids. A side line; the headline is workload 3."""
    from janus_b200 import synthetic
    from janus_b200.config import SHAPES
    from janus_b200.model import DecisionReadout
    device = torch.device("cuda", 0)
    wid = args.workload
    shape_name, mode, _, batch = synthetic.WORKLOADS[wid]
    shape = SHAPES[shape_name]
    weights = synthetic.make_weights(shape, seed=0, head="pointer" if mode == "listwise" else "scalar", device=device)
    model = DecisionReadout(shape, weights, mode, device=device)
    del weights
    torch.cuda.empty_cache()
    packs = synthetic.workload_requests(wid, seed=7000, batch=batch)
    prepared = model.prepare(packs)
    for _ in range(args.warmup):
        model.run(prepared)
    torch.cuda.synchronize()
    ev = []
    for _ in range(args.steps):
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record()
        model.run(prepared)
        b.record()
        ev.append((a, b))
    torch.cuda.synchronize()
    model.check_status()
    ms = sum(a.elapsed_time(b) for a, b in ev) / args.steps
    singles = synthetic.workload_requests(wid, seed=8000, batch=max(1, args.latency_requests))
    dev_ms, e2e_ms = [], []
    for pk in singles:
        prep1 = model.prepare([pk])
        model.run(prep1)  # warm the shapes of this request
        torch.cuda.synchronize()
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record()
        model.run(prep1)
        b.record()
        torch.cuda.synchronize()
        dev_ms.append(a.elapsed_time(b))
        t0 = time.perf_counter()
        model.probabilities([pk])
        e2e_ms.append((time.perf_counter() - t0) * 1000.0)
    pct = lambda xs, q: float(statistics.quantiles(xs, n=10)[q // 10 - 1]) if len(xs) >= 2 else float(xs[0])
    print(json.dumps({
        "metric": f"decision requests/s and p50/p90 ms per request (workload {wid})",
        "value": batch / (ms / 1000.0), "unit": "requests/s", "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": ms,
        "request_latency_ms": {"per": f"single request (batch 1), {len(singles)} requests one at a time",
                               "device": {"p50": statistics.median(dev_ms), "p90": pct(dev_ms, 90)},
                               "e2e": {"p50": statistics.median(e2e_ms), "p90": pct(e2e_ms, 90)}},
        "config": {"workload": {2: "0.8b-listwise-2k-state-1q", 4: "0.8b-tree-4k-state-32q-stress"}.get(wid, str(wid)),
                   "requests_per_step": batch, "tokens_per_step": sum(p.token_count for p in packs),
                   "mode": mode, "data": "synthetic"},
    }), flush=True)


def run_prefix(args):
    """Repeated states (a prefix-cache hit for every request): the state level of the 16 requests is encoded once
    into snapshots; each timed step then runs the branch levels only, from the snapshots. A side line for the
    serving cache, not the headline (whose states are all new)."""
    from janus_b200 import synthetic
    from janus_b200.config import SHAPES
    from janus_b200.model import DecisionReadout
    device = torch.device("cuda", 0)
    shape = SHAPES["4b"]
    weights = synthetic.make_weights(shape, seed=0, head="scalar", device=device)
    model = DecisionReadout(shape, weights, "tree", device=device)
    del weights
    packs = [synthetic.q4b_request(seed=j) for j in range(args.requests)]
    s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    s.record()
    snaps = model.encode_prefixes(packs)
    e.record()
    torch.cuda.synchronize()
    encode_ms = s.elapsed_time(e)
    prepared = model.prepare(packs, prefixes=snaps)
    for _ in range(args.warmup):
        model.run(prepared)
    torch.cuda.synchronize()
    ev = []
    for _ in range(args.steps):
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record()
        model.run(prepared)
        b.record()
        ev.append((a, b))
    torch.cuda.synchronize()
    model.check_status()
    ms = sum(a.elapsed_time(b) for a, b in ev) / args.steps
    print(json.dumps({
        "metric": "decision requests/s with every state a prefix-cache hit (4B shape, 8K state, 8 questions)",
        "value": args.requests / (ms / 1000.0), "unit": "requests/s", "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": ms, "state_encode_ms": encode_ms,
        "snapshot_bytes_per_request": snaps[0].bytes if snaps else 0,
        "config": {"workload": "4b-tree-8k-state-8q, states from snapshots", "requests_per_gpu": args.requests},
    }))


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=10)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", default="b200", choices=["b200", "reference"])
    ap.add_argument("--requests", type=int, default=REQUESTS_PER_GPU)
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--latency-requests", type=int, default=8, help="single requests timed one at a time")
    ap.add_argument("--layers", type=int, default=0, help="debug: fewer layers (not a valid bench number)")
    ap.add_argument("--op", default="readout", choices=["readout", "moe", "prefix", "gemm", "a3b", "workload"])
    ap.add_argument("--workload", type=int, default=2, choices=[2, 4], help="--op workload: BASELINE configuration")
    ap.add_argument("--ep", action="store_true", help="--op a3b: expert parallel over the torchrun group")
    ap.add_argument("--gemm-tokens", type=int, default=131072)
    ap.add_argument("--moe-tokens", type=int, default=131072)
    ap.add_argument("--moe-format", default="int4", choices=["int4", "nvfp4"])
    ap.add_argument("--vs-reference", action="store_true", help="--op moe: also time the reference's Triton MoE")
    args = ap.parse_args()
    if args.warmup < 3:
        args.warmup = 3
    if args.op == "moe":
        run_moe(args)
        return
    if args.op == "prefix":
        run_prefix(args)
        return
    if args.op == "gemm":
        run_gemm(args)
        return
    if args.op == "a3b":
        run_a3b(args)
        return
    if args.op == "workload":
        run_workload(args)
        return
    if args.impl == "reference":
        run_reference(args)
        return

    world, rank, local = dist_env()
    torch.cuda.set_device(local)
    device = torch.device("cuda", local)
    pg = None
    if world > 1:
        import datetime
        import torch.distributed as dist
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=600), device_id=device)
        pg = dist

    from janus_b200 import ops, synthetic
    from janus_b200.config import SHAPES
    from janus_b200.model import DecisionReadout

    shape = SHAPES["4b"]
    if args.layers:
        shape = shape.with_layers(args.layers)
    weights = synthetic.make_weights(shape, seed=0, head="scalar", device=device)
    model = DecisionReadout(shape, weights, "tree", device=device)
    del weights
    torch.cuda.empty_cache()
    packs = [synthetic.q4b_request(seed=1000 * rank + j) for j in range(args.requests)]
    tokens = sum(p.token_count for p in packs)
    prepared = model.prepare(packs)
    levels, readout, plan = prepared

    def barrier():
        if pg is not None:
            pg.barrier(device_ids=[local])

    def max_over_ranks(x):
        if pg is None:
            return x
        t = torch.tensor([x], dtype=torch.float64, device=device)
        pg.all_reduce(t, op=pg.ReduceOp.MAX)
        return float(t.item())

    # warm-up
    for _ in range(args.warmup):
        model.run(prepared)
    torch.cuda.synchronize()

    # timed device pass
    attn_flops = attention_flops(levels, shape)
    # levels the chunk scan runs: long rows, and the leaf level's state fork as a segmented scan
    chunked = [model._chunked(lv) or model._packed_fork(lv) for lv in levels]
    ops.TIMED.clear()
    ops.TIMED["tree_attention"] = []
    ops.TIMED["gdn_chunk_scan"] = []
    ops.TIMED["gdn_fork_recurrent"] = []
    ops.TIMED["gemm_bf16"] = []
    ops.FLOPS.clear()
    import tempfile
    clocks = Clocks(local, os.path.join(tempfile.gettempdir(), f"janus_b200_clocks_{os.getpid()}_rank{rank}.csv"))
    barrier()
    torch.cuda.synchronize()
    launches0 = ops.LAUNCHES[0]
    step_events = []
    for _ in range(args.steps):
        s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        s.record()
        model.run(prepared)
        e.record()
        step_events.append((s, e))
    torch.cuda.synchronize()
    model.check_status()
    barrier()
    clock = clocks.stop()
    launches = (ops.LAUNCHES[0] - launches0) // args.steps
    gemm_flops_step = ops.FLOPS.get("gemm_bf16", 0.0) / args.steps
    step_ms = [s.elapsed_time(e) for s, e in step_events]
    total_ms = max_over_ranks(sum(step_ms))
    ms_per_step = total_ms / args.steps
    value = world * args.requests / (ms_per_step / 1000.0)

    # per-kernel device time inside the timed region
    kernel_ms = {name: sum(s.elapsed_time(e) for s, e in rec) / args.steps for name, rec in ops.TIMED.items() if rec}
    n_attn_layers = sum(1 for t in shape.layer_types if t != "linear_attention")
    n_lin_layers = shape.layers - n_attn_layers
    attn_launch = ops.TIMED["tree_attention"]
    per_attn = [s.elapsed_time(e) for s, e in attn_launch]
    gemm_launches = list(ops.TIMED["gemm_bf16"])
    ops.TIMED.clear()

    # where one (extra, untimed) step's device time goes, per library op; the rest is cuBLAS GEMMs and torch glue
    ops.TIMED.clear()
    ops.TIMED.update({name: [] for name in ops.OPS})
    model.run(prepared)
    torch.cuda.synchronize()
    op_ms = {name: round(sum(s.elapsed_time(e) for s, e in rec), 2) for name, rec in ops.TIMED.items() if rec}
    ops.TIMED.clear()

    # the roofline of each of the library's timed kernels; the line's `roofline` is the dominant one's
    pk, pk_kind = peaks()

    def kernel_roofline(name):
        if name == "tree_attention":
            flops_step = n_attn_layers * sum(attn_flops)
            launches_per_step = len(per_attn) // args.steps
            achieved = flops_step / (kernel_ms[name] / 1000.0) / 1e12
            peak = pk["bf16_tflops_sustained"]
            return {"kernel": "tree_attention", "bound": "tensor", "achieved": achieved, "peak": peak,
                    "unit": "TFLOP/s", "frac": achieved / peak, "traffic": None,
                    "peak_kind": f"{pk_kind} bf16 sustained",
                    "algorithmic_per_launch": flops_step / max(1, launches_per_step),
                    "launches_per_step": launches_per_step, "ms_per_step": kernel_ms[name]}
        if name == "gemm_bf16":  # the tcgen05 dense GEMM: the MLP's gate/up with the SwiGLU epilogue (2 M N K each)
            achieved = gemm_flops_step / (kernel_ms[name] / 1000.0) / 1e12
            peak = pk["bf16_tflops_sustained"]
            return {"kernel": "gemm_bf16", "bound": "tensor", "achieved": achieved, "peak": peak, "unit": "TFLOP/s",
                    "frac": achieved / peak, "traffic": None, "peak_kind": f"{pk_kind} bf16 sustained",
                    "launches_per_step": len(gemm_launches) // args.steps, "ms_per_step": kernel_ms[name]}
        if name in ("gdn_chunk_scan", "gdn_fork_recurrent"):
            alg = chunk_algorithmic(levels, shape, chunked if name == "gdn_chunk_scan" else [not c for c in chunked])
            fl = sum(f for f, _ in alg) * n_lin_layers
            by = sum(b for _, b in alg) * n_lin_layers
            sec = kernel_ms[name] / 1000.0
            t_peak = pk["bf16_tflops_sustained"] * 1e12
            b_peak = pk["hbm_gbs"] * 1e9
            if fl / t_peak > by / b_peak:
                r = {"kernel": name, "bound": "tensor", "achieved": fl / sec / 1e12, "peak": t_peak / 1e12,
                     "unit": "TFLOP/s", "frac": fl / sec / t_peak, "traffic": None}
            else:
                r = {"kernel": name, "bound": "hbm", "achieved": by / sec / 1e9, "peak": b_peak / 1e9,
                     "unit": "GB/s", "frac": by / sec / b_peak, "traffic": None}
            r["ms_per_step"] = kernel_ms[name]
            r["peak_kind"] = pk_kind
            return r
        return None

    dominant = max(kernel_ms, key=kernel_ms.get) if kernel_ms else None
    roof = kernel_roofline(dominant) if dominant else None
    roofline_kernels = {}
    for name in kernel_ms:
        r = kernel_roofline(name)
        if r is not None:
            roofline_kernels[name] = {k: r[k] for k in ("bound", "achieved", "peak", "unit", "frac", "ms_per_step")}
    traffic = ncu_traffic()
    if (roof is not None and roof["kernel"] in traffic and not args.layers
            and not (roof["kernel"] == "gemm_bf16" and not shape.intermediate)):
        # DRAM traffic of one level-0 launch (ncu) beside the algorithmic bytes of that launch
        lv0 = levels[0]
        if roof["kernel"] == "tree_attention":
            alg0 = lv0.T * (3 * shape.heads * shape.head_dim * 2 + 2 * shape.kv_heads * shape.head_dim * 2)
        elif roof["kernel"] == "gemm_bf16":  # the MLP's gate/up + SwiGLU: y in, weights, the I-wide product out
            I = shape.intermediate
            alg0 = lv0.T * shape.hidden * 2 + 2 * I * shape.hidden * 2 + lv0.T * I * 2
        else:
            alg0 = chunk_algorithmic(levels[:1], shape, [True])[0][1]
        t_bytes, t_requests, t_file = traffic[roof["kernel"]]
        roof["traffic"] = t_bytes * args.requests / t_requests
        roof["traffic_per"] = f"level-0 launch (ncu capture at {t_requests} requests, profiles/{t_file}, scaled)"
        roof["algorithmic_bytes_per_level0_launch"] = float(alg0)

    # end to end through the public API: host packing -> H2D -> device pass -> D2H -> softmax
    e2e_ms = []
    h2d = d2h = 0
    barrier()
    for _ in range(max(3, args.steps // 2)):
        torch.cuda.synchronize()
        t0 = time.perf_counter()
        probs = model.probabilities(packs)  # pack -> H2D -> device pass -> D2H of logits + status -> softmax
        e2e_ms.append((time.perf_counter() - t0) * 1000.0)
        h2d, d2h = model.last_plan.h2d_bytes, model._readout.n_slots * 4 + model.status.numel() * 4
    e2e_step = max_over_ranks(statistics.median(e2e_ms))
    e2e_value = world * args.requests / (e2e_step / 1000.0)

    # per-request latency: requests of the workload one at a time (batch 1), device time of the readout pass and
    # end to end through the public API
    lat_dev, lat_e2e = [], []
    for j, p1 in enumerate(packs[:args.latency_requests]):
        prep1 = model.prepare([p1])
        if j == 0:
            model.run(prep1)
            model.probabilities([p1])
        torch.cuda.synchronize()
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record()
        model.run(prep1)
        b.record()
        torch.cuda.synchronize()
        lat_dev.append(a.elapsed_time(b))
        t0 = time.perf_counter()
        model.probabilities([p1])
        lat_e2e.append((time.perf_counter() - t0) * 1000.0)
    model.check_status()

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        cores = os.cpu_count() or 1
        torch.set_num_threads(cores)
        v, sample, detail = cpu_reference_rate(1, 0)
        cpu = {"value": v, "unit": UNIT, "cores": cores, "sample": sample, **detail}

    if rank == 0:
        p = lambda q: nearest_rank(step_ms, q)
        line = {"metric": METRIC, "value": value, "unit": UNIT, "n_gpus": world, "steps": args.steps,
                "warmup": args.warmup, "ms_per_step": ms_per_step, "higher_is_better": True, "scaling": "weak",
                "vs_baseline": None, "dtype": "bf16", "data": "synthetic",
                "config": {"workload": "4b-tree-8k-state-8q" + (f"-{args.layers}layers-INVALID" if args.layers else ""),
                           "requests_per_gpu": args.requests, "tokens_per_gpu": tokens, "state_tokens": 8192,
                           "questions": 8, "parallelism": f"dp{world} (replicas)",
                           "l2": "inputs larger than L2 (activations of a level are GBs)"},
                "latency_ms": {"p50": p(0.5), "p90": p(0.9), "per": "batch step (every request of the batch completes at its end)"},
                "request_latency_ms": {
                    "per": f"single request (batch 1), {len(lat_dev)} requests of the workload one at a time",
                    "device": {"p50": nearest_rank(lat_dev, 0.5), "p90": nearest_rank(lat_dev, 0.9)},
                    "e2e": {"p50": nearest_rank(lat_e2e, 0.5), "p90": nearest_rank(lat_e2e, 0.9)}},
                "e2e": {"value": e2e_value, "unit": UNIT, "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h,
                        "ms_per_step": e2e_step},
                "gpu_launches": launches, "kernel_ms_per_step": kernel_ms, "op_ms_one_step": op_ms, "roofline": roof,
                "roofline_kernels": roofline_kernels, "cpu_baseline": cpu,
                "clocks": clock}
        print(json.dumps(line), flush=True)
    if pg is not None:
        pg.destroy_process_group()


if __name__ == "__main__":
    main()
