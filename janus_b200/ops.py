"""torch-tensor wrappers over the C ABI (include/janus_b200.h). Each op checks dtypes/devices/contiguity, launches
on the current CUDA stream of the tensors' device and returns the output tensors; errors raise (ValueError for bad
arguments, janus_b200._lib.JanusError for CUDA failures). There is no CPU path."""

import ctypes

import torch

from . import _lib

BF16, F32, I32 = torch.bfloat16, torch.float32, torch.int32

# Instrumentation for the benchmark: LAUNCHES counts the kernels launched through this module; for op names in
# TIMED, every call records a CUDA event pair on the launching stream into TIMED[name] (start, end, call kwargs
# summary) so kernel durations can be read after a synchronize.
LAUNCHES = [0]
TIMED = {}
OPS = []  # names of the instrumented ops
FLOPS = {}  # op name -> tensor-core FLOPs issued so far (the dense GEMM: 2 M N K per call)


def _instrument(name, kernels=1):
    OPS.append(name)

    def wrap(fn):
        def inner(*args, **kwargs):
            LAUNCHES[0] += kernels
            rec = TIMED.get(name)
            if rec is None:
                return fn(*args, **kwargs)
            s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            s.record()
            out = fn(*args, **kwargs)
            e.record()
            rec.append((s, e))
            return out
        inner.__name__, inner.__doc__ = fn.__name__, fn.__doc__
        return inner
    return wrap


def _ptr(t):
    return None if t is None else ctypes.c_void_p(t.data_ptr())


def _opt(t, dtype, name):
    """An optional tensor argument: None passes as a null pointer."""
    return None if t is None else _need(t, dtype, name)


def _stream(t):
    return ctypes.c_void_p(torch.cuda.current_stream(t.device).cuda_stream)


def _need(t, dtype, name, contiguous=True):
    if t is None:
        raise ValueError(f"{name} is required")
    if not t.is_cuda:
        raise ValueError(f"{name} must be a CUDA tensor (janus_b200 has no CPU path)")
    if t.dtype != dtype:
        raise ValueError(f"{name} must be {dtype}, got {t.dtype}")
    if contiguous and not t.is_contiguous():
        raise ValueError(f"{name} must be contiguous")
    return t


@_instrument("embed_rmsnorm", 1)
def embed_rmsnorm(table, ids, norm_w, eps, x=None, y=None):
    _need(table, BF16, "table"); _need(ids, I32, "ids"); _need(norm_w, BF16, "norm_w")
    T, H = ids.shape[0], table.shape[1]
    x = torch.empty(T, H, dtype=F32, device=ids.device) if x is None else x
    y = torch.empty(T, H, dtype=BF16, device=ids.device) if y is None else y
    _lib.check(_lib.load().janus_b200_embed_rmsnorm(_ptr(table), table.shape[0], H, _ptr(ids), T, _ptr(norm_w), eps,
                                                    _ptr(x), _ptr(y), _stream(ids)), "embed_rmsnorm")
    return x, y


@_instrument("add_rmsnorm", 1)
def add_rmsnorm(x, delta, norm_w, eps, y=None):
    """x += delta (in place; delta may be None or a row-strided bf16 view), returns y = rmsnorm(x) * (1 + w)."""
    _need(x, F32, "x"); _need(norm_w, BF16, "norm_w")
    T, H = x.shape
    if delta is not None:
        _need(delta, BF16, "delta", contiguous=False)
        if delta.stride(1) != 1 or delta.shape != (T, H):
            raise ValueError("delta must be [T, H] with unit column stride")
    y = torch.empty(T, H, dtype=BF16, device=x.device) if y is None else y
    _lib.check(_lib.load().janus_b200_add_rmsnorm(_ptr(x), _ptr(delta), 0 if delta is None else delta.stride(0), T, H,
                                                  _ptr(norm_w), eps, _ptr(y), _stream(x)), "add_rmsnorm")
    return y


@_instrument("silu_mul", 1)
def silu_mul(gu, out=None):
    _need(gu, BF16, "gu")
    T, two_i = gu.shape
    out = torch.empty(T, two_i // 2, dtype=BF16, device=gu.device) if out is None else out
    _lib.check(_lib.load().janus_b200_silu_mul(_ptr(gu), T, two_i // 2, _ptr(out), _stream(gu)), "silu_mul")
    return out


@_instrument("gated_rmsnorm", 1)
def gated_rmsnorm(core, z, w, eps, out=None):
    """core bf16 [T, Hv, Dv]; z bf16 [T, Hv*Dv] view with unit column stride."""
    _need(core, BF16, "core"); _need(z, BF16, "z", contiguous=False); _need(w, BF16, "w")
    T, Hv, Dv = core.shape
    if z.stride(1) != 1 or z.shape != (T, Hv * Dv):
        raise ValueError("z must be [T, Hv*Dv] with unit column stride")
    out = torch.empty(T, Hv * Dv, dtype=BF16, device=core.device) if out is None else out
    _lib.check(_lib.load().janus_b200_gated_rmsnorm(_ptr(core), _ptr(z), z.stride(0), T, Hv, Dv, _ptr(w), eps, _ptr(out),
                                                    _stream(core)), "gated_rmsnorm")
    return out


@_instrument("gdn_prologue", 1)
def gdn_prologue(proj, row_start, row_of_token, parent, tail_in, keep_tail, conv_w, A_log, dt_bias, Hk, Dk, Hv, Dv):
    """proj bf16 [T, >= C + Hv*Dv + 2Hv] (unit column stride). Returns q, k, v, g, beta, tail_out (or None)."""
    _need(proj, BF16, "proj", contiguous=False)
    if proj.stride(1) != 1:
        raise ValueError("proj must have unit column stride")
    T = proj.shape[0]
    B = row_start.shape[0] - 1
    C = 2 * Hk * Dk + Hv * Dv
    K = conv_w.shape[-1]
    dev = proj.device
    q = torch.empty(T, Hk, Dk, dtype=BF16, device=dev)
    k = torch.empty(T, Hk, Dk, dtype=BF16, device=dev)
    v = torch.empty(T, Hv, Dv, dtype=BF16, device=dev)
    g = torch.empty(T, Hv, dtype=F32, device=dev)
    beta = torch.empty(T, Hv, dtype=F32, device=dev)
    tail_out = torch.empty(B, K - 1, C, dtype=BF16, device=dev) if keep_tail else None
    if tail_in is not None:
        _need(tail_in, BF16, "tail_in")
    _lib.check(_lib.load().janus_b200_gdn_prologue(
        _ptr(proj), proj.stride(0), T, B, _ptr(_need(row_start, I32, "row_start")),
        _ptr(_need(row_of_token, I32, "row_of_token")), _ptr(parent), _ptr(tail_in), _ptr(tail_out),
        _ptr(_need(conv_w, BF16, "conv_w")), _ptr(_need(A_log, BF16, "A_log")), _ptr(_need(dt_bias, BF16, "dt_bias")),
        Hk, Dk, Hv, Dv, K, _ptr(q), _ptr(k), _ptr(v), _ptr(g), _ptr(beta), _stream(proj)), "gdn_prologue")
    return q, k, v, g, beta, tail_out


@_instrument("gdn_fork_recurrent", 1)
def gdn_fork_recurrent(q, k, v, g, beta, row_start, child_start, state_in, keep_state, scale):
    """Rows grouped under P = len(child_start) - 1 parents; state_in [P, Hv, Dk, Dv] fp32 or None."""
    T, Hk, Dk = q.shape
    Hv, Dv = v.shape[1], v.shape[2]
    B = row_start.shape[0] - 1
    P = child_start.shape[0] - 1
    o = torch.empty(T, Hv, Dv, dtype=BF16, device=q.device)
    state_out = torch.empty(B, Hv, Dk, Dv, dtype=F32, device=q.device) if keep_state else None
    if state_in is not None:
        _need(state_in, F32, "state_in")
        if state_in.shape[0] != P:
            raise ValueError(f"state_in has {state_in.shape[0]} rows for {P} parents")
    for t, n in ((q, "q"), (k, "k"), (v, "v")):
        _need(t, BF16, n)
    _lib.check(_lib.load().janus_b200_gdn_fork_recurrent(
        _ptr(q), _ptr(k), _ptr(v), _ptr(_need(g, F32, "g")), _ptr(_need(beta, F32, "beta")), T, B,
        _ptr(_need(row_start, I32, "row_start")), _ptr(_need(child_start, I32, "child_start")), P, _ptr(state_in),
        _ptr(state_out), Hk, Hv, Dk, Dv, scale, _ptr(o), _stream(q)), "gdn_fork_recurrent")
    return o, state_out


@_instrument("gdn_chunk_scan", 2)
def gdn_chunk_scan(q, k, v, g, beta, row_start, chunk_start, n_chunks, state_in, state_row, keep_state, scale,
                   status=None, segment=None, fused=None):
    """Long rows in 64-token chunks; row b starts from state_in[state_row[b]] (None: zeros / identity map).
    chunk_start int32 [B+1] (first chunk of each row), n_chunks = chunk_start[B]. status: optional device int32
    word set to 1 if a bounded device-side wait ran out. segment: optional int32 [T] ids of token segments that do
    not interact, each starting from the row's initial state (rows of at most 64 tokens, no kept state).
    fused: True runs the one-launch form (janus_b200_gdn_chunk_scan_fused: the prep of chunk c+1 under the state
    pass of chunk c, nothing through HBM), False or None the two-launch form (prep over all chunks in parallel into
    a workspace, then the state pass); the two give bit-identical results. The two-launch form is the faster one on
    every measured shape (the prep's latency chain per chunk is about 3.5x the state pass's, and only the parallel
    prep over all chunks hides it), so it is the default."""
    if segment is not None:
        _need(segment, I32, "segment")
        if keep_state:
            raise ValueError("gdn_chunk_scan: a segmented scan keeps no state")
    T, Hk, Dk = q.shape
    Hv, Dv = v.shape[1], v.shape[2]
    B = row_start.shape[0] - 1
    o = torch.empty(T, Hv, Dv, dtype=BF16, device=q.device)
    state_out = torch.empty(B, Hv, Dk, Dv, dtype=F32, device=q.device) if keep_state else None
    if state_in is not None:
        _need(state_in, F32, "state_in")
    if state_row is not None:
        _need(state_row, I32, "state_row")
    for t, n in ((q, "q"), (k, "k"), (v, "v")):
        _need(t, BF16, n)
    lib = _lib.load()
    if fused:
        if segment is not None:
            raise ValueError("gdn_chunk_scan: the one-launch form takes no segments")
        _lib.check(lib.janus_b200_gdn_chunk_scan_fused(
            _ptr(q), _ptr(k), _ptr(v), _ptr(_need(g, F32, "g")), _ptr(_need(beta, F32, "beta")), T, B,
            _ptr(_need(row_start, I32, "row_start")), _ptr(_need(chunk_start, I32, "chunk_start")), n_chunks,
            _ptr(state_in), _ptr(state_row), _ptr(state_out), Hk, Hv, Dk, Dv, scale, _ptr(o), _ptr(status),
            _stream(q)), "gdn_chunk_scan_fused")
        return o, state_out
    nbytes = lib.janus_b200_gdn_chunk_scan_workspace(T, n_chunks, Hv)
    ws = torch.empty(max(1, nbytes), dtype=torch.uint8, device=q.device)
    _lib.check(lib.janus_b200_gdn_chunk_scan(
        _ptr(q), _ptr(k), _ptr(v), _ptr(_need(g, F32, "g")), _ptr(_need(beta, F32, "beta")), T, B,
        _ptr(_need(row_start, I32, "row_start")), _ptr(_need(chunk_start, I32, "chunk_start")), n_chunks,
        _ptr(state_in), _ptr(state_row), _ptr(segment), _ptr(state_out), Hk, Hv, Dk, Dv, scale, _ptr(ws), ws.numel(),
        _ptr(o), _ptr(status), _stream(q)), "gdn_chunk_scan")
    return o, state_out


@_instrument("attn_qk_prep", 1)
def attn_qk_prep(qkv, positions, inv_freq, q_norm_w, k_norm_w, eps, Hq, Hkv, D, k_out=None, v_out=None):
    _need(qkv, BF16, "qkv", contiguous=False)
    if qkv.stride(1) != 1:
        raise ValueError("qkv must have unit column stride")
    T = qkv.shape[0]
    dev = qkv.device
    q = torch.empty(T, Hq, D, dtype=BF16, device=dev)
    k = torch.empty(T, Hkv, D, dtype=BF16, device=dev) if k_out is None else k_out
    v = torch.empty(T, Hkv, D, dtype=BF16, device=dev) if v_out is None else v_out
    _lib.check(_lib.load().janus_b200_attn_qk_prep(
        _ptr(qkv), qkv.stride(0), T, _ptr(_need(positions, I32, "positions")), _ptr(_need(inv_freq, F32, "inv_freq")),
        inv_freq.shape[0] * 2, _ptr(_need(q_norm_w, BF16, "q_norm_w")), _ptr(_need(k_norm_w, BF16, "k_norm_w")), eps,
        Hq, Hkv, D, _ptr(q), _ptr(k), _ptr(v), _stream(qkv)), "attn_qk_prep")
    return q, k, v


def selftest_wait_timeout(device="cuda"):
    """Run the device-side wait self-test (a wait on a barrier phase nothing completes, bounded at ~1 s) and return
    the status word it set (1: the wait ran out and was reported)."""
    status = torch.zeros(1, dtype=I32, device=device)
    _lib.check(_lib.load().janus_b200_selftest_wait_timeout(_ptr(status), _stream(status)), "selftest_wait_timeout")
    return int(status.item())


def tree_attention_tile_tokens(D, Hq, Hkv):
    """Query tokens per attention tile the library accepts for this layout."""
    n = _lib.load().janus_b200_tree_attention_tile_tokens(D, Hq, Hkv)
    if n <= 0:
        raise ValueError(f"tree_attention: no kernel for D={D}, Hq={Hq}, Hkv={Hkv}")
    return n


@_instrument("tree_attention", 1)
def tree_attention(q, keys, values, anc_lo, anc_hi, row_start, row_of_token, tiles, gate, scale, out=None,
                   status=None):
    """q bf16 [T, Hq, D]; keys/values: per level [T_l, Hkv, D] (last = own); anc_lo/anc_hi: per ancestor level
    int32 [B]; tiles int32 [n, 2]; gate: bf16 view [T, Hq, D] (any strides with unit last stride)."""
    _need(q, BF16, "q")
    T, Hq, D = q.shape
    Hkv = keys[-1].shape[1]
    n = len(keys)
    if len(values) != n or len(anc_lo) != n - 1 or len(anc_hi) != n - 1:
        raise ValueError("tree_attention: one key/value array per level and one range pair per ancestor level")
    for t in (*keys, *values):
        _need(t, BF16, "keys/values")
    for t in (*anc_lo, *anc_hi):
        _need(t, I32, "ancestor ranges")
    _need(gate, BF16, "gate", contiguous=False)
    if gate.stride(2) != 1:
        raise ValueError("gate must have unit last stride")
    out = torch.empty(T, Hq * D, dtype=BF16, device=q.device) if out is None else out
    arr = lambda ts: (ctypes.c_void_p * max(1, len(ts)))(*[t.data_ptr() for t in ts])
    for t in (*keys, *values):
        if t.dim() != 3 or t.shape[1:] != (Hkv, D) or not t.is_contiguous():
            raise ValueError("tree_attention: keys/values must be contiguous [T_l, Hkv, D]")
    if any(k.shape[0] != v.shape[0] for k, v in zip(keys, values)) or keys[-1].shape[0] != T:
        raise ValueError("tree_attention: per-level key and value counts differ, or the own level is not T tokens")
    karr, varr, larr, harr = arr(keys), arr(values), arr(anc_lo), arr(anc_hi)
    counts = (ctypes.c_int64 * n)(*[k.shape[0] for k in keys])
    _lib.check(_lib.load().janus_b200_tree_attention(
        _ptr(q), T, Hq, Hkv, D, n, ctypes.cast(karr, ctypes.c_void_p), ctypes.cast(varr, ctypes.c_void_p),
        ctypes.cast(counts, ctypes.c_void_p), ctypes.cast(larr, ctypes.c_void_p), ctypes.cast(harr, ctypes.c_void_p),
        _ptr(_need(row_start, I32, "row_start")),
        _ptr(_need(row_of_token, I32, "row_of_token")), _ptr(_need(tiles, I32, "tiles")), tiles.shape[0], _ptr(gate),
        gate.stride(0), gate.stride(1), scale, _ptr(out), _ptr(status), _stream(q)), "tree_attention")
    return out


@_instrument("head_scalar", 1)
def head_scalar(x, rows, final_w, rms_eps, ln_w, ln_b, ln_eps, w_out, b_out, logits=None):
    _need(x, F32, "x"); _need(rows, I32, "rows")
    n = rows.shape[0]
    logits = torch.empty(n, dtype=F32, device=x.device) if logits is None else logits
    _lib.check(_lib.load().janus_b200_head_scalar(_ptr(x), x.shape[1], _ptr(rows), n, _ptr(_opt(final_w, BF16, "final_w")),
                                                  rms_eps, _ptr(_need(ln_w, F32, "ln_w")), _ptr(_need(ln_b, F32, "ln_b")),
                                                  ln_eps, _ptr(_need(w_out, F32, "w_out")), _ptr(_need(b_out, F32, "b_out")),
                                                  _ptr(logits), _stream(x)), "head_scalar")
    return logits


@_instrument("head_pointer", 2)
def head_pointer(x, option_rows, option_question, decision_rows, final_w, rms_eps, ln_w, ln_b, ln_eps, wq, wk,
                 logits=None, workspace=None):
    _need(x, F32, "x")
    n, Q, R = option_rows.shape[0], decision_rows.shape[0], wq.shape[0]
    logits = torch.empty(n, dtype=F32, device=x.device) if logits is None else logits
    workspace = torch.empty((n + Q) * R, dtype=F32, device=x.device) if workspace is None else workspace
    _lib.check(_lib.load().janus_b200_head_pointer(
        _ptr(x), x.shape[1], _ptr(_need(option_rows, I32, "option_rows")), _ptr(_need(option_question, I32, "option_question")),
        n, _ptr(_need(decision_rows, I32, "decision_rows")), Q, _ptr(_opt(final_w, BF16, "final_w")), rms_eps,
        _ptr(_need(ln_w, F32, "ln_w")), _ptr(_need(ln_b, F32, "ln_b")), ln_eps, _ptr(_need(wq, F32, "wq")),
        _ptr(_need(wk, F32, "wk")), R, _ptr(workspace), workspace.numel() * 4, _ptr(logits), _stream(x)), "head_pointer")
    return logits


@_instrument("gemm_bf16", 1)
def gemm_bf16(a, w, swiglu=False, out=None, status=None):
    """a bf16 [M, K] (unit column stride), w bf16 [N, K] -> a w^T bf16 [M, N] on the tcgen05 GEMM; swiglu: w in
    the interleaved gate/up order of `swiglu_weight`, result silu(gate) * up [M, N / 2]."""
    _need(a, BF16, "a", contiguous=False)
    _need(w, BF16, "w", contiguous=False)
    if a.stride(1) != 1 or w.stride(1) != 1:
        raise ValueError("gemm_bf16: a and w need unit column stride")
    M, K = a.shape
    N = w.shape[0]
    if w.shape[1] != K:
        raise ValueError(f"gemm_bf16: a has K = {K}, w has {w.shape[1]}")
    n_out = N // 2 if swiglu else N
    FLOPS["gemm_bf16"] = FLOPS.get("gemm_bf16", 0.0) + 2.0 * M * N * K
    out = torch.empty(M, n_out, dtype=BF16, device=a.device) if out is None else out
    _need(out, BF16, "out", contiguous=False)
    _lib.check(_lib.load().janus_b200_gemm_bf16(_ptr(a), a.stride(0), _ptr(w), w.stride(0), M, N, K, int(bool(swiglu)),
                                                _ptr(out), out.stride(0), _ptr(status), _stream(a)), "gemm_bf16")
    return out


def swiglu_weight(gate, up):
    """The gate/up weight in the order the SwiGLU epilogue reads: 256-row blocks of 128 gate rows followed by the
    128 matching up rows. gate, up [I, H] with I a multiple of 128 -> [2I, H]."""
    I, H = gate.shape
    if up.shape != gate.shape or I % 128:
        raise ValueError("swiglu_weight: gate and up [I, H] with I a multiple of 128")
    return torch.stack([gate.reshape(I // 128, 128, H), up.reshape(I // 128, 128, H)], 1).reshape(2 * I, H).contiguous()


MOE_TILE = 128  # rows per tile of the routing plan = the M of the grouped GEMMs' tensor-core tiles


def moe_max_tiles(S, E, k):
    return (S * k + E * (MOE_TILE - 1) + MOE_TILE - 1) // MOE_TILE


@_instrument("moe_route", 4)
def moe_route(logits, k):
    """fp32 router logits [S, E] -> (topk_idx, topk_w, sorted_ids, tile_expert, n_tiles) on the device."""
    _need(logits, F32, "logits")
    S, E = logits.shape
    dev = logits.device
    mt = moe_max_tiles(S, E, k)
    topk_idx = torch.empty(S, k, dtype=I32, device=dev)
    topk_w = torch.empty(S, k, dtype=F32, device=dev)
    sorted_ids = torch.empty(mt * MOE_TILE, dtype=I32, device=dev)
    tile_expert = torch.empty(mt, dtype=I32, device=dev)
    n_tiles = torch.empty(1, dtype=I32, device=dev)
    ws = torch.empty(3 * E, dtype=I32, device=dev)
    _lib.check(_lib.load().janus_b200_moe_route(_ptr(logits), S, E, k, MOE_TILE, _ptr(topk_idx), _ptr(topk_w),
                                                _ptr(sorted_ids), _ptr(tile_expert), mt, _ptr(n_tiles), _ptr(ws),
                                                ws.numel() * 4, _stream(logits)), "moe_route")
    return topk_idx, topk_w, sorted_ids, tile_expert, n_tiles


@_instrument("moe_route_fused", 4)
def moe_route_fused(x, w_router, k, w_gate=None, status=None):
    """The router GEMM fused with the routing: x bf16 [S, H] (unit column stride), w_router bf16 [E, H] (E <= 256),
    optional w_gate bf16 [1, H] (the shared expert's gate row) -> ((topk_idx, topk_w, sorted_ids, tile_expert,
    n_tiles), gate_logit fp32 [S] or None), the router logits never leaving the tensor memory."""
    _need(x, BF16, "x", contiguous=False)
    if x.stride(1) != 1:
        raise ValueError("x must have unit column stride")
    _need(w_router, BF16, "w_router")
    S, H = x.shape
    E = w_router.shape[0]
    if w_router.shape[1] != H or (w_gate is not None and tuple(w_gate.shape) != (1, H)):
        raise ValueError("moe_route_fused: w_router [E, H] and w_gate [1, H] must match x [S, H]")
    dev = x.device
    mt = moe_max_tiles(S, E, k)
    topk_idx = torch.empty(S, k, dtype=I32, device=dev)
    topk_w = torch.empty(S, k, dtype=F32, device=dev)
    sorted_ids = torch.empty(mt * MOE_TILE, dtype=I32, device=dev)
    tile_expert = torch.empty(mt, dtype=I32, device=dev)
    n_tiles = torch.empty(1, dtype=I32, device=dev)
    gate = torch.empty(S, dtype=F32, device=dev) if w_gate is not None else None
    ws = torch.empty(3 * E, dtype=I32, device=dev)
    _lib.check(_lib.load().janus_b200_moe_route_fused(
        _ptr(x), x.stride(0), S, H, _ptr(w_router), E, _ptr(_opt(w_gate, BF16, "w_gate")), k, MOE_TILE, _ptr(topk_idx),
        _ptr(topk_w), _ptr(gate), _ptr(sorted_ids), _ptr(tile_expert), mt, _ptr(n_tiles), _ptr(ws), ws.numel() * 4,
        _ptr(status), _stream(x)), "moe_route_fused")
    return (topk_idx, topk_w, sorted_ids, tile_expert, n_tiles), gate


@_instrument("moe_grouped_w4a16", 1)
def moe_grouped_w4a16(x, codes, scales, plan, gated, k, topk_w=None, out=None, status=None):
    """x bf16 [rows, K] (unit column stride); codes uint8 [E, NW, K/2], scales bf16 [E, NW, K/128] (NW = 2N gated).
    status: optional device int32 [1], zero on entry, set to 1 by a device-side wait that ran out."""
    _need(x, BF16, "x", contiguous=False)
    if x.stride(1) != 1:
        raise ValueError("x must have unit column stride")
    _need(codes, torch.uint8, "codes"); _need(scales, BF16, "scales")
    E, NW, half_k = codes.shape
    K = 2 * half_k
    N = NW // 2 if gated else NW
    topk_idx, _, sorted_ids, tile_expert, n_tiles = plan
    mt = tile_expert.shape[0]
    S = topk_idx.shape[0]
    if out is None:
        out = torch.empty((mt * MOE_TILE if gated else S * k), N, dtype=BF16, device=x.device)
    _lib.check(_lib.load().janus_b200_moe_grouped_w4a16(
        _ptr(x), x.stride(0), _ptr(codes), _ptr(scales), E, N, K, 1 if gated else 0, _ptr(sorted_ids),
        _ptr(tile_expert), _ptr(n_tiles), mt, k, _ptr(topk_w), _ptr(out), out.stride(0), _ptr(status), _stream(x)),
        "moe_grouped_w4a16")
    return out


@_instrument("moe_grouped_nvfp4", 1)
def moe_grouped_nvfp4(x, codes, block_scales, global_scales, plan, gated, k, topk_w=None, out=None, status=None):
    """moe_grouped_w4a16 on NVFP4 experts: codes uint8 [E, NW, K/2] (e2m1 pairs), block_scales e4m3 [E, NW, K/16]
    (torch.float8_e4m3fn or its uint8 bytes), global_scales fp32 [E, NW] (one per weight row)."""
    _need(x, BF16, "x", contiguous=False)
    if x.stride(1) != 1:
        raise ValueError("x must have unit column stride")
    _need(codes, torch.uint8, "codes")
    if block_scales.dtype == torch.float8_e4m3fn:
        block_scales = block_scales.view(torch.uint8)
    _need(block_scales, torch.uint8, "block_scales"); _need(global_scales, F32, "global_scales")
    E, NW, half_k = codes.shape
    K = 2 * half_k
    if block_scales.shape != (E, NW, K // 16) or global_scales.shape != (E, NW):
        raise ValueError("moe_grouped_nvfp4: block_scales [E, NW, K/16] and global_scales [E, NW]")
    N = NW // 2 if gated else NW
    topk_idx, _, sorted_ids, tile_expert, n_tiles = plan
    mt = tile_expert.shape[0]
    S = topk_idx.shape[0]
    if out is None:
        out = torch.empty((mt * MOE_TILE if gated else S * k), N, dtype=BF16, device=x.device)
    _lib.check(_lib.load().janus_b200_moe_grouped_nvfp4(
        _ptr(x), x.stride(0), _ptr(codes), _ptr(block_scales), _ptr(global_scales), E, N, K, 1 if gated else 0,
        _ptr(sorted_ids), _ptr(tile_expert), _ptr(n_tiles), mt, k, _ptr(topk_w), _ptr(out), out.stride(0),
        _ptr(status), _stream(x)), "moe_grouped_nvfp4")
    return out


@_instrument("moe_combine", 1)
def moe_combine(y, k, shared, shared_gate_logit, out=None):
    _need(y, BF16, "y")
    S = y.shape[0] // k
    H = y.shape[1]
    out = torch.empty(S, H, dtype=BF16, device=y.device) if out is None else out
    if shared is not None:
        _need(shared, BF16, "shared"); _need(shared_gate_logit, F32, "shared_gate_logit")
    _lib.check(_lib.load().janus_b200_moe_combine(_ptr(y), k, _ptr(shared), _ptr(shared_gate_logit), S, H, _ptr(out),
                                                  _stream(y)), "moe_combine")
    return out


# ------------------------------------------------------------------------------------------ expert parallel

@_instrument("moe_plan", 4)
def moe_plan(slot_expert, E):
    """Tile plan from explicit slot -> local expert ids (int32 [R, k], negative = no expert on this rank):
    (slot_expert, None, sorted_ids, tile_expert, n_tiles), the structure moe_grouped_w4a16 takes."""
    _need(slot_expert, I32, "slot_expert")
    R, k = slot_expert.shape
    dev = slot_expert.device
    mt = moe_max_tiles(R, E, k)
    sorted_ids = torch.empty(mt * MOE_TILE, dtype=I32, device=dev)
    tile_expert = torch.empty(mt, dtype=I32, device=dev)
    n_tiles = torch.empty(1, dtype=I32, device=dev)
    ws = torch.empty(3 * E, dtype=I32, device=dev)
    _lib.check(_lib.load().janus_b200_moe_plan(_ptr(slot_expert), R * k, E, MOE_TILE, _ptr(sorted_ids),
                                               _ptr(tile_expert), mt, _ptr(n_tiles), _ptr(ws), ws.numel() * 4,
                                               _stream(slot_expert)), "moe_plan")
    return slot_expert, None, sorted_ids, tile_expert, n_tiles


@_instrument("moe_reduce_slots", 1)
def moe_reduce_slots(y, k, slot_expert, out=None):
    """fp32 [R, H]: per row the sum of its slots' expert outputs (bf16 [R*k, H]) that have an expert here."""
    _need(y, BF16, "y")
    R, H = y.shape[0] // k, y.shape[1]
    out = torch.empty(R, H, dtype=F32, device=y.device) if out is None else out
    if slot_expert is not None:
        _need(slot_expert, I32, "slot_expert")
    _lib.check(_lib.load().janus_b200_moe_reduce_slots(_ptr(y), k, _ptr(slot_expert), R, H, _ptr(out), _stream(y)),
               "moe_reduce_slots")
    return out


@_instrument("moe_combine_ep", 1)
def moe_combine_ep(partials, row_index, shared, shared_gate_logit, out=None):
    """bf16 [S, H] = sum over ranks of the partial rows row_index [S, W] (-1: none) + sigmoid(gate) * shared."""
    _need(partials, F32, "partials"); _need(row_index, I32, "row_index")
    S, W = row_index.shape
    H = partials.shape[1]
    out = torch.empty(S, H, dtype=BF16, device=row_index.device) if out is None else out
    if shared is not None:
        _need(shared, BF16, "shared"); _need(shared_gate_logit, F32, "shared_gate_logit")
    _lib.check(_lib.load().janus_b200_moe_combine_ep(_ptr(partials), _ptr(row_index), W, _ptr(shared),
                                                     _ptr(shared_gate_logit), S, H, _ptr(out), _stream(row_index)),
               "moe_combine_ep")
    return out
