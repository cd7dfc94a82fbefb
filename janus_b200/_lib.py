"""ctypes binding of libjanus_b200.so (include/janus_b200.h). The library is built in-tree by janus_b200.build;
there is no fallback: importing an op without the library raises."""

import ctypes
from ctypes import c_float, c_int32, c_int64, c_size_t, c_void_p
from pathlib import Path

LIB_PATH = Path(__file__).resolve().parent / "libjanus_b200.so"

# name: argtypes (all return int status)
SIGNATURES = {
    "janus_b200_version": [],
    "janus_b200_last_error": [c_void_p, c_size_t],
    "janus_b200_embed_rmsnorm": [c_void_p, c_int64, c_int64, c_void_p, c_int64, c_void_p, c_float, c_void_p, c_void_p,
                                 c_void_p],
    "janus_b200_add_rmsnorm": [c_void_p, c_void_p, c_int64, c_int64, c_int64, c_void_p, c_float, c_void_p, c_void_p],
    "janus_b200_silu_mul": [c_void_p, c_int64, c_int64, c_void_p, c_void_p],
    "janus_b200_gated_rmsnorm": [c_void_p, c_void_p, c_int64, c_int64, c_int64, c_int64, c_void_p, c_float, c_void_p,
                                 c_void_p],
    "janus_b200_gdn_prologue": [c_void_p, c_int64, c_int64, c_int64, c_void_p, c_void_p, c_void_p, c_void_p, c_void_p,
                                c_void_p, c_void_p, c_void_p, c_int64, c_int64, c_int64, c_int64, c_int64, c_void_p,
                                c_void_p, c_void_p, c_void_p, c_void_p, c_void_p],
    "janus_b200_gdn_fork_recurrent": [c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_int64, c_int64, c_void_p,
                                      c_void_p, c_int64, c_void_p, c_void_p, c_int64, c_int64, c_int64, c_int64,
                                      c_float, c_void_p, c_void_p],
    "janus_b200_gdn_chunk_scan": [c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_int64, c_int64, c_void_p,
                                  c_void_p, c_int64, c_void_p, c_void_p, c_void_p, c_void_p, c_int64, c_int64, c_int64,
                                  c_int64, c_float, c_void_p, c_size_t, c_void_p, c_void_p, c_void_p],
    "janus_b200_gdn_chunk_scan_workspace": [c_int64, c_int64, c_int64],
    "janus_b200_gdn_chunk_scan_fused": [c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_int64, c_int64, c_void_p,
                                        c_void_p, c_int64, c_void_p, c_void_p, c_void_p, c_int64, c_int64, c_int64,
                                        c_int64, c_float, c_void_p, c_void_p, c_void_p],
    "janus_b200_attn_qk_prep": [c_void_p, c_int64, c_int64, c_void_p, c_void_p, c_int64, c_void_p, c_void_p, c_float,
                                c_int64, c_int64, c_int64, c_void_p, c_void_p, c_void_p, c_void_p],
    "janus_b200_tree_attention": [c_void_p, c_int64, c_int64, c_int64, c_int64, c_int32, c_void_p, c_void_p, c_void_p,
                                  c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_int64, c_void_p, c_int64, c_int64, c_float,
                                  c_void_p, c_void_p, c_void_p],
    "janus_b200_tree_attention_tile_tokens": [c_int64, c_int64, c_int64],
    "janus_b200_selftest_wait_timeout": [c_void_p, c_void_p],
    "janus_b200_head_scalar": [c_void_p, c_int64, c_void_p, c_int64, c_void_p, c_float, c_void_p, c_void_p, c_float,
                               c_void_p, c_void_p, c_void_p, c_void_p],
    "janus_b200_head_pointer": [c_void_p, c_int64, c_void_p, c_void_p, c_int64, c_void_p, c_int64, c_void_p, c_float,
                                c_void_p, c_void_p, c_float, c_void_p, c_void_p, c_int64, c_void_p, c_size_t,
                                c_void_p, c_void_p],
    "janus_b200_moe_route": [c_void_p, c_int64, c_int64, c_int64, c_int64, c_void_p, c_void_p, c_void_p, c_void_p,
                             c_int64, c_void_p, c_void_p, c_size_t, c_void_p],
    "janus_b200_moe_route_fused": [c_void_p, c_int64, c_int64, c_int64, c_void_p, c_int64, c_void_p, c_int64, c_int64,
                                   c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_int64, c_void_p, c_void_p,
                                   c_size_t, c_void_p, c_void_p],
    "janus_b200_moe_grouped_w4a16": [c_void_p, c_int64, c_void_p, c_void_p, c_int64, c_int64, c_int64, c_int32,
                                     c_void_p, c_void_p, c_void_p, c_int64, c_int64, c_void_p, c_void_p, c_int64,
                                     c_void_p, c_void_p],
    "janus_b200_gemm_bf16": [c_void_p, c_int64, c_void_p, c_int64, c_int64, c_int64, c_int64, c_int32, c_void_p,
                             c_int64, c_void_p, c_void_p],
    "janus_b200_moe_grouped_nvfp4": [c_void_p, c_int64, c_void_p, c_void_p, c_void_p, c_int64, c_int64, c_int64,
                                     c_int32, c_void_p, c_void_p, c_void_p, c_int64, c_int64, c_void_p, c_void_p,
                                     c_int64, c_void_p, c_void_p],
    "janus_b200_moe_combine": [c_void_p, c_int64, c_void_p, c_void_p, c_int64, c_int64, c_void_p, c_void_p],
    "janus_b200_moe_plan": [c_void_p, c_int64, c_int64, c_int64, c_void_p, c_void_p, c_int64, c_void_p, c_void_p,
                            c_size_t, c_void_p],
    "janus_b200_moe_reduce_slots": [c_void_p, c_int64, c_void_p, c_int64, c_int64, c_void_p, c_void_p],
    "janus_b200_moe_combine_ep": [c_void_p, c_void_p, c_int64, c_void_p, c_void_p, c_int64, c_int64, c_void_p,
                                  c_void_p],
    "janus_b200_head_pointer_noalloc": [c_void_p, c_int64, c_void_p, c_void_p, c_int64, c_void_p, c_int64, c_void_p,
                                        c_float, c_void_p, c_void_p, c_float, c_void_p, c_void_p, c_int64, c_void_p,
                                        c_void_p],
}

SIZE_RESULTS = {"janus_b200_gdn_chunk_scan_workspace"}  # entry points returning size_t

_LIB = None


def load(path=None):
    """The loaded library (cached). Raises OSError when it is missing: build it with `python -m janus_b200.build`."""
    global _LIB
    if _LIB is not None and path is None:
        return _LIB
    p = Path(path) if path else LIB_PATH
    if not p.exists():
        raise OSError(f"{p} is missing; build it with `python -m janus_b200.build` (nvcc, sm_100a)")
    lib = ctypes.CDLL(str(p))
    for name, args in SIGNATURES.items():
        fn = getattr(lib, name)
        fn.argtypes = args
        fn.restype = c_size_t if name in SIZE_RESULTS else c_int32
    if path is None:
        _LIB = lib
    return lib


def last_error():
    lib = load()
    buf = ctypes.create_string_buffer(1024)
    lib.janus_b200_last_error(ctypes.cast(buf, c_void_p), 1024)
    return buf.value.decode(errors="replace")


class JanusError(RuntimeError):
    """A CUDA launch or runtime failure reported by libjanus_b200 (status JANUS_ERR_CUDA / TIMEOUT)."""


STATUS = {0: "OK", -1: "INVALID", -2: "ALIGNMENT", -3: "UNSUPPORTED", -4: "WORKSPACE", -5: "CUDA", -6: "TIMEOUT"}


def check(status, what):
    """Maps a status to the reference's error convention: argument errors -> ValueError, the rest -> RuntimeError."""
    if status == 0:
        return
    msg = f"{what}: {STATUS.get(status, status)}: {last_error()}"
    if status in (-1, -2, -3, -4):
        raise ValueError(msg)
    raise JanusError(msg)
