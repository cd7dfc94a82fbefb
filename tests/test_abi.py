"""The C ABI library (no GPU needed): it loads, and it exports every function include/janus_b200.h declares."""

import re
from pathlib import Path

ROOT = Path(__file__).resolve().parent.parent


def declared():
    text = (ROOT / "include" / "janus_b200.h").read_text()
    return sorted(set(re.findall(r"\b(?:int|size_t)\s+(janus_b200_\w+)\s*\(", text)))


def test_library_exports_every_declared_symbol():
    from janus_b200 import _lib
    lib = _lib.load()
    names = declared()
    assert len(names) >= 10
    missing = [n for n in names if not hasattr(lib, n)]
    assert not missing, missing
    assert set(_lib.SIGNATURES) == set(names), set(names) ^ set(_lib.SIGNATURES)
    assert lib.janus_b200_version() >= 100


def test_argument_errors_need_no_gpu():
    from janus_b200 import _lib
    lib = _lib.load()
    st = lib.janus_b200_silu_mul(None, 4, 8, None, None)
    assert st == -1
    assert "silu_mul" in _lib.last_error()


def test_pointer_head_rejects_tables_it_cannot_serve():
    """Options without a question, an absurd rank and a row count beyond int range are refused before any launch
    (non-null placeholder pointers: nothing is dereferenced on the host, nothing reaches a device)."""
    import ctypes
    from janus_b200 import _lib
    lib = _lib.load()
    p = ctypes.c_void_p(16)
    for fn in (lib.janus_b200_head_pointer, lib.janus_b200_head_pointer_noalloc):
        ws = (p, 1 << 30) if fn is lib.janus_b200_head_pointer else ()
        for n, Q, R, what in ((5, 0, 128, "no question"), (5, 1, 1 << 40, "rank"), (1 << 40, 1, 128, "options")):
            st = fn(p, 1024, p, p, n, p, Q, p, 1e-6, p, p, 1e-5, p, p, R, *ws, p, None)
            assert st == -1, (fn, what)
            assert what in _lib.last_error(), _lib.last_error()


def test_every_op_the_readout_calls_is_wrapped():
    """janus_b200.model only calls ops that janus_b200.ops defines (a CPU check of the host path's wiring)."""
    from janus_b200 import ops
    used = set(re.findall(r"\bops\.(\w+)\(", (ROOT / "janus_b200" / "model.py").read_text()))
    assert used and all(callable(getattr(ops, n, None)) for n in used), used - set(dir(ops))


def test_gemm_rejects_shapes_and_layouts_it_cannot_serve():
    """The dense GEMM refuses an unknown epilogue, N or K off the tile granularity, a SwiGLU width that does not split
    into 128-row gate/up blocks, misaligned operands and an output stride too small, before any CUDA call
    (placeholder pointers: nothing is dereferenced on the host)."""
    import ctypes
    from janus_b200 import _lib
    lib = _lib.load()
    p = ctypes.c_void_p(256)
    odd = ctypes.c_void_p(258)
    cases = [  # a, lda, w, ldw, M, N, K, epilogue, out, ldo, expected words in the error
        (p, 64, p, 64, 128, 256, 64, 2, p, 256, "epilogue"),
        (p, 64, p, 64, 128, 200, 64, 0, p, 256, "multiple of 16"),
        (p, 60, p, 60, 128, 256, 60, 0, p, 256, "multiple of 16"),
        (p, 64, p, 64, 128, 384, 64, 1, p, 192, "256 for swiglu"),
        (odd, 64, p, 64, 128, 256, 64, 0, p, 256, "aligned"),
        (p, 64, p, 64, 128, 256, 64, 1, p, 64, "aligned"),
        (p, 64, p, 64, -1, 256, 64, 0, p, 256, "sizes"),
        (None, 64, p, 64, 128, 256, 64, 0, p, 256, "null"),
    ]
    for a, lda, w, ldw, M, N, K, ep, out, ldo, words in cases:
        st = lib.janus_b200_gemm_bf16(a, lda, w, ldw, M, N, K, ep, out, ldo, None, None)
        assert st < 0, (M, N, K, ep, ldo)
        assert words in _lib.last_error(), (words, _lib.last_error())


def test_swiglu_weight_interleaves_128_row_blocks():
    """The SwiGLU epilogue's weight order (host-side, no GPU): 256-row blocks of 128 gate rows then the matching 128
    up rows; widths that are not multiples of 128 are refused."""
    import pytest
    import torch
    from janus_b200 import ops
    I, H = 384, 8
    gate = torch.arange(I * H, dtype=torch.float32).reshape(I, H).to(torch.bfloat16)
    up = -gate - 1
    w = ops.swiglu_weight(gate, up)
    assert w.shape == (2 * I, H) and w.is_contiguous()
    for b in range(I // 128):
        assert torch.equal(w[256 * b:256 * b + 128], gate[128 * b:128 * (b + 1)])
        assert torch.equal(w[256 * b + 128:256 * (b + 1)], up[128 * b:128 * (b + 1)])
    with pytest.raises(ValueError):
        ops.swiglu_weight(gate[:200], up[:200])
