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


def test_every_op_the_readout_calls_is_wrapped():
    """janus_b200.model only calls ops that janus_b200.ops defines (a CPU check of the host path's wiring)."""
    from janus_b200 import ops
    used = set(re.findall(r"\bops\.(\w+)\(", (ROOT / "janus_b200" / "model.py").read_text()))
    assert used and all(callable(getattr(ops, n, None)) for n in used), used - set(dir(ops))
