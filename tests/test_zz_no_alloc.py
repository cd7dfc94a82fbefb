"""The allocation-free PointerHead entry point (janus_b200_head_pointer_noalloc), called through the C ABI.

Some callers cannot allocate device memory on the request path: a host runtime that binds this library over
FFI without a device allocator of its own, or a serving loop that must not call cudaMalloc while work is queued
(cudaMalloc can synchronise the device). This entry point takes no workspace and uses a static device array instead.
The test checks it against the workspace entry point on the same inputs, twice in a row (the static array keeps the
previous call's contents), and that a call larger than the array is rejected before any launch. It sits in a file
collected last so a stop at the first failure has already run every other test; it also passes alone."""

import ctypes

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu
P = lambda t: ctypes.c_void_p(t.data_ptr())


def _inputs(seed, n_opts, n_dec, H=1024, R=128, T=64):
    g = torch.Generator().manual_seed(seed)
    x = torch.randn(T, H, generator=g) * 2
    fw = (0.1 * torch.randn(H, generator=g)).to(torch.bfloat16)
    lw, lb = 1 + 0.1 * torch.randn(H, generator=g), 0.1 * torch.randn(H, generator=g)
    wq, wk = 0.02 * torch.randn(R, H, generator=g), 0.02 * torch.randn(R, H, generator=g)
    orows = torch.randint(0, T, (n_opts,), generator=g, dtype=torch.int32)
    oq = torch.randint(0, n_dec, (n_opts,), generator=g, dtype=torch.int32)
    drows = torch.randint(0, T, (n_dec,), generator=g, dtype=torch.int32)
    return [t.cuda() for t in (x, orows, oq, drows, fw, lw, lb, wq, wk)]


def _call(lib, noalloc, x, orows, oq, drows, fw, lw, lb, wq, wk):
    n, Q, R, H = orows.shape[0], drows.shape[0], wq.shape[0], x.shape[1]
    logits = torch.full((n,), float("nan"), device="cuda")
    stream = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    if noalloc:
        st = lib.janus_b200_head_pointer_noalloc(P(x), H, P(orows), P(oq), n, P(drows), Q, P(fw), 1e-6, P(lw), P(lb),
                                                 1e-5, P(wq), P(wk), R, P(logits), stream)
    else:
        ws = torch.empty((n + Q) * R, device="cuda")
        st = lib.janus_b200_head_pointer(P(x), H, P(orows), P(oq), n, P(drows), Q, P(fw), 1e-6, P(lw), P(lb), 1e-5,
                                         P(wq), P(wk), R, P(ws), ws.numel() * 4, P(logits), stream)
    return st, logits


def test_noalloc_pointer_head_matches_workspace_entry_point_twice():
    from janus_b200 import _lib
    lib = _lib.load()
    for seed, (n, q) in enumerate([(300, 40), (37, 5)]):  # the second call is smaller: stale rows must not leak in
        args = _inputs(seed, n, q)
        st_ref, ref = _call(lib, False, *args)
        st, got = _call(lib, True, *args)
        torch.cuda.synchronize()
        assert st_ref == 0 and st == 0, _lib.last_error()
        np.testing.assert_allclose(got.cpu().numpy(), ref.cpu().numpy(), atol=2e-4, rtol=2e-4)


def test_noalloc_rejects_calls_beyond_its_static_scratch():
    from janus_b200 import _lib
    lib = _lib.load()
    args = _inputs(9, 2100, 8)  # (2100 + 8) * 128 floats > 262144
    st, logits = _call(lib, True, *args)
    assert st == -4
    assert "static scratch" in _lib.last_error()
    assert torch.isnan(logits).all()  # nothing launched
