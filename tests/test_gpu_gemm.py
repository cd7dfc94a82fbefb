"""The tcgen05 dense GEMM (janus_b200_gemm_bf16) against a torch fp32 matmul of the same bf16 operands.

bf16 output, one rounding of an fp32 accumulation: within 2^-7 relative (one bf16 unit in the last place) plus a
small absolute term for fp32 accumulation-order differences on O(1) results. Shapes cover the model's projections
(N = 12352 is not a multiple of the 256-column tile), ragged M and K, and the SwiGLU epilogue."""

import pytest
import torch

pytestmark = pytest.mark.gpu
BF = torch.bfloat16


def _ref(a, w):
    return a.float() @ w.float().t()


def _close(got, want):
    err = (got.float() - want).abs()
    lim = 2.0 ** -7 * want.abs() + 2e-3
    assert bool((err <= lim).all()), f"max err {float(err.max()):.3e}, worst ratio {float((err / lim).max()):.2f}"


@pytest.mark.parametrize("M,N,K", [(300, 512, 256), (1000, 12352, 2560), (129, 2560, 4096), (64, 256, 136),
                                   (2048, 10240, 2560)])
def test_gemm_plain(M, N, K):
    from janus_b200 import ops
    g = torch.Generator(device="cuda").manual_seed(M + N + K)
    a = torch.randn(M, K, generator=g, device="cuda").to(BF)
    w = (torch.randn(N, K, generator=g, device="cuda") * 0.02).to(BF)
    status = torch.zeros(1, dtype=torch.int32, device="cuda")
    out = ops.gemm_bf16(a, w, status=status)
    torch.cuda.synchronize()
    assert int(status.item()) == 0 and out.shape == (M, N)
    _close(out, _ref(a, w))
    assert torch.equal(ops.gemm_bf16(a, w), out)  # fixed accumulation order: run to run identical


def test_gemm_strided_operands():
    """A row-strided view of a wider activation (the merged projection's column slices) and an output view."""
    from janus_b200 import ops
    g = torch.Generator(device="cuda").manual_seed(5)
    big = torch.randn(777, 4096 + 64, generator=g, device="cuda").to(BF)
    a = big[:, 64:]
    w = (torch.randn(384, 4096, generator=g, device="cuda") * 0.02).to(BF)
    out_buf = torch.zeros(777, 512, dtype=BF, device="cuda")
    ops.gemm_bf16(a, w, out=out_buf[:, 64:448])
    _close(out_buf[:, 64:448], _ref(a, w))
    assert bool((out_buf[:, :64] == 0).all()) and bool((out_buf[:, 448:] == 0).all())


@pytest.mark.parametrize("M,I,K", [(1000, 9216, 2560), (77, 512, 1024)])
def test_gemm_swiglu(M, I, K):
    from janus_b200 import ops
    g = torch.Generator(device="cuda").manual_seed(M + I)
    a = torch.randn(M, K, generator=g, device="cuda").to(BF)
    gate = (torch.randn(I, K, generator=g, device="cuda") * 0.02).to(BF)
    up = (torch.randn(I, K, generator=g, device="cuda") * 0.02).to(BF)
    w = ops.swiglu_weight(gate, up)
    out = ops.gemm_bf16(a, w, swiglu=True)
    assert out.shape == (M, I)
    want = torch.nn.functional.silu(_ref(a, gate)) * _ref(a, up)
    _close(out, want)


@pytest.mark.parametrize("M,N,K,swiglu", [(5000, 12352, 2560, False), (16384, 2560, 1024, False),
                                          (3000, 1024, 2560, True), (100, 768, 512, False)])
def test_gemm_tall_and_pair_tiles_agree(M, N, K, swiglu, monkeypatch):
    """The tall-tile form (512 x 256 per CTA pair, the default) and the 256 x 256 form (JANUS_B200_GEMM=pair) issue
    the same MMAs in the same k order for every output element: bit-identical results, several items per pair."""
    from janus_b200 import ops
    g = torch.Generator(device="cuda").manual_seed(M + N)
    a = torch.randn(M, K, generator=g, device="cuda").to(BF)
    w = (torch.randn(N, K, generator=g, device="cuda") * 0.02).to(BF)
    if swiglu:
        w = ops.swiglu_weight(w[:N // 2], w[N // 2:])
    status = torch.zeros(1, dtype=torch.int32, device="cuda")
    monkeypatch.delenv("JANUS_B200_GEMM", raising=False)
    tall = ops.gemm_bf16(a, w, swiglu=swiglu, status=status)
    monkeypatch.setenv("JANUS_B200_GEMM", "pair")
    pair = ops.gemm_bf16(a, w, swiglu=swiglu, status=status)
    torch.cuda.synchronize()
    assert int(status.item()) == 0
    assert torch.equal(tall, pair)
    if not swiglu:
        _close(tall, _ref(a, w))
