"""The NVFP4 expert codec against the reference's own (tests/golden/nvfp4.npz, written by make_golden.py --nvfp4 from
janus/hybrid.py:400-440): the synthetic quantiser (janus_b200.synthetic.nvfp4_quantize) reproduces its codes, block
scales and global scales, and the oracle's decode (the checker of the GPU kernel) its bf16 weights, bit for bit."""

import numpy as np
import torch

from janus_b200 import synthetic
from oracle import hybrid as oracle
from tests.golden_cases import GOLDEN


def test_nvfp4_codec_matches_the_reference_bit_for_bit():
    z = np.load(GOLDEN / "nvfp4.npz")
    w = torch.from_numpy(z["w"])
    codes, bs, gl = synthetic.nvfp4_quantize(w)
    for e in range(w.shape[0]):
        np.testing.assert_array_equal(codes[e].numpy(), z[f"codes{e}"])
        np.testing.assert_array_equal(bs[e].view(torch.uint8).numpy(), z[f"bscales{e}"])
        assert float(gl[e, 0]) == float(z[f"global{e}"]) and bool((gl[e] == gl[e, 0]).all())
        deq = oracle.nvfp4_dequantize(torch.from_numpy(z[f"codes{e}"]),
                                      torch.from_numpy(z[f"bscales{e}"]).view(torch.float8_e4m3fn), gl[e])
        np.testing.assert_array_equal(deq.float().numpy(), z[f"dequant{e}"])
    x = torch.from_numpy(z["enc_x"])
    np.testing.assert_array_equal(synthetic.e2m1_encode(x).numpy(), z["enc_codes"])


def test_gate_and_up_halves_get_their_own_global_scale():
    g = torch.Generator().manual_seed(3)
    w = torch.randn(2, 8, 64, generator=g) * 0.02
    w[:, 4:] *= 10.0
    _, _, gl = synthetic.nvfp4_quantize(w, [(0, 4), (4, 8)])
    assert bool((gl[:, :4] == gl[:, :1]).all()) and bool((gl[:, 4:] == gl[:, 4:5]).all())
    assert bool((gl[:, 4] > 5 * gl[:, 0]).all())
