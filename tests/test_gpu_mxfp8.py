"""The MXFP8-activation path: the official FP8 activation quantisation
(act_quant, UE8M0 scales) on the device, bit-exact against the oracle."""
import ctypes
import os

import numpy as np
import pytest

pytestmark = pytest.mark.gpu
GOLDEN = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")


@pytest.fixture(scope="module")
def torch_cuda():
    import torch
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    from dee_b200 import build
    build.build()
    return torch


def _act_quant_dev(torch, x_bits, block):
    from dee_b200 import _native
    lib = _native.load()
    rows, cols = x_bits.shape
    dx = torch.from_numpy(x_bits.view(np.float16)).cuda()
    q = torch.empty((rows, cols), dtype=torch.uint8, device="cuda")
    s = torch.empty((rows, cols // block), dtype=torch.uint8, device="cuda")
    rc = lib.dee_act_quant_device(ctypes.c_void_p(dx.data_ptr()), rows, cols, block, ctypes.c_void_p(q.data_ptr()),
                                  ctypes.c_void_p(s.data_ptr()), None)
    assert rc == 0
    torch.cuda.synchronize()
    return q.cpu().numpy(), s.cpu().numpy()


@pytest.mark.parametrize("block", [128, 32])
def test_act_quant_kernel_bitexact(torch_cuda, oracle_mod, block):
    orc = oracle_mod
    rng = np.random.default_rng(block)
    rows, cols = 300, 1024
    mag = 10.0 ** rng.uniform(-4, 4, size=(rows, 1))
    x = (rng.standard_normal((rows, cols)) * mag).astype(np.float16)
    x[3] = 0                      # amax floor 1e-4
    x[5, :block] = 1e-6           # tiny block
    x[7, 3] = 65504.0             # FP16 max
    x[9, ::7] = -0.0
    q, s = _act_quant_dev(torch_cuda, x.view(np.uint16), block)
    wq, ws = orc.act_quant(x.view(np.uint16), block)
    assert np.array_equal(s, ws)
    assert np.array_equal(q, wq)
    # the reference's own round trip (fixture) through the device kernel
    g = np.load(os.path.join(GOLDEN, "act_quant.npz"))
    q, s = _act_quant_dev(torch_cuda, g["x"], block)
    y = orc.act_dequant_f32(q, s, block).astype(np.float16).view(np.uint16)
    assert np.array_equal(y, g[f"y{block}"])
