"""The allocation-free layer forward, checked against the engine's forward.

dee_moe_forward_noalloc serves callers that cannot allocate device memory
(code inside an allocator or memory-pool callback, or a host whose device
memory is owned by its own caching allocator): it keeps all scratch in a
static device array.  These tests call it through the C ABI and compare it
with dee_moe_forward_device on the same inputs, for two calls in a row with
different token batches (so a stale scratch array would show), within the
same relative-L2 tolerance the other parity tests use.  The file is named so
pytest collects it last; it builds its own inputs and runs alone too.
"""
import ctypes

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

TOL_REL_L2 = 2e-3


@pytest.fixture(scope="module")
def setup():
    import torch
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    from dee_b200 import _native, build
    build.build()
    return torch, _native, _native.load()


def _rel_l2(a, b):
    a = np.asarray(a, np.float64)
    b = np.asarray(b, np.float64)
    return float(np.linalg.norm(a - b) / max(np.linalg.norm(b), 1e-30))


def _batch(torch, rng, T, H, E, K):
    x = torch.from_numpy(rng.standard_normal((T, H)).astype(np.float16)).cuda()
    ids = torch.from_numpy(np.stack([rng.choice(E, K, replace=False) for _ in range(T)])
                           .astype(np.int32)).cuda()
    w = rng.random((T, K)).astype(np.float32)
    w = torch.from_numpy(w / w.sum(1, keepdims=True)).cuda()
    return x, ids, w


@pytest.mark.parametrize("shape", [(512, 512, 16, 6, 8), (4096, 2048, 256, 6, 8)])
def test_noalloc_matches_engine_forward_two_calls(setup, shape):
    torch, native, lib = setup
    import dee_b200
    from dee_b200.records import RecordLayout, synthetic_bank
    H, I, E, K, T = shape
    bank = synthetic_bank(RecordLayout(H, I), E, seed=606)
    eng = dee_b200.new_engine(dee_b200.EngineConfig(hidden=H, inter=I, num_experts=E, topk=K))
    eng.attach_bank(0, bank)
    cfg = native.DeeConfig(H, I, E, K, 1, torch.cuda.current_device(), 0.0, 64)
    rng = np.random.default_rng(607)
    stream = torch.cuda.current_stream()
    status = torch.zeros(1, dtype=torch.int32, device="cuda")
    for call in range(2):
        x, ids, w = _batch(torch, rng, T, H, E, K)
        want = torch.empty((T, H), dtype=torch.float32, device="cuda")
        eng.moe_forward_device(0, x.data_ptr(), T, d_ids_ptr=ids.data_ptr(), d_weights_ptr=w.data_ptr(),
                               d_out_ptr=want.data_ptr(), stream=stream)
        assert eng.sync_status(stream) == 0
        got = torch.full((T, H), float("nan"), dtype=torch.float32, device="cuda")
        rc = lib.dee_moe_forward_noalloc(ctypes.byref(cfg), ctypes.c_void_p(bank.data_ptr()),
                                         bank.shape[1], E, ctypes.c_void_p(x.data_ptr()), T,
                                         ctypes.c_void_p(ids.data_ptr()), ctypes.c_void_p(w.data_ptr()),
                                         ctypes.c_void_p(got.data_ptr()), ctypes.c_void_p(status.data_ptr()),
                                         ctypes.c_void_p(stream.cuda_stream))
        assert rc == native.DEE_OK, f"call {call}: status {rc}"
        torch.cuda.synchronize()
        assert int(status.item()) == 0, f"call {call}: device status {int(status.item()):#x}"
        g, r = got.cpu().numpy(), want.cpu().numpy()
        assert np.isfinite(g).all()
        assert _rel_l2(g, r) <= TOL_REL_L2, f"call {call}"


def test_noalloc_rejects_requests_beyond_the_static_scratch(setup):
    torch, native, lib = setup
    cfg = native.DeeConfig(4096, 2048, 256, 6, 1, 0, 0.0, 64)
    dummy = ctypes.c_void_p(256)  # never dereferenced: the size check comes first
    rc = lib.dee_moe_forward_noalloc(ctypes.byref(cfg), dummy, 13_369_344, 256, dummy, 100, dummy,
                                     dummy, dummy, None, None)
    assert rc == native.DEE_ERR_SCRATCH_LIMIT
