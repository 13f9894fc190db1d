"""The allocation-free layer forward, checked against the engine's forward.

dee_moe_forward_noalloc serves callers that cannot allocate device memory
(code inside an allocator or memory-pool callback, or a host whose device
memory is owned by its own caching allocator): it keeps all scratch in a
static device array.  The GPU tests call it through the C ABI and compare it
with dee_moe_forward_device on the same inputs, for two calls in a row with
different token batches (so a stale scratch array would show).  Both entry
points run the same kernels on the same grouping, so the outputs must be
bit-identical; the relative-L2 bar of the other parity tests (2e-3) is only
reported in the failure message.  The cases cover the decode kernel (48
selections), the tcgen05 kernel (600 selections at a small shape), and the
edge of the static scratch at the DeepSeek-V4 shape (144 and 145 selections
run, 146 are refused).

The refusal tests need no GPU: every argument is checked on the host before
any CUDA call, so they also run in the CPU suite.  The file is named so
pytest collects it last; it builds its own inputs and runs alone too.
"""
import ctypes

import numpy as np
import pytest

TOL_REL_L2 = 2e-3
FULL = (4096, 2048, 256)   # H, I, E of the DeepSeek-V4 layer
RECORD_BYTES_FULL = 13_369_344


@pytest.fixture(scope="module")
def native_lib():
    from dee_b200 import _native, build
    build.build()
    return _native, _native.load()


@pytest.fixture(scope="module")
def setup(native_lib):
    import torch
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    native, lib = native_lib
    return torch, native, lib


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


_BANKS = {}


def _bank(H, I, E):
    from dee_b200.records import RecordLayout, synthetic_bank
    key = (H, I, E)
    if key not in _BANKS:
        _BANKS.clear()
        _BANKS[key] = synthetic_bank(RecordLayout(H, I), E, seed=606)
    return _BANKS[key]


# (H, I, E, K, T): 48 selections take the decode kernel; 600 the tcgen05
# kernel; 144 and 145 selections at the DeepSeek-V4 shape are the largest
# requests the 4 MiB scratch holds
@pytest.mark.gpu
@pytest.mark.parametrize("shape", [(512, 512, 16, 6, 8), (4096, 2048, 256, 6, 8), (512, 512, 16, 6, 100),
                                   (4096, 2048, 256, 6, 24), (4096, 2048, 256, 5, 29)])
def test_noalloc_matches_engine_forward_two_calls(setup, shape):
    torch, native, lib = setup
    import dee_b200
    H, I, E, K, T = shape
    bank = _bank(H, I, E)
    eng = dee_b200.new_engine(dee_b200.EngineConfig(hidden=H, inter=I, num_experts=E, topk=K))
    eng.attach_bank(0, bank)
    cfg = native.DeeConfig(H, I, E, K, 1, torch.cuda.current_device(), 0.0, 64)
    rng = np.random.default_rng(607 + T)
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
        assert np.array_equal(g.view(np.uint32), r.view(np.uint32)), \
            f"call {call}: not bit-identical to the engine (rel L2 {_rel_l2(g, r):.2e}, bar {TOL_REL_L2})"
    del eng


def _call_refused(native, lib, cfg, T, x=256, out=256, ids=256, w=256, status=None):
    """Call with addresses that are never dereferenced: every check below
    runs on the host before any CUDA call."""
    p = ctypes.c_void_p
    return lib.dee_moe_forward_noalloc(ctypes.byref(cfg), p(256), RECORD_BYTES_FULL, cfg.num_experts, p(x), T,
                                       p(ids), p(w), p(out), p(status) if status else None, None)


def test_noalloc_refuses_requests_beyond_the_static_scratch(native_lib):
    native, lib = native_lib
    H, I, E = FULL
    # 146 selections need 4,196,096 bytes of scratch: one more than fits
    cfg = native.DeeConfig(H, I, E, 2, 1, 0, 0.0, 64)
    assert _call_refused(native, lib, cfg, 73) == native.DEE_ERR_SCRATCH_LIMIT
    cfg6 = native.DeeConfig(H, I, E, 6, 1, 0, 0.0, 64)
    assert _call_refused(native, lib, cfg6, 100) == native.DEE_ERR_SCRATCH_LIMIT


def test_noalloc_refuses_misaligned_pointers_before_launching(native_lib):
    native, lib = native_lib
    H, I, E = FULL
    cfg = native.DeeConfig(H, I, E, 6, 1, 0, 0.0, 64)
    # a column slice of an FP16 tensor starts 2 bytes off a 16-byte boundary
    assert _call_refused(native, lib, cfg, 8, x=256 + 2) == native.DEE_ERR_INVALID
    assert _call_refused(native, lib, cfg, 8, out=256 + 4) == native.DEE_ERR_INVALID
    assert _call_refused(native, lib, cfg, 8, ids=256 + 2) == native.DEE_ERR_INVALID
    assert _call_refused(native, lib, cfg, 8, w=256 + 1) == native.DEE_ERR_INVALID
    assert _call_refused(native, lib, cfg, 8, status=256 + 2) == native.DEE_ERR_INVALID
