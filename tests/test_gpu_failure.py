"""Failure detection on the GPU without a GPU fault.

Every device wait in this library is bounded: when it runs out the kernel
sets a bit in the engine's status word and returns, the CUDA context stays
usable and the host learns of it from dee_engine_sync_status (fail closed,
as the reference reports failures through last_error_message,
dee.cpp/include/dee/engine.h:434-436).  These tests make waits run out on
purpose -- on flags and barriers that nothing ever sets -- and check the
report and that the next ordinary call still computes the right result.
"""
import ctypes
import time

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

H, I, E, K, WORLD = 512, 512, 16, 6, 2
EPR = E // WORLD
STATUS_PIPELINE_TIMEOUT = 1 << 0
STATUS_PEER_TIMEOUT = 1 << 6


@pytest.fixture(scope="module")
def torch_cuda():
    import torch
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    from dee_b200 import build
    build.build()
    return torch


def _engine(E_):
    import dee_b200
    return dee_b200.new_engine(dee_b200.EngineConfig(hidden=H, inter=I, num_experts=E_, topk=K, max_tokens=64))


def test_pipeline_wait_gives_up_and_reports(torch_cuda):
    """The bounded mbarrier wait of the pipeline kernels, on a barrier that
    nothing arrives on: it returns after its 50 ms limit with the pipeline
    timeout bit set."""
    torch = torch_cuda
    from dee_b200 import _native
    lib = _native.load()
    status = torch.zeros(1, dtype=torch.int32, device="cuda")
    torch.cuda.synchronize()
    t0 = time.perf_counter()
    rc = lib.dee_wait_selftest(50_000_000, ctypes.c_void_p(status.data_ptr()),
                               ctypes.c_void_p(torch.cuda.current_stream().cuda_stream))
    assert rc == 0
    torch.cuda.synchronize()
    elapsed = time.perf_counter() - t0
    assert int(status.item()) == STATUS_PIPELINE_TIMEOUT
    assert 0.04 <= elapsed < 1.5, elapsed
    # out-of-range limits are refused before any launch
    assert lib.dee_wait_selftest(10, ctypes.c_void_p(status.data_ptr()), None) == _native.DEE_ERR_INVALID


def test_missing_peer_rank_is_reported_and_context_stays_usable(torch_cuda, oracle_mod):
    """Two expert-parallel ranks emulated in this process on one GPU (the
    NVLink peer path with the blocks mapped by address).  Rank 1 never
    dispatches: rank 0's wait for rank 1's rows runs out after the engine's
    50 ms limit, and so does its wait for rank 1's returned rows; each sets
    status bit 6 and the stream goes on.  Afterwards an ordinary layer call
    on the same device returns the oracle's result."""
    torch = torch_cuda
    orc = oracle_mod
    layout = orc.Layout(H, I)
    recs = orc.synthetic_records(layout, E, seed=5150, kind="normal")
    T = 4
    ranks = []
    for r in range(WORLD):
        eng = _engine(EPR)
        bank = torch.from_numpy(np.ascontiguousarray(recs[r * EPR:(r + 1) * EPR])).cuda()
        eng.attach_bank(0, bank)
        eng.set_wait_limit(0.05)
        _, block = eng.ep_p2p_init(WORLD, r, T)
        ranks.append(dict(eng=eng, bank=bank, block=block))
    for rk in ranks:
        rk["eng"].ep_p2p_connect(None, [x["block"] for x in ranks])
    rng = np.random.default_rng(5151)
    x16 = orc.f16_bits(rng.standard_normal((T, H)))
    ids = np.stack([rng.choice(E, K, replace=False) for _ in range(T)]).astype(np.int32)
    w = rng.random((T, K)).astype(np.float32)
    w /= w.sum(axis=1, keepdims=True)
    dx = torch.from_numpy(x16.view(np.float16)).cuda()
    dids = torch.from_numpy(ids).cuda()
    dw = torch.from_numpy(w).cuda()
    out = torch.empty((T, H), dtype=torch.float32, device="cuda")
    eng0 = ranks[0]["eng"]
    torch.cuda.synchronize()
    t0 = time.perf_counter()
    eng0.ep_p2p_dispatch_device(dx.data_ptr(), dids.data_ptr())
    eng0.ep_p2p_experts_device(0)
    eng0.ep_p2p_combine_device(dw.data_ptr(), out.data_ptr())
    st = eng0.sync_status()
    elapsed = time.perf_counter() - t0
    assert st & STATUS_PEER_TIMEOUT, hex(st)
    assert "peer rank" in eng0.last_error_message()
    assert 0.09 <= elapsed < 1.5, elapsed  # two waits of 50 ms (rows in, rows back)
    assert eng0.sync_status() == 0  # the read cleared the word
    # the context is usable: an ordinary one-GPU layer on the same device
    full = _engine(E)
    full.attach_bank(0, torch.from_numpy(recs).cuda())
    ref = torch.empty((T, H), dtype=torch.float32, device="cuda")
    full.moe_forward_device(0, dx.data_ptr(), T, d_ids_ptr=dids.data_ptr(), d_weights_ptr=dw.data_ptr(),
                            d_out_ptr=ref.data_ptr())
    assert full.sync_status() == 0
    want = orc.combine_f32(orc.moe_layer_raw(recs, layout, x16, ids), w)
    assert orc.rel_l2(ref.cpu().numpy(), want) <= 2e-3
    for eng in (ranks[0]["eng"], ranks[1]["eng"], full):
        eng.close()


def test_wait_limit_is_range_checked(torch_cuda):
    import dee_b200
    eng = _engine(EPR)
    with pytest.raises(dee_b200.DeeError):
        eng.set_wait_limit(1e-6)
    with pytest.raises(dee_b200.DeeError):
        eng.set_wait_limit(5.0)
    eng.set_wait_limit(0.5)


def test_offload_copy_failure_is_reported_not_computed(torch_cuda, oracle_mod):
    """The offload tier's injected submit failure (the reference's
    AsyncPrefetcher.debug_fail_next_submit, include/dee/async_prefetcher.h:232):
    the prepare call reports it and names the expert, the expert is left not
    resident, so a forward run anyway reports bit 4 (expert not resident)
    rather than reading an unfilled slot; the next prepare cold-loads it and
    the layer then matches the oracle."""
    torch = torch_cuda
    orc = oracle_mod
    import dee_b200
    layers, T = 2, 4
    layout = orc.Layout(H, I)
    recs = orc.synthetic_records(layout, layers * E, seed=6060, kind="normal")
    host = torch.from_numpy(recs).pin_memory()
    pool = torch.empty((3 * K * T, recs.shape[1]), dtype=torch.uint8, device="cuda")
    eng = dee_b200.new_engine(dee_b200.EngineConfig(hidden=H, inter=I, num_experts=E, topk=K,
                                                    num_layers=layers, max_tokens=64))
    eng.offload_attach(host, layers, pool, pool.shape[0])
    rng = np.random.default_rng(6061)
    x16 = orc.f16_bits(rng.standard_normal((T, H)))
    ids = np.stack([rng.choice(E, K, replace=False) for _ in range(T)]).astype(np.int32)
    w = rng.random((T, K)).astype(np.float32)
    w /= w.sum(axis=1, keepdims=True)
    dx = torch.from_numpy(x16.view(np.float16)).cuda()
    dids = torch.from_numpy(ids).cuda()
    dw = torch.from_numpy(w).cuda()
    out = torch.empty((T, H), dtype=torch.float32, device="cuda")
    layer = 1
    eng.offload_debug_fail_next_copy()
    with pytest.raises(dee_b200.DeeError, match="could not be queued"):
        eng.offload_prepare_device(layer, dids.data_ptr(), T)
    eng.moe_forward_device(layer, dx.data_ptr(), T, d_ids_ptr=dids.data_ptr(), d_weights_ptr=dw.data_ptr(),
                           d_out_ptr=out.data_ptr())
    assert eng.sync_status() & (1 << 4)
    cold = eng.offload_prepare_device(layer, dids.data_ptr(), T)
    assert cold == 1  # only the expert whose copy failed
    eng.moe_forward_device(layer, dx.data_ptr(), T, d_ids_ptr=dids.data_ptr(), d_weights_ptr=dw.data_ptr(),
                           d_out_ptr=out.data_ptr())
    assert eng.sync_status() == 0
    want = orc.combine_f32(orc.moe_layer_raw(recs[layer * E:(layer + 1) * E], layout, x16, ids), w)
    assert orc.rel_l2(out.cpu().numpy(), want) <= 2e-3
