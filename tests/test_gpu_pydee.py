"""The pybind11 binding on the GPU: dee_b200._pydee.Engine (the reference's
pydee method names and argument order over the C ABI, GIL released around
each engine call) gives the same bits as the ctypes binding for
moe_forward_batch_device (host int32 ids) and moe_forward_combined_device
(device int64 ids, caller's stream)."""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu

H, I, E, K = 512, 512, 16, 6


@pytest.fixture(scope="module")
def setup(oracle_mod):
    import torch
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    from dee_b200 import build
    build.build()
    build.build_pydee()
    import dee_b200._pydee as pydee
    return torch, pydee


@pytest.mark.parametrize("T", [8, 300])
def test_pydee_matches_ctypes_binding(setup, oracle_mod, T):
    torch, pydee = setup
    import dee_b200
    orc = oracle_mod
    layout = orc.Layout(H, I)
    recs = orc.synthetic_records(layout, E, seed=1111 + T, kind="normal")
    bank = torch.from_numpy(recs).cuda()
    rng = np.random.default_rng(1112 + T)
    x16 = orc.f16_bits(rng.standard_normal((T, H)))
    ids = np.stack([rng.choice(E, K, replace=False) for _ in range(T)]).astype(np.int32)
    w = rng.random((T, K)).astype(np.float32)
    w /= w.sum(1, keepdims=True)
    dx = torch.from_numpy(x16.view(np.float16)).cuda()

    eng = pydee.Engine()
    assert eng.init(pydee.EngineConfig(hidden=H, inter=I, num_experts=E, topk=K, max_tokens=T,
                                       device_id=torch.cuda.current_device())), eng.last_error_message()
    assert eng.attach_bank(0, bank.data_ptr(), E, bank.shape[1]), eng.last_error_message()
    ref = dee_b200.new_engine(dee_b200.EngineConfig(hidden=H, inter=I, num_experts=E, topk=K, max_tokens=T))
    ref.attach_bank(0, bank)

    raw = torch.zeros((T, K, H), dtype=torch.float32, device="cuda")
    raw_ref = torch.zeros_like(raw)
    assert eng.moe_forward_batch_device(0, dx.data_ptr(), T, ids, K, raw.data_ptr()), eng.last_error_message()
    assert ref.moe_forward_batch_device(0, dx.data_ptr(), T, ids, K, raw_ref.data_ptr())
    assert torch.equal(raw, raw_ref)
    assert orc.rel_l2(raw.cpu().numpy(), orc.moe_layer_raw(recs, layout, x16, ids)) <= 2e-3

    stream = torch.cuda.Stream()
    d_ids = torch.from_numpy(ids.astype(np.int64)).cuda()
    d_w = torch.from_numpy(w).cuda()
    out = torch.empty((T, H), dtype=torch.float16, device="cuda")
    out_ref = torch.empty_like(out)
    torch.cuda.synchronize()
    assert eng.moe_forward_combined_device(0, dx.data_ptr(), T, d_ids.data_ptr(), K, d_w.data_ptr(),
                                           out.data_ptr(), 0, stream.cuda_stream), eng.last_error_message()
    assert eng.sync_status(stream.cuda_stream) == 0
    assert ref.moe_forward_combined_device(0, dx.data_ptr(), T, d_ids.data_ptr(), K, d_w.data_ptr(),
                                           out_ref.data_ptr(), 0, stream.cuda_stream)
    assert ref.sync_status(stream) == 0
    assert torch.equal(out, out_ref)
    eng.close()
