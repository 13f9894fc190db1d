"""The FP16 chain pinned to the reference's own GPU path.

oracle/_ref/libdee_ref_cuda.so is the reference project's FP4 decode
(dee.cpp/src/cuda_convert.cu:252-288) and batched cuBLAS SwiGLU
(dee.cpp/src/swiglu_cuda.cu:387-431) compiled from its sources, sequenced
per expert as Engine::moe_forward_batch_device_impl does
(dee.cpp/src/engine.cpp:776-1190; oracle/ref_cuda_shim.cu).  These tests
run both that chain and this library on the same records and tokens on the
same GPU and compare the raw FP32 expert rows [T, K, H]:
  * this library against the reference device path: relative L2 <= 2e-3
    over the layer and 5x that per selection;
  * the CPU oracle (the restatement every other parity test uses) against
    the reference device path, with the same bars -- so the oracle itself
    is pinned to the reference's GPU output, not only to its CPU code.
The file skips when the reference library was not built (the reference
sources were absent where the build ran).
"""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu

TOL_REL_L2 = 2e-3


@pytest.fixture(scope="module")
def ref(oracle_mod):
    import torch
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    if oracle_mod.ref_cuda_lib() is None:
        pytest.skip("oracle/_ref/libdee_ref_cuda.so not built (reference sources absent at build time)")
    from dee_b200 import build
    build.build()
    return torch


def _case(torch, orc, H, I, E, K, T, seed, limit=0.0, zipf=False):
    import dee_b200
    from dee_b200.records import RecordLayout, synthetic_bank
    layout = orc.Layout(H, I)
    bank = synthetic_bank(RecordLayout(H, I), E, seed=seed)
    rng = np.random.default_rng(seed + 1)
    x16 = orc.f16_bits(rng.standard_normal((T, H)))
    if zipf:
        p = 1.0 / np.arange(1, E + 1) ** 1.1
        p /= p.sum()
        ids = np.stack([rng.choice(E, K, replace=False, p=p) for _ in range(T)]).astype(np.int32)
    else:
        ids = np.stack([rng.choice(E, K, replace=False) for _ in range(T)]).astype(np.int32)
    eng = dee_b200.new_engine(dee_b200.EngineConfig(hidden=H, inter=I, num_experts=E, topk=K,
                                                    swiglu_limit=limit, max_tokens=max(T, 64)))
    eng.attach_bank(0, bank)
    dx = torch.from_numpy(x16.view(np.float16)).cuda()
    raw = torch.zeros((T, K, H), dtype=torch.float32, device="cuda")
    assert eng.moe_forward_batch_device(0, dx.data_ptr(), T, ids, K, raw.data_ptr()), eng.last_error_message()
    torch.cuda.synchronize()
    got = raw.cpu().numpy()
    want = orc.ref_cuda_moe_layer_raw(bank.data_ptr(), bank.shape[1], E, layout, x16, ids, limit)
    eng.close()
    return layout, bank, x16, ids, got, want


def _check(orc, got, want, T, K):
    assert np.isfinite(want).all() and np.isfinite(got).all()
    assert orc.rel_l2(got, want) <= TOL_REL_L2
    per = max(orc.rel_l2(got[t, r], want[t, r]) for t in range(T) for r in range(K))
    assert per <= 5 * TOL_REL_L2, per


@pytest.mark.parametrize("T,limit", [(1, 0.0), (8, 0.0), (33, 7.0), (300, 0.0)])
def test_small_shape_against_reference_gpu_path(ref, oracle_mod, T, limit):
    """H=I=512, 16 experts: decode-sized and prefill-sized token counts,
    with and without the SwiGLU clamp (swiglu_cuda.cu's swiglu_limit)."""
    orc = oracle_mod
    H, I, E, K = 512, 512, 16, 6
    layout, bank, x16, ids, got, want = _case(ref, orc, H, I, E, K, T, seed=900 + T, limit=limit)
    _check(orc, got, want, T, K)
    if limit == 0.0:
        recs = bank.cpu().numpy()
        _check(orc, orc.moe_layer_raw(recs, layout, x16, ids), want, T, K)


@pytest.mark.parametrize("T", [8, 512])
def test_deepseek_v4_shape_against_reference_gpu_path(ref, oracle_mod, T):
    """The DeepSeek-V4 expert shape (H=4096, I=2048, 13,369,344-byte records)
    over 32 experts: T=8 runs the decode kernels, T=512 with Zipf(1.1)
    expert popularity runs the tensor-memory grouped GEMM with ragged
    groups of up to a few hundred rows."""
    orc = oracle_mod
    H, I, E, K = 4096, 2048, 32, 6
    layout, bank, x16, ids, got, want = _case(ref, orc, H, I, E, K, T, seed=1200 + T, zipf=(T > 64))
    assert bank.shape[1] == 13_369_344
    _check(orc, got, want, T, K)
    if T == 8:
        recs = bank.cpu().numpy()
        _check(orc, orc.moe_layer_raw(recs, layout, x16, ids), want, T, K)
