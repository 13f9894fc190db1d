"""The official DeepSeek-V4 MoE semantics on the GPU (weight before w2,
FP32 SwiGLU chain with clamp 10, F8_E4M3 shared expert added) against the
reference's own outputs (tests/golden/official.npz) and the oracle's FP32
restatement.  Bar: relative L2 <= 2e-3 (the kernels' operands are FP16)."""
from pathlib import Path

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

GOLDEN = Path(__file__).resolve().parent / "golden"
TOL = 2e-3


@pytest.fixture(scope="module")
def torch_cuda():
    import torch
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    from dee_b200 import build
    build.build()
    return torch


def _engine(H, I, E, K, limit=10.0, max_tokens=128):
    import dee_b200
    return dee_b200.new_engine(dee_b200.EngineConfig(hidden=H, inter=I, num_experts=E, topk=K,
                                                     swiglu_limit=limit, max_tokens=max_tokens))


def _attach_shared(torch, eng, shared):
    dev = {k: torch.from_numpy(np.ascontiguousarray(v)).cuda() for k, v in shared.items()}
    eng.attach_shared_expert(0, dev["w1"], dev["s1"], dev["w3"], dev["s3"], dev["w2"], dev["s2"])


def _run(torch, eng, x32, ids, w, H):
    T = ids.shape[0]
    dx = torch.from_numpy(x32.astype(np.float16)).cuda()
    di = torch.from_numpy(np.ascontiguousarray(ids, dtype=np.int32)).cuda()
    dw = torch.from_numpy(np.ascontiguousarray(w, dtype=np.float32)).cuda()
    out = torch.empty((T, H), dtype=torch.float32, device="cuda")
    sh = torch.empty((T, H), dtype=torch.float32, device="cuda")
    eng.moe_forward_official_device(0, dx.data_ptr(), T, di.data_ptr(), dw.data_ptr(), out.data_ptr(),
                                    sh.data_ptr())
    torch.cuda.synchronize()
    assert eng.sync_status() == 0
    return out.cpu().numpy(), sh.cpu().numpy()


def test_official_layer_matches_reference_fixture(torch_cuda, oracle_mod):
    torch = torch_cuda
    orc = oracle_mod
    g = np.load(GOLDEN / "official.npz")
    layout = orc.Layout(512, 512)
    recs = orc.synthetic_records(layout, 16, seed=int(g["records_seed"]), kind="normal")
    eng = _engine(512, 512, 16, 6)
    bank = torch.from_numpy(recs).cuda()
    eng.attach_bank(0, bank)
    _attach_shared(torch, eng, {k: g["sh_" + k] for k in ("w1", "s1", "w3", "s3", "w2", "s2")})
    out, sh = _run(torch, eng, g["x"], g["expert_ids"].astype(np.int32), g["routing_weights"], 512)
    assert orc.rel_l2(sh, g["shared_output"]) <= TOL
    assert orc.rel_l2(out, g["moe_output"]) <= TOL
    assert np.array_equal(eng.journal_ids(5), g["expert_ids"].astype(np.int32))


@pytest.mark.parametrize("T", [1, 37, 100])
def test_official_layer_matches_oracle(torch_cuda, oracle_mod, T):
    """37 tokens: a ragged last 8-token tile of the shared expert; 100 tokens
    (600 selections): the routed part runs the tcgen05 kernel's official
    epilogue."""
    torch = torch_cuda
    orc = oracle_mod
    H, I, E, K, Is = 1024, 512, 16, 6, 512
    layout = orc.Layout(H, I)
    recs = orc.synthetic_records(layout, E, seed=808 + T, kind="normal")
    rng = np.random.default_rng(809 + T)
    x = rng.standard_normal((T, H)).astype(np.float16).astype(np.float32)
    ids = np.stack([rng.choice(E, K, replace=False) for _ in range(T)]).astype(np.int32)
    w = rng.random((T, K)).astype(np.float32)
    w = w / w.sum(axis=1, keepdims=True) * np.float32(1.5)
    e4 = rng.integers(0, 256, (Is, H), dtype=np.uint8)
    e4[(e4 & 0x7F) == 0x7F] = 0x38  # no NaN codes
    shared = {
        "w1": e4, "s1": rng.integers(0x70, 0x76, ((Is + 127) // 128, H // 128), dtype=np.uint8),
        "w3": np.roll(e4, 7, axis=1), "s3": rng.integers(0x70, 0x76, ((Is + 127) // 128, H // 128), dtype=np.uint8),
        "w2": np.ascontiguousarray(np.roll(e4, 3, axis=0).T.reshape(H, Is)),
        "s2": rng.integers(0x70, 0x76, (H // 128, (Is + 127) // 128), dtype=np.uint8),
    }
    eng = _engine(H, I, E, K)
    bank = torch.from_numpy(recs).cuda()
    eng.attach_bank(0, bank)
    _attach_shared(torch, eng, shared)
    out, sh = _run(torch, eng, x, ids, w, H)
    want, want_sh = orc.official_layer(recs, layout, x, ids, w, shared, 10.0)
    assert orc.rel_l2(sh, want_sh) <= TOL
    assert orc.rel_l2(out, want) <= TOL
    per = [orc.rel_l2(out[t], want[t]) for t in range(T)]
    assert max(per) <= 5 * TOL
