"""GPU parity: the CUDA path through the C ABI against the CPU oracle.

Bars (stated per test): bit-exact for decode, quantise, routing ids, the
combines given identical raw rows and the permutation; relative L2 <= 2e-3
for expert outputs against the oracle's restatement of the reference
dequant + cuBLAS FP16 chain.
"""
import ctypes

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

TOL_REL_L2 = 2e-3


@pytest.fixture(scope="module")
def torch_cuda():
    import torch
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    major, minor = torch.cuda.get_device_capability()
    assert (major, minor) == (10, 0), f"needs sm_100 (B200), got sm_{major}{minor}"
    from dee_b200 import build
    build.build()
    return torch


@pytest.fixture(scope="module")
def lib(torch_cuda):
    from dee_b200 import _native
    return _native.load()


def _engine(H, I, E, K, layers=1, limit=0.0, max_tokens=64):
    import dee_b200
    return dee_b200.new_engine(dee_b200.EngineConfig(hidden=H, inter=I, num_experts=E, topk=K,
                                                     num_layers=layers, swiglu_limit=limit,
                                                     max_tokens=max_tokens))


def _rand_ids(rng, T, E, K, allow_dup=False):
    if allow_dup:
        return rng.integers(0, E, (T, K)).astype(np.int32)
    return np.stack([rng.choice(E, K, replace=False) for _ in range(T)]).astype(np.int32)


def test_fp4_decode_bitexact(torch_cuda, lib, oracle_mod):
    torch = torch_cuda
    rng = np.random.default_rng(1)
    out, n = 256, 512
    packed = rng.integers(0, 256, (out, n // 2), dtype=np.uint8)
    scale = np.tile(np.arange(256, dtype=np.uint8), out * (n // 32) // 256 + 1)[: out * (n // 32)]
    scale = scale.reshape(out, n // 32)
    dp = torch.from_numpy(packed).cuda()
    ds = torch.from_numpy(scale).cuda()
    dst = torch.empty((out, n), dtype=torch.float16, device="cuda")
    assert lib.dee_fp4_decode_device(dp.data_ptr(), ds.data_ptr(), dst.data_ptr(), out, n, None) == 0
    torch.cuda.synchronize()
    got = dst.cpu().numpy().view(np.uint16)
    want = oracle_mod.fp4_decode_f16(packed, scale)
    assert np.array_equal(got, want)


def test_fp4_quantize_matches_oracle(torch_cuda, lib, oracle_mod):
    torch = torch_cuda
    rng = np.random.default_rng(2)
    w = (rng.standard_normal((128, 1024)) * 0.02).astype(np.float32)
    w[0, :32] = 0
    w[1, 5] = 3.0
    dw = torch.from_numpy(w).cuda()
    p = torch.empty((128, 512), dtype=torch.uint8, device="cuda")
    s = torch.empty((128, 32), dtype=torch.uint8, device="cuda")
    assert lib.dee_fp4_quantize_device(dw.data_ptr(), 128, 1024, p.data_ptr(), s.data_ptr(), None) == 0
    torch.cuda.synchronize()
    wp, ws = oracle_mod.quantize_fp4(w)
    assert np.array_equal(p.cpu().numpy(), wp)
    assert np.array_equal(s.cpu().numpy(), ws)


# spread 3: some exp terms fall below the exact-tree bound, so the denominator
# is summed serially; spread 0.5: every term is above it and the warp sums a
# tree, which must give the identical double
@pytest.mark.parametrize("T,E,K,spread", [(2, 3, 2, 0), (1000, 256, 6, 3.0), (37, 16, 6, 3.0),
                                          (500, 256, 6, 0.5), (64, 200, 8, 0.5)])
def test_route_topk_matches_oracle(torch_cuda, oracle_mod, T, E, K, spread):
    torch = torch_cuda
    if (T, E, K) == (2, 3, 2):
        logits = np.array([[1, 2, 3], [-1, 4, 2]], np.float32)  # test_real_router.cpp:91-116
    else:
        logits = (np.random.default_rng(T).standard_normal((T, E)) * spread).astype(np.float32)
        logits[0, :8] = 1.25  # exact ties
    eng = _engine(512, 512, E, K)
    dl = torch.from_numpy(logits).cuda()
    ids = torch.empty((T, K), dtype=torch.int32, device="cuda")
    w = torch.empty((T, K), dtype=torch.float32, device="cuda")
    eng.route_topk_device(dl.data_ptr(), T, ids.data_ptr(), w.data_ptr())
    assert eng.sync_status() == 0
    ids_ref, w_ref = oracle_mod.route_topk(logits, K)
    assert np.array_equal(ids.cpu().numpy(), ids_ref)
    ulp = np.abs(w.cpu().numpy().view(np.int32) - w_ref.view(np.int32))
    assert ulp.max() <= 2
    if (T, E, K) == (2, 3, 2):
        np.testing.assert_allclose(w.cpu().numpy(), [[0.7310586, 0.2689414], [0.8807971, 0.1192029]],
                                   atol=1e-5)


def _run_layer(torch, eng, bank_dev, x16, ids, weights, layer=0, raw_out=True):
    T, K = ids.shape
    H = eng.cfg.hidden
    dx = torch.from_numpy(x16.view(np.float16)).cuda()
    raw = torch.zeros((T, K, H), dtype=torch.float32, device="cuda")
    assert eng.moe_forward_batch_device(layer, dx.data_ptr(), T, ids, K, raw.data_ptr()), \
        eng.last_error_message()
    return raw.cpu().numpy()


@pytest.mark.parametrize("T,dup", [(1, False), (5, True), (8, False), (33, False), (300, False)])
def test_moe_raw_small_shape(torch_cuda, oracle_mod, T, dup):
    torch = torch_cuda
    orc = oracle_mod
    H, I, E, K = 512, 512, 16, 6
    layout = orc.Layout(H, I)
    recs = orc.synthetic_records(layout, E, seed=31 + T, kind="normal")
    rng = np.random.default_rng(T)
    x16 = orc.f16_bits(rng.standard_normal((T, H)))
    ids = _rand_ids(rng, T, E, K, allow_dup=dup)
    eng = _engine(H, I, E, K)
    bank = torch.from_numpy(recs).cuda()
    eng.attach_bank(0, bank)
    raw = _run_layer(torch, eng, bank, x16, ids, None)
    want = orc.moe_layer_raw(recs, layout, x16, ids)
    assert np.isfinite(raw).all()
    assert orc.rel_l2(raw, want) <= TOL_REL_L2
    # per selection as well: no row may be silently wrong
    per = [orc.rel_l2(raw[t, r], want[t, r]) for t in range(T) for r in range(K)]
    assert max(per) <= 5 * TOL_REL_L2
    assert np.array_equal(eng.journal_ids(T), ids)


def _skewed_ids(rng, T, E, K, s=1.3):
    """Distinct per-token ids drawn with Zipf(s) expert popularity: a few
    experts take many rows (several 128-row tiles), most take a handful."""
    p = np.arange(1, E + 1, dtype=np.float64) ** -s
    p /= p.sum()
    perm = rng.permutation(E)
    return np.stack([perm[rng.choice(E, size=K, replace=False, p=p)] for _ in range(T)]).astype(np.int32)


@pytest.mark.parametrize("H,I,T", [(512, 1024, 400), (1024, 512, 700)])
def test_moe_raw_skewed_groups(torch_cuda, oracle_mod, H, I, T):
    """The tensor-memory grouped GEMM over ragged groups: tiles of every
    token-box size (16, 32, 64 and 128 rows) and experts spanning several
    tiles, against the oracle per selection."""
    torch = torch_cuda
    orc = oracle_mod
    E, K = 48, 6
    layout = orc.Layout(H, I)
    recs = orc.synthetic_records(layout, E, seed=H + I + T, kind="normal")
    rng = np.random.default_rng(T)
    x16 = orc.f16_bits(rng.standard_normal((T, H)))
    ids = _skewed_ids(rng, T, E, K, s=1.5)
    counts = np.bincount(ids.ravel(), minlength=E)
    assert counts.max() > 256 and (counts[counts > 0] <= 16).any()
    assert ((counts > 16) & (counts <= 32)).any() and ((counts > 32) & (counts <= 64)).any()
    eng = _engine(H, I, E, K, max_tokens=T)
    bank = torch.from_numpy(recs).cuda()
    eng.attach_bank(0, bank)
    raw = _run_layer(torch, eng, bank, x16, ids, None)
    want = orc.moe_layer_raw(recs, layout, x16, ids)
    assert np.isfinite(raw).all()
    assert orc.rel_l2(raw, want) <= TOL_REL_L2
    per = [orc.rel_l2(raw[t, r], want[t, r]) for t in range(T) for r in range(K)]
    assert max(per) <= 5 * TOL_REL_L2


def test_full_shape_prefill_rows_match_decode(torch_cuda):
    """DeepSeek-V4 shapes, 4096 tokens with Zipf(1.1)-skewed routing through
    the tensor-memory grouped GEMM: the raw rows of sampled tokens equal
    (within the FP32-summation tolerance) the same tokens' rows from the
    register-dequant decode kernel, itself checked against the oracle at these
    shapes in test_full_shape_decode."""
    torch = torch_cuda
    from dee_b200.records import RecordLayout, synthetic_bank
    H, I, E, K, T = 4096, 2048, 256, 6, 4096
    bank = synthetic_bank(RecordLayout(H, I), E, seed=77)
    eng = _engine(H, I, E, K, max_tokens=T)
    eng.attach_bank(0, bank)
    rng = np.random.default_rng(78)
    ids = _skewed_ids(rng, T, E, K, s=1.1)
    x16 = rng.standard_normal((T, H)).astype(np.float16).view(np.uint16)
    raw = _run_layer(torch, eng, bank, x16, ids, None)
    assert np.isfinite(raw).all()
    sample = np.concatenate([rng.choice(T, 8, replace=False)])
    dec = _run_layer(torch, eng, bank, x16[sample].copy(), ids[sample].copy(), None)
    for i, t in enumerate(sample):
        for r in range(K):
            num = np.linalg.norm((raw[t, r] - dec[i, r]).astype(np.float64))
            den = np.linalg.norm(dec[i, r].astype(np.float64))
            assert num <= 1e-3 * den, (t, r, num / den)


def _plant_edge_rows(layout, recs, rng, experts, frac=0.25):
    """Give a fraction of the W2 rows of `experts` one scale byte for the
    whole row, drawn from the limits of the exact-FP16 dequant range: 60, 100
    and 103 underflow or round in FP16, 104 and 140 are the last exact bytes,
    141 and 142 overflow for |value| >= 2 (their rows keep only nibbles of
    magnitude <= 1.5).  Returns {expert: (rows, bytes)}."""
    H, I = layout.hidden, layout.inter
    edge = np.array([60, 100, 103, 104, 140, 141, 142], dtype=np.uint8)
    planted = {}
    for e in experts:
        rec = recs[e]
        sc = rec[layout.s2:layout.s2 + H * I // 32].reshape(H, I // 32)
        pk = rec[layout.w2:layout.w2 + H * I // 2].reshape(H, I // 2)
        rows = np.flatnonzero(rng.random(H) < frac)
        vals = rng.choice(edge, size=rows.size)
        sc[rows] = vals[:, None]
        big = rows[vals >= 141]
        pk[big] &= np.uint8(0xBB)  # keep the sign and the two low code bits of each nibble
        planted[e] = (rows, vals)
    return planted


@pytest.mark.parametrize("T,H,I", [(8, 512, 512), (100, 512, 512), (48, 1024, 2048), (48, 4096, 2048)])
def test_moe_raw_edge_scales(torch_cuda, oracle_mod, T, H, I):
    """Scale bytes outside the exact-FP16 range take the FP16-rounded dequant
    path; rows without them take the fast one.  Every output feature is
    compared at its own magnitude.  T <= 64 runs the decode kernel, T=100 the
    tensor-memory grouped GEMM; both projections share the dequant code.
    The decode kernel copies scale rows of 32, 64 or 128 bytes (K = 1024,
    2048, 4096) with swizzled tensor loads and shorter ones with bulk
    copies: H, I = 512 / 1024 and 2048 / 4096 and 2048 cover each kind."""
    torch = torch_cuda
    orc = oracle_mod
    E, K = 16, 6
    layout = orc.Layout(H, I)
    recs = orc.synthetic_records(layout, E, seed=404, kind="normal")
    rng = np.random.default_rng(405)
    _plant_edge_rows(layout, recs, rng, experts=range(E))
    x16 = orc.f16_bits(rng.standard_normal((T, H)))
    ids = _rand_ids(rng, T, E, K)
    eng = _engine(H, I, E, K, max_tokens=128)
    bank = torch.from_numpy(recs).cuda()
    eng.attach_bank(0, bank)
    raw = _run_layer(torch, eng, bank, x16, ids, None).reshape(T * K, H)
    want = orc.moe_layer_raw(recs, layout, x16, ids).reshape(T * K, H)
    assert np.isfinite(want).all() and np.isfinite(raw).all()
    flat = ids.reshape(-1)
    n_zero, worst = 0, 0.0
    for e in np.unique(flat):
        w, r = want[flat == e], raw[flat == e]
        den = np.linalg.norm(w.astype(np.float64), axis=0)
        num = np.linalg.norm((r - w).astype(np.float64), axis=0)
        zero = den == 0
        assert not r[:, zero].any()  # rows whose weights dequantise to zeros (byte 60)
        n_zero += int(zero.sum())
        worst = max(worst, float((num[~zero] / den[~zero]).max()))
    assert n_zero > 0
    assert worst <= 5 * TOL_REL_L2, worst


def test_combines_bitexact_given_raw(torch_cuda, oracle_mod):
    torch = torch_cuda
    orc = oracle_mod
    H, I, E, K, T = 512, 512, 16, 6, 9
    layout = orc.Layout(H, I)
    recs = orc.synthetic_records(layout, E, seed=77, kind="normal")
    rng = np.random.default_rng(78)
    x16 = orc.f16_bits(rng.standard_normal((T, H)))
    ids = _rand_ids(rng, T, E, K)
    w = rng.random((T, K)).astype(np.float32)
    w /= w.sum(1, keepdims=True)
    eng = _engine(H, I, E, K)
    eng.attach_bank(0, torch.from_numpy(recs).cuda())
    dx = torch.from_numpy(x16.view(np.float16)).cuda()
    dids = torch.from_numpy(ids).cuda()
    dids64 = dids.long()
    dw = torch.from_numpy(w).cuda()
    out32 = torch.empty((T, H), dtype=torch.float32, device="cuda")
    raw = torch.empty((T, K, H), dtype=torch.float32, device="cuda")
    eng.moe_forward_device(0, dx.data_ptr(), T, d_ids_ptr=dids.data_ptr(), d_weights_ptr=dw.data_ptr(),
                           d_out_ptr=out32.data_ptr(), d_raw_ptr=raw.data_ptr())
    assert eng.sync_status() == 0
    raw_np = raw.cpu().numpy()
    assert np.array_equal(out32.cpu().numpy(), orc.combine_f32(raw_np, w))
    out16 = torch.empty((T, H), dtype=torch.float16, device="cuda")
    raw2 = torch.empty_like(raw)
    stream = torch.cuda.current_stream()
    assert eng.moe_forward_combined_device(0, dx.data_ptr(), T, dids64.data_ptr(), K, dw.data_ptr(),
                                           out16.data_ptr(), raw2.data_ptr(), stream.cuda_stream)
    assert eng.sync_status(stream) == 0
    assert np.array_equal(raw2.cpu().numpy(), raw_np)  # deterministic across calls
    assert np.array_equal(out16.cpu().numpy().view(np.uint16), orc.combine_f16(raw_np, w, ids))


def test_rows_independent_of_batch_composition(torch_cuda, oracle_mod):
    torch = torch_cuda
    orc = oracle_mod
    H, I, E, K = 512, 512, 16, 6
    layout = orc.Layout(H, I)
    recs = orc.synthetic_records(layout, E, seed=90, kind="normal")
    rng = np.random.default_rng(91)
    x16 = orc.f16_bits(rng.standard_normal((20, H)))
    ids = _rand_ids(rng, 20, E, K)
    eng = _engine(H, I, E, K, max_tokens=128)
    bank = torch.from_numpy(recs).cuda()
    eng.attach_bank(0, bank)
    full = _run_layer(torch, eng, bank, x16, ids, None)
    for t in (0, 7, 19):
        alone = _run_layer(torch, eng, bank, x16[t:t + 1].copy(), ids[t:t + 1].copy(), None)
        assert np.array_equal(alone[0], full[t])


def test_bad_host_ids_fail_closed(torch_cuda):
    torch = torch_cuda
    eng = _engine(512, 512, 16, 6)
    eng.attach_bank(0, torch.zeros((16, 417792), dtype=torch.uint8, device="cuda"))
    dx = torch.zeros((2, 512), dtype=torch.float16, device="cuda")
    raw = torch.zeros((2, 6, 512), dtype=torch.float32, device="cuda")
    ids = np.array([[0, 1, 2, 3, 4, 5], [0, 1, 2, 3, 4, 16]], np.int32)
    assert not eng.moe_forward_batch_device(0, dx.data_ptr(), 2, ids, 6, raw.data_ptr())
    assert "outside" in eng.last_error_message()


def test_bad_device_ids_reported(torch_cuda):
    torch = torch_cuda
    eng = _engine(512, 512, 16, 6)
    eng.attach_bank(0, torch.zeros((16, 417792), dtype=torch.uint8, device="cuda"))
    dx = torch.zeros((2, 512), dtype=torch.float16, device="cuda")
    ids = torch.tensor([[0, 1, 2, 3, 4, 5], [0, 1, 2, 3, 4, 99]], dtype=torch.int64, device="cuda")
    w = torch.full((2, 6), 1 / 6, dtype=torch.float32, device="cuda")
    out = torch.empty((2, 512), dtype=torch.float16, device="cuda")
    s = torch.cuda.current_stream()
    assert eng.moe_forward_combined_device(0, dx.data_ptr(), 2, ids.data_ptr(), 6, w.data_ptr(),
                                           out.data_ptr(), 0, s.cuda_stream)
    assert eng.sync_status(s) & (1 << 4)


@pytest.mark.parametrize("T", [2, 4])
def test_one_launch_layer_recovers_after_bad_ids(torch_cuda, oracle_mod, T):
    """A batch of at most 24 selections runs the one-launch layer, whose
    counters between CTAs advance by a fixed amount per launch.  A device id
    outside the bank is reported (status bit 4), its selection left out and
    the counters kept in step; after the status read the next calls of the
    same engine (several, so a drifted counter would show) match the oracle
    and the two-call route + forward bit for bit."""
    torch = torch_cuda
    orc = oracle_mod
    H, I, E, K = 512, 512, 16, 6
    layout = orc.Layout(H, I)
    recs = orc.synthetic_records(layout, E, seed=4242, kind="normal")
    eng = _engine(H, I, E, K)
    eng.attach_bank(0, torch.from_numpy(recs).cuda())
    rng = np.random.default_rng(4243 + T)
    x16 = orc.f16_bits(rng.standard_normal((T, H)))
    dx = torch.from_numpy(x16.view(np.float16)).cuda()
    bad = _rand_ids(rng, T, E, K)
    bad[T - 1, K - 1] = E + 3
    dbad = torch.from_numpy(bad).cuda()
    w = torch.full((T, K), 1.0 / K, dtype=torch.float32, device="cuda")
    out = torch.empty((T, H), dtype=torch.float32, device="cuda")
    eng.moe_forward_device(0, dx.data_ptr(), T, d_ids_ptr=dbad.data_ptr(), d_weights_ptr=w.data_ptr(),
                           d_out_ptr=out.data_ptr())
    assert eng.sync_status() & (1 << 4)
    for step in range(3):
        ids = _rand_ids(rng, T, E, K)
        dids = torch.from_numpy(ids).cuda()
        raw = torch.empty((T, K, H), dtype=torch.float32, device="cuda")
        eng.moe_forward_device(0, dx.data_ptr(), T, d_ids_ptr=dids.data_ptr(), d_weights_ptr=w.data_ptr(),
                               d_out_ptr=out.data_ptr(), d_raw_ptr=raw.data_ptr())
        assert eng.sync_status() == 0, eng.last_error_message()
        want_raw = orc.moe_layer_raw(recs, layout, x16, ids)
        assert orc.rel_l2(raw.cpu().numpy(), want_raw) <= TOL_REL_L2
        assert np.array_equal(out.cpu().numpy(), orc.combine_f32(raw.cpu().numpy(), w.cpu().numpy()))


@pytest.mark.parametrize("T", [2, 4])
def test_one_launch_layer_raw_only_call_leaves_combine_counters(torch_cuda, oracle_mod, T):
    """A call of the one-launch layer without a combine output adds nothing
    to the (token, feature block) counters of the fused combine -- a
    selection left out for a bad id included.  Combined calls that follow it
    on the same engine, with no status read in between, complete each block
    only once all K of its rows are stored, so every output equals the
    rank-order combine of that call's own rows bit for bit.  The status read
    at the end still reports the first call's bad id."""
    torch = torch_cuda
    orc = oracle_mod
    H, I, E, K = 512, 512, 16, 6
    layout = orc.Layout(H, I)
    recs = orc.synthetic_records(layout, E, seed=4343, kind="normal")
    eng = _engine(H, I, E, K)
    eng.attach_bank(0, torch.from_numpy(recs).cuda())
    rng = np.random.default_rng(4344 + T)
    x16 = orc.f16_bits(rng.standard_normal((T, H)))
    dx = torch.from_numpy(x16.view(np.float16)).cuda()
    bad = _rand_ids(rng, T, E, K)
    bad[0, 1] = E + 5
    dbad = torch.from_numpy(bad).cuda()
    raw0 = torch.empty((T, K, H), dtype=torch.float32, device="cuda")
    eng.moe_forward_device(0, dx.data_ptr(), T, d_ids_ptr=dbad.data_ptr(), d_raw_ptr=raw0.data_ptr())
    for step in range(3):
        xs = orc.f16_bits(rng.standard_normal((T, H)))
        dxs = torch.from_numpy(xs.view(np.float16)).cuda()
        dids = torch.from_numpy(_rand_ids(rng, T, E, K)).cuda()
        w = torch.from_numpy(rng.uniform(0.05, 1.0, (T, K)).astype(np.float32)).cuda()
        out = torch.empty((T, H), dtype=torch.float32, device="cuda")
        raw = torch.empty((T, K, H), dtype=torch.float32, device="cuda")
        eng.moe_forward_device(0, dxs.data_ptr(), T, d_ids_ptr=dids.data_ptr(), d_weights_ptr=w.data_ptr(),
                               d_out_ptr=out.data_ptr(), d_raw_ptr=raw.data_ptr())
        torch.cuda.synchronize()
        assert np.array_equal(out.cpu().numpy(), orc.combine_f32(raw.cpu().numpy(), w.cpu().numpy())), step
    assert eng.sync_status() & (1 << 4)


def test_entry_points_refuse_misaligned_pointers(torch_cuda, oracle_mod):
    """A device pointer off the alignment its kernels need -- offset the way
    a column slice would be -- is refused with DEE_ERR_INVALID naming the
    pointer, before anything is launched; the same engine then runs the
    layer on the aligned pointers and matches the oracle."""
    import dee_b200
    torch = torch_cuda
    orc = oracle_mod
    H, I, E, K, T = 512, 512, 16, 6, 4
    layout = orc.Layout(H, I)
    recs = orc.synthetic_records(layout, E, seed=4545, kind="normal")
    eng = _engine(H, I, E, K)
    eng.attach_bank(0, torch.from_numpy(recs).cuda())
    rng = np.random.default_rng(4546)
    x16 = orc.f16_bits(rng.standard_normal((T, H)))
    logits = rng.standard_normal((T, E)).astype(np.float32)
    # every buffer has a spare 16 bytes, so base + offset stays inside it
    dx = torch.zeros(T * H + 8, dtype=torch.float16, device="cuda")
    dx[:T * H] = torch.from_numpy(x16.view(np.float16).reshape(-1)).cuda()
    dl = torch.zeros(T * E + 4, dtype=torch.float32, device="cuda")
    dl[:T * E] = torch.from_numpy(logits.reshape(-1)).cuda()
    ids = torch.zeros(T * K + 4, dtype=torch.int32, device="cuda")
    w = torch.zeros(T * K + 4, dtype=torch.float32, device="cuda")
    out = torch.zeros(T * H + 4, dtype=torch.float32, device="cuda")
    raw = torch.zeros(T * K * H + 4, dtype=torch.float32, device="cuda")
    ids64 = torch.zeros(T * K + 2, dtype=torch.int64, device="cuda")
    out16 = torch.zeros(T * H + 8, dtype=torch.float16, device="cuda")
    x, lg, i, wp, o, r = (t.data_ptr() for t in (dx, dl, ids, w, out, raw))
    torch.cuda.synchronize()
    n0 = eng.launch_count()
    cases = [
        ("d_x_f16", lambda: eng.moe_forward_routed_device(0, x + 2, T, lg, i, wp, d_out_ptr=o)),
        ("d_x_f16", lambda: eng.moe_forward_device(0, x + 8, T, d_ids_ptr=i, d_weights_ptr=wp, d_out_ptr=o)),
        ("d_logits", lambda: eng.moe_forward_routed_device(0, x, T, lg + 2, i, wp, d_out_ptr=o)),
        ("d_ids", lambda: eng.moe_forward_device(0, x, T, d_ids_ptr=i + 2, d_weights_ptr=wp, d_out_ptr=o)),
        ("d_weights", lambda: eng.route_topk_device(lg, T, i, wp + 1)),
        ("d_out_f32", lambda: eng.moe_forward_device(0, x, T, d_ids_ptr=i, d_weights_ptr=wp, d_out_ptr=o + 4)),
        ("d_raw", lambda: eng.moe_forward_device(0, x, T, d_ids_ptr=i, d_raw_ptr=r + 8)),
        ("d_raw", lambda: eng.moe_forward_mxfp8_device(0, x, T, i, r + 4)),
    ]
    for name, call in cases:
        with pytest.raises(dee_b200.DeeError, match=name + " must be"):
            call()
    # the pydee-style entry answers False and keeps the reason
    assert not eng.moe_forward_combined_device(0, x, T, ids64.data_ptr() + 4, K, wp, out16.data_ptr(), 0, 0)
    assert "d_expert_ids must be 8-byte aligned" in eng.last_error_message()
    assert not eng.moe_forward_combined_device(0, x, T, ids64.data_ptr(), K, wp, out16.data_ptr() + 1, 0, 0)
    assert "d_output_f16 must be 2-byte aligned" in eng.last_error_message()
    torch.cuda.synchronize()
    assert eng.launch_count() == n0
    assert eng.sync_status() == 0
    eng.moe_forward_routed_device(0, x, T, lg, i, wp, d_out_ptr=o, d_raw_ptr=r)
    assert eng.sync_status() == 0, eng.last_error_message()
    ids_ref, _ = orc.route_topk(logits, K)
    assert np.array_equal(ids[:T * K].cpu().numpy().reshape(T, K), ids_ref)
    got_raw = raw[:T * K * H].cpu().numpy().reshape(T, K, H)
    assert orc.rel_l2(got_raw, orc.moe_layer_raw(recs, layout, x16, ids_ref)) <= TOL_REL_L2
    got_w = w[:T * K].cpu().numpy().reshape(T, K)
    assert np.array_equal(out[:T * H].cpu().numpy().reshape(T, H), orc.combine_f32(got_raw, got_w))


@pytest.mark.parametrize("T", [8, 64])
def test_full_shape_decode(torch_cuda, oracle_mod, T):
    """DeepSeek-V4 shapes (H=4096, I=2048, E=256, K=6), device-built bank."""
    torch = torch_cuda
    orc = oracle_mod
    from dee_b200.records import RecordLayout, synthetic_bank
    H, I, E, K = 4096, 2048, 256, 6
    bank = synthetic_bank(RecordLayout(H, I), E, seed=5)
    rng = np.random.default_rng(500 + T)
    x16 = orc.f16_bits(rng.standard_normal((T, H)))
    ids = _rand_ids(rng, T, E, K)
    eng = _engine(H, I, E, K)
    eng.attach_bank(0, bank)
    raw = _run_layer(torch, eng, bank, x16, ids, None)
    used = np.unique(ids)
    recs = np.zeros((E, bank.shape[1]), np.uint8)
    recs[used] = bank[torch.from_numpy(used).cuda().long()].cpu().numpy()
    want = orc.moe_layer_raw(recs, orc.Layout(H, I), x16, ids)
    assert orc.rel_l2(raw, want) <= TOL_REL_L2


@pytest.mark.parametrize("hashed", [False, True])
def test_dsv4_router_matches_reference_fixture(torch_cuda, oracle_mod, hashed):
    """Selection ids exact against the reference's own torch router outputs;
    weights within 1e-6 relative (device expf/log1pf vs torch CPU)."""
    import os
    torch = torch_cuda
    g = np.load(os.path.join(os.path.dirname(__file__), "golden", "moe_layer.npz"))
    T, E = g["logits"].shape
    eng = _engine(512, 512, E, 6)
    dl = torch.from_numpy(g["logits"]).cuda()
    ids = torch.empty((T, 6), dtype=torch.int32, device="cuda")
    w = torch.empty((T, 6), dtype=torch.float32, device="cuda")
    if hashed:
        t2e = torch.from_numpy(g["tid2eid"]).cuda()
        inp = torch.from_numpy(g["input_ids"]).cuda()
        eng.route_dsv4_device(dl.data_ptr(), T, ids.data_ptr(), w.data_ptr(), d_tid2eid_ptr=t2e.data_ptr(),
                              d_input_ids_ptr=inp.data_ptr())
        want_ids, want_w = g["hash_ids"], g["hash_weights"]
    else:
        db = torch.from_numpy(g["bias"]).cuda()
        eng.route_dsv4_device(dl.data_ptr(), T, ids.data_ptr(), w.data_ptr(), d_bias_ptr=db.data_ptr())
        want_ids, want_w = g["expert_ids"], g["routing_weights"]
    assert eng.sync_status() == 0
    assert np.array_equal(ids.cpu().numpy(), want_ids.astype(np.int32))
    np.testing.assert_allclose(w.cpu().numpy(), want_w, rtol=1e-6)


def test_dsv4_router_large_matches_oracle(torch_cuda, oracle_mod):
    torch = torch_cuda
    rng = np.random.default_rng(17)
    T, E = 2048, 256
    logits = (rng.standard_normal((T, E)) * 2).astype(np.float32)
    bias = (rng.standard_normal(E) * 0.05).astype(np.float32)
    eng = _engine(512, 512, E, 6)
    ids = torch.empty((T, 6), dtype=torch.int32, device="cuda")
    w = torch.empty((T, 6), dtype=torch.float32, device="cuda")
    dl, db = torch.from_numpy(logits).cuda(), torch.from_numpy(bias).cuda()
    eng.route_dsv4_device(dl.data_ptr(), T, ids.data_ptr(), w.data_ptr(), d_bias_ptr=db.data_ptr())
    assert eng.sync_status() == 0
    want_ids, want_w, _ = oracle_mod.route_dsv4(logits, 6, bias=bias)
    assert np.array_equal(ids.cpu().numpy(), want_ids)
    np.testing.assert_allclose(w.cpu().numpy(), want_w, rtol=2e-6)


def _group_dev(torch, eng, lib, ids):
    T, K = ids.shape
    di = torch.from_numpy(np.ascontiguousarray(ids, dtype=np.int32)).cuda()
    perm = torch.full((T * K,), -7, dtype=torch.int32, device="cuda")
    row_of = torch.full((T * K,), -7, dtype=torch.int32, device="cuda")
    offs = torch.full((eng.cfg.num_experts + 1,), -7, dtype=torch.int32, device="cuda")
    s = torch.cuda.current_stream()
    rc = lib.dee_group_by_expert_device(eng._h, ctypes.c_void_p(di.data_ptr()), T, K,
                                        ctypes.c_void_p(perm.data_ptr()), ctypes.c_void_p(row_of.data_ptr()),
                                        ctypes.c_void_p(offs.data_ptr()), ctypes.c_void_p(s.cuda_stream))
    assert rc == 0
    torch.cuda.synchronize()
    return perm.cpu().numpy(), row_of.cpu().numpy(), offs.cpu().numpy(), eng.sync_status()


@pytest.mark.parametrize("T,K,E,skew", [(1, 6, 256, 0.0), (8, 6, 256, 0.0), (300, 6, 64, 0.0), (341, 6, 16, 0.0),
                                         (342, 6, 16, 0.0), (700, 6, 48, 1.5), (4096, 6, 256, 1.1),
                                         (5000, 8, 256, 0.0), (3000, 1, 7, 0.0)])
def test_group_by_expert_bitexact(torch_cuda, lib, oracle_mod, T, K, E, skew):
    """The grouping (one CTA for up to 2048 selections, two multi-CTA passes
    above) against the oracle's restatement of engine.cpp:812-823: perm,
    row_of and offsets bit-exact, rows of an expert in (rank, token) order."""
    rng = np.random.default_rng(T * 31 + E)
    ids = _skewed_ids(rng, T, E, K, s=skew) if skew else _rand_ids(rng, T, E, K)
    eng = _engine(512, 512, E, K, max_tokens=T)
    perm, row_of, offs, status = _group_dev(torch_cuda, eng, lib, ids)
    counts, w_offs, w_perm = oracle_mod.group(ids, E)
    assert status == 0
    assert np.array_equal(offs, w_offs)
    assert np.array_equal(perm, w_perm)
    assert np.array_equal(row_of[perm], np.arange(T * K, dtype=np.int32))


@pytest.mark.parametrize("T", [10, 3000])
def test_group_by_expert_rejects_bad_ids(torch_cuda, lib, T):
    """An id outside [0, E) sets the bad-expert status bit and leaves that
    position out (row_of = -1); the valid selections are still grouped."""
    rng = np.random.default_rng(T)
    E, K = 32, 6
    ids = _rand_ids(rng, T, E, K)
    ids[T // 2, 3] = E + 5
    ids[T - 1, 0] = -3
    eng = _engine(512, 512, E, K, max_tokens=T)
    perm, row_of, offs, status = _group_dev(torch_cuda, eng, lib, ids)
    assert status & (1 << 4)
    bad = [(T // 2) * K + 3, (T - 1) * K + 0]
    assert all(row_of[p] == -1 for p in bad)
    n = offs[E]
    assert n == T * K - 2
    assert np.array_equal(np.sort(perm[:n]), np.setdiff1d(np.arange(T * K), bad))


def test_two_devices_one_process(torch_cuda, oracle_mod):
    """One process drives engines on two GPUs (decode and prefill kernels on
    each): every kernel's shared-memory opt-in is made per device, and both
    devices return the same bits for the same inputs."""
    torch = torch_cuda
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    import dee_b200
    orc = oracle_mod
    H, I, E, K = 512, 512, 16, 6
    layout = orc.Layout(H, I)
    recs = orc.synthetic_records(layout, E, seed=61, kind="normal")
    rng = np.random.default_rng(61)
    outs = []
    for dev in (0, 1):
        with torch.cuda.device(dev):
            eng = dee_b200.new_engine(dee_b200.EngineConfig(hidden=H, inter=I, num_experts=E, topk=K,
                                                            device_id=dev, max_tokens=300))
            bank = torch.from_numpy(recs).to(f"cuda:{dev}")
            eng.attach_bank(0, bank)
            got = []
            for T in (8, 300):  # the decode kernel, then the tcgen05 prefill kernel
                r = np.random.default_rng(T)
                x16 = orc.f16_bits(r.standard_normal((T, H)))
                ids = _rand_ids(r, T, E, K)
                dx = torch.from_numpy(x16.view(np.float16)).to(f"cuda:{dev}")
                raw = torch.zeros((T, K, H), dtype=torch.float32, device=f"cuda:{dev}")
                assert eng.moe_forward_batch_device(0, dx.data_ptr(), T, ids, K, raw.data_ptr())
                torch.cuda.synchronize(dev)
                assert eng.sync_status() == 0
                got.append(raw.cpu().numpy())
            outs.append(got)
            del eng
    for a, b in zip(outs[0], outs[1]):
        assert np.array_equal(a, b)


@pytest.mark.parametrize("T,K", [(3, 2), (5, 4), (8, 4), (200, 2)])
def test_batch_with_fewer_selections_than_configured(torch_cuda, lib, oracle_mod, T, K):
    """The C entry takes topk <= EngineConfig::topk like
    Engine::moe_forward_batch_device (engine.cpp:780-781): K = 4 or 2 on a
    top-6 engine, raw [T, K, H] against the oracle and the journal holding
    the call's [T, K] ids; the Python method keeps pydee's binding rule
    (pydee.cpp:443-444) and refuses a topk other than the configured one."""
    torch = torch_cuda
    orc = oracle_mod
    H, I, E = 512, 512, 16
    layout = orc.Layout(H, I)
    recs = orc.synthetic_records(layout, E, seed=T + K, kind="normal")
    eng = _engine(H, I, E, 6, max_tokens=T)
    eng.attach_bank(0, torch.from_numpy(recs).cuda())
    rng = np.random.default_rng(T * 7 + K)
    x16 = orc.f16_bits(rng.standard_normal((T, H)))
    ids = _rand_ids(rng, T, E, K)
    dx = torch.from_numpy(x16.view(np.float16)).cuda()
    raw = torch.zeros((T, K, H), dtype=torch.float32, device="cuda")
    rc = lib.dee_moe_forward_batch_device(eng._h, 0, ctypes.c_void_p(dx.data_ptr()), T,
                                          ids.ctypes.data_as(ctypes.c_void_p), K, ctypes.c_void_p(raw.data_ptr()))
    assert rc == 0, eng.last_error_message()
    want = orc.moe_layer_raw(recs, layout, x16, ids)
    assert orc.rel_l2(raw.cpu().numpy(), want) <= TOL_REL_L2
    journal = np.empty(T * K, dtype=np.int32)
    assert lib.dee_journal_ids_host(eng._h, journal.ctypes.data_as(ctypes.c_void_p), T * K) == T * K
    assert np.array_equal(journal.reshape(T, K), ids)
    with pytest.raises(RuntimeError, match="does not match EngineConfig.topk"):
        eng.moe_forward_batch_device(0, dx.data_ptr(), T, ids, K, raw.data_ptr())
    # device ids and weights with the combine (T * K <= 24 takes the
    # one-launch layer): rank-order sum of the K rows, bit for bit
    w = rng.random((T, K)).astype(np.float32)
    dids = torch.from_numpy(ids).cuda()
    dw = torch.from_numpy(w).cuda()
    out = torch.empty((T, H), dtype=torch.float32, device="cuda")
    raw2 = torch.empty((T, K, H), dtype=torch.float32, device="cuda")
    rc = lib.dee_moe_forward_device(eng._h, 0, ctypes.c_void_p(dx.data_ptr()), T, ctypes.c_void_p(dids.data_ptr()),
                                    None, K, ctypes.c_void_p(dw.data_ptr()), ctypes.c_void_p(out.data_ptr()),
                                    ctypes.c_void_p(raw2.data_ptr()), None)
    assert rc == 0, eng.last_error_message()
    assert eng.sync_status() == 0
    assert np.array_equal(raw2.cpu().numpy(), raw.cpu().numpy())
    assert np.array_equal(out.cpu().numpy(), orc.combine_f32(raw2.cpu().numpy(), w))


@pytest.mark.parametrize("T,dup", [(1, False), (8, True), (64, False)])
def test_decode_combine_bitexact_over_calls(torch_cuda, oracle_mod, T, dup):
    """Decode-sized calls (T * K <= 384, the register-dequant kernel) three
    times in a row on one engine, with repeated expert ids in a token and at
    the 384-selection boundary: out is bit-identical to the oracle's
    rank-order combine of the same raw rows, and the raw rows match the
    oracle's FP16 chain.  At H = 1024 the gate/up items have two K stages, so
    the pair of consumer warps of an item goes through its reduction barrier
    many times per CTA."""
    torch = torch_cuda
    orc = oracle_mod
    H, I, E, K = 1024, 512, 16, 6
    layout = orc.Layout(H, I)
    recs = orc.synthetic_records(layout, E, seed=818, kind="normal")
    eng = _engine(H, I, E, K, max_tokens=64)
    eng.attach_bank(0, torch.from_numpy(recs).cuda())
    rng = np.random.default_rng(819 + T)
    for call in range(3):
        x16 = orc.f16_bits(rng.standard_normal((T, H)))
        ids = _rand_ids(rng, T, E, K, allow_dup=dup)
        w = rng.random((T, K)).astype(np.float32)
        w /= w.sum(1, keepdims=True)
        dx = torch.from_numpy(x16.view(np.float16)).cuda()
        dids = torch.from_numpy(ids).cuda()
        dw = torch.from_numpy(w).cuda()
        out = torch.full((T, H), float("nan"), dtype=torch.float32, device="cuda")
        raw = torch.empty((T, K, H), dtype=torch.float32, device="cuda")
        eng.moe_forward_device(0, dx.data_ptr(), T, d_ids_ptr=dids.data_ptr(), d_weights_ptr=dw.data_ptr(),
                               d_out_ptr=out.data_ptr(), d_raw_ptr=raw.data_ptr())
        assert eng.sync_status() == 0
        raw_np = raw.cpu().numpy()
        assert np.array_equal(out.cpu().numpy(), orc.combine_f32(raw_np, w)), f"call {call}"
        assert orc.rel_l2(raw_np, orc.moe_layer_raw(recs, layout, x16, ids)) <= TOL_REL_L2


@pytest.mark.parametrize("T,E,H,I", [(1, 64, 512, 512), (3, 16, 512, 512), (4, 256, 512, 512), (8, 256, 512, 512),
                                     (33, 64, 512, 512), (64, 256, 512, 512), (65, 64, 512, 512),
                                     (100, 16, 512, 512), (1, 32, 4096, 2048), (4, 32, 4096, 2048)])
def test_routed_forward_matches_route_then_forward(torch_cuda, oracle_mod, T, E, H, I):
    """dee_moe_forward_routed_device against dee_route_topk_device followed
    by dee_moe_forward_device: ids, weights, raw rows, the combined output
    and the journal bit-identical.  T*K <= 24 takes the one-launch layer
    (routing, grouping and token rows inside the decode kernel; (3, 16) puts
    several rows in a tile, and the DeepSeek-V4 shape runs it at full size);
    up to 384 selections with E <= 256 the fused router+permutation kernel;
    (65, 64) and (100, 16) the two-kernel fallback inside the same entry
    point.  Ids also equal the oracle's."""
    torch = torch_cuda
    orc = oracle_mod
    K = 6
    layout = orc.Layout(H, I)
    recs = orc.synthetic_records(layout, E, seed=77 + E, kind="normal")
    rng = np.random.default_rng(7000 + T)
    x16 = orc.f16_bits(rng.standard_normal((T, H)))
    logits = (rng.standard_normal((T, E)) * 2.0).astype(np.float32)
    eng = _engine(H, I, E, K)
    bank = torch.from_numpy(recs).cuda()
    eng.attach_bank(0, bank)
    dx = torch.from_numpy(x16.view(np.float16)).cuda()
    dl = torch.from_numpy(logits).cuda()

    def run(fused):
        ids = torch.full((T, K), -7, dtype=torch.int32, device="cuda")
        w = torch.full((T, K), -1.0, dtype=torch.float32, device="cuda")
        out = torch.empty((T, H), dtype=torch.float32, device="cuda")
        raw = torch.empty((T, K, H), dtype=torch.float32, device="cuda")
        if fused:
            eng.moe_forward_routed_device(0, dx.data_ptr(), T, dl.data_ptr(), ids.data_ptr(), w.data_ptr(),
                                          d_out_ptr=out.data_ptr(), d_raw_ptr=raw.data_ptr())
        else:
            eng.route_topk_device(dl.data_ptr(), T, ids.data_ptr(), w.data_ptr())
            eng.moe_forward_device(0, dx.data_ptr(), T, d_ids_ptr=ids.data_ptr(), d_weights_ptr=w.data_ptr(),
                                   d_out_ptr=out.data_ptr(), d_raw_ptr=raw.data_ptr())
        assert eng.sync_status() == 0, eng.last_error_message()
        return [t.cpu().numpy() for t in (ids, w, out, raw)] + [eng.journal_ids(T)]

    a = run(True)
    b = run(False)
    for got, want in zip(a, b):
        assert np.array_equal(got.view(np.uint32) if got.dtype == np.float32 else got,
                              want.view(np.uint32) if want.dtype == np.float32 else want)
    ids_ref, _ = orc.route_topk(logits, K)
    assert np.array_equal(a[0], ids_ref)
    assert np.array_equal(a[4], a[0])
