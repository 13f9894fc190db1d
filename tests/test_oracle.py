"""CPU checks that pin the oracle to the reference before it checks the GPU.

Known answers come from the reference's own tests (cited per test); the
fixtures in tests/golden come from the reference's Python semantics (see
tests/golden/make_golden.py).
"""
import hashlib
import os

import numpy as np
import pytest

GOLDEN = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")


def _load(name):
    return np.load(os.path.join(GOLDEN, name), allow_pickle=False)


def _records(orc, layout, n, seed, sha):
    recs = orc.synthetic_records(layout, n, seed=int(seed), kind="normal")
    assert hashlib.sha256(recs.tobytes()).hexdigest() == str(sha), "synthetic record generator drifted"
    return recs


# --- FP4 known answers: dee.cpp/tests/test_deepseek_v4_fp4_decode.cpp:43-105 ---

def test_e2m1_table_and_scales(oracle_mod):
    orc = oracle_mod
    assert list(orc.E2M1_TABLE) == [0.0, 0.5, 1.0, 1.5, 2.0, 3.0, 4.0, 6.0,
                                    0.0, -0.5, -1.0, -1.5, -2.0, -3.0, -4.0, -6.0]
    L = orc.lib()
    assert L.dee_ref_scale_host(0x7F) == 1.0
    assert L.dee_ref_scale_host(0x80) == 2.0
    assert L.dee_ref_scale_host(0x86) == 128.0
    assert L.dee_ref_scale_host(0x76) == 1.0 / 512.0
    assert L.dee_ref_scale_device(0x00) == 0.0
    assert L.dee_ref_scale_device(0xFF) == np.finfo(np.float32).max


def test_fp4_matrix_and_nibble_order(oracle_mod):
    orc = oracle_mod
    out, n = 2, 64
    packed = np.zeros((out, n // 2), np.uint8)
    packed[0, :] = 0x2 | (0x2 << 4)
    packed[1, :] = 0x3 | (0x3 << 4)
    scale = np.array([[0x7F, 0x80], [0x81, 0x82]], np.uint8)
    w = orc.fp4_dequant_f32(packed, scale)
    assert w[0, 0] == 1.0 and w[0, 32] == 2.0 and w[1, 0] == 6.0 and w[1, 32] == 12.0
    one = np.zeros((out, n // 2), np.uint8)
    one[0, 0] = 0x0F
    w = orc.fp4_dequant_f32(one, np.full((out, 2), 0x7F, np.uint8))
    assert w[0, 0] == -6.0 and w[0, 1] == 0.0
    h = orc.fp4_decode_f16(one, np.full((out, 2), 0x7F, np.uint8))
    assert h[0, 0] == np.float16(-6.0).view(np.uint16) and h[0, 1] == 0


def test_decode_matches_reference_python(oracle_mod):
    g = _load("decode.npz")
    w = oracle_mod.fp4_dequant_f32(g["packed"], g["scale"])
    assert np.array_equal(w.view(np.uint32), g["w"].view(np.uint32))


def test_decode_matches_reference_cpp(oracle_mod):
    ref = oracle_mod.ref_lib()
    if ref is None:
        pytest.skip("oracle/_ref not built (reference sources absent on this machine)")
    rng = np.random.default_rng(7)
    packed = rng.integers(0, 256, (16, 256), dtype=np.uint8)
    scale = rng.integers(0, 256, (16, 16), dtype=np.uint8)
    got = oracle_mod.fp4_dequant_f32(packed, scale)
    want = np.empty_like(got)
    ref.dee_refimpl_fp4_dequantize(packed.ctypes.data, scale.ctypes.data, 16, 512, want.ctypes.data)
    assert np.array_equal(got.view(np.uint32), want.view(np.uint32))


def test_device_decode_semantics_fp16(oracle_mod):
    """cuda_convert.cu:217-245: FP16(table * scale), FP32_MAX clamp, zero floor."""
    orc = oracle_mod
    rng = np.random.default_rng(11)
    packed = rng.integers(0, 256, (8, 512), dtype=np.uint8)
    scale = np.arange(256, dtype=np.uint8).reshape(8, 32)
    h = orc.fp4_decode_f16(packed, scale)
    nib = np.stack([packed & 15, packed >> 4], -1).reshape(8, 1024)
    vals = orc.E2M1_TABLE[nib]
    s = np.array([orc.lib().dee_ref_scale_device(int(b)) for b in range(256)], np.float32).reshape(8, 32)
    with np.errstate(over="ignore"):
        want = (vals * np.repeat(s, 32, axis=1)).astype(np.float32).astype(np.float16).view(np.uint16)
    assert np.array_equal(h, want)


def test_f16_conversion_matches_ieee(oracle_mod):
    L = oracle_mod.lib()
    rng = np.random.default_rng(3)
    xs = np.concatenate([rng.standard_normal(4000).astype(np.float32) * 10.0 ** rng.integers(-9, 6, 4000),
                         np.array([65504, 65519.99, 65520, 1e9, -0.0, 5.96e-8, 2.98e-8, 2.99e-8,
                                   6.1e-5, np.inf, -np.inf], np.float32)]).astype(np.float32)
    for x in xs:
        with np.errstate(over="ignore"):
            want = np.float32(x).astype(np.float16).view(np.uint16)
        assert L.dee_ref_f32_to_f16(float(x)) == want, x
        assert L.dee_ref_f16_to_f32(int(want)) == np.float16(np.uint16(want).view(np.float16)).astype(np.float32)


def test_quantizer_matches_reference_round_trip(oracle_mod):
    g = _load("quant.npz")
    p, s = oracle_mod.quantize_fp4(g["w"])
    wq = oracle_mod.fp4_dequant_f32(p, s)
    assert np.array_equal(wq, g["wq"])


# --- router: dee.cpp/tests/test_real_router.cpp:71-116, test_router_cuda.cpp:37-53 ---

def test_router_golden(oracle_mod):
    ids, w = oracle_mod.route_topk(np.array([[1, 2, 3], [-1, 4, 2]], np.float32), 2)
    assert ids.tolist() == [[2, 1], [1, 2]]
    np.testing.assert_allclose(w, [[0.7310586, 0.2689414], [0.8807971, 0.1192029]], atol=1e-5)


def test_router_ties_prefer_lower_id(oracle_mod):
    ids, w = oracle_mod.route_topk(np.array([[0.5, 2.0, 2.0, 2.0, -1.0]], np.float32), 3)
    assert ids.tolist() == [[1, 2, 3]]
    assert np.all(w == w[0, 0])


def test_router_rejects_nonfinite(oracle_mod):
    with pytest.raises(ValueError):
        oracle_mod.route_topk(np.array([[np.nan, 1.0, 2.0]], np.float32), 2)


def test_router_exp_rounding_does_not_change_ids(oracle_mod):
    """The device router evaluates exp in double and rounds once; emulate it
    in numpy and compare ids with the oracle (which calls libm expf) on
    seeded logits: ids must be identical, weights within 2 ulp."""
    rng = np.random.default_rng(12)
    T, E, K = 4000, 256, 6
    logits = (rng.standard_normal((T, E)) * 2.0).astype(np.float32)
    ids_ref, w_ref = oracle_mod.route_topk(logits, K)
    m = logits.max(axis=1, keepdims=True)
    p = np.exp((logits - m).astype(np.float32).astype(np.float64)).astype(np.float32)
    den = np.zeros(T, np.float64)
    for e in range(E):
        den += p[:, e].astype(np.float64)
    inv = (1.0 / den).astype(np.float32)
    p = (p * inv[:, None]).astype(np.float32)
    order = np.lexsort((np.tile(np.arange(E), (T, 1)), -p), axis=1)[:, :K]
    assert np.array_equal(order.astype(np.int32), ids_ref)
    sel = np.take_along_axis(p, order, 1)
    s = np.zeros(T, np.float32)
    for k in range(K):
        s = (s + sel[:, k]).astype(np.float32)
    w = (sel / s[:, None]).astype(np.float32)
    ulp = np.abs(w.view(np.int32) - w_ref.view(np.int32))
    assert ulp.max() <= 2


# --- grouping: engine.cpp:812-823 ---

def test_group_order(oracle_mod):
    ids = np.array([[2, 1], [1, 2], [1, 0]], np.int32)  # T=3, K=2
    counts, offsets, perm = oracle_mod.group(ids, 3)
    assert counts.tolist() == [1, 3, 2]
    # expert 1: rank 0 tokens 1, 2 then rank 1 token 0 -> positions 2, 4, 1
    assert perm[offsets[1]:offsets[2]].tolist() == [2, 4, 1]
    assert perm[offsets[2]:offsets[3]].tolist() == [0, 3]


# --- expert chain vs the reference FP32 semantics (tolerance 2e-3 rel L2) ---

@pytest.mark.parametrize("limit", [0, 10])
def test_fp16_chain_vs_reference_fp32(oracle_mod, limit):
    orc = oracle_mod
    g = _load("expert.npz")
    layout = orc.Layout(512, 512)
    recs = _records(orc, layout, 3, g["records_seed"], g["records_sha256"])
    x16 = orc.f16_bits(g["x"])
    L = orc.lib()
    for e in range(3):
        y = np.empty((5, 512), np.float32)
        L.dee_ref_expert_f16(recs[e].ctypes.data, 512, 512, x16.ctypes.data, 5, float(limit), y.ctypes.data)
        assert orc.rel_l2(y, g[f"y_limit{limit}"][e]) < 2e-3


def test_fp16_chain_vs_reference_cpp_executor(oracle_mod):
    orc = oracle_mod
    ref = orc.ref_lib()
    if ref is None:
        pytest.skip("oracle/_ref not built")
    layout = orc.Layout(512, 512)
    recs = orc.synthetic_records(layout, 2, seed=9, kind="normal")
    x = np.random.default_rng(10).standard_normal(512).astype(np.float16)
    y = np.empty((1, 512), np.float32)
    orc.lib().dee_ref_expert_f16(recs[1].ctypes.data, 512, 512, x.view(np.uint16).ctypes.data, 1, 0.0,
                                 y.ctypes.data)
    yr = np.empty(512, np.float32)
    xf = x.astype(np.float32)
    assert ref.dee_refimpl_expert(recs[1].ctypes.data, 512, 512, xf.ctypes.data, 1.0, 0.0, yr.ctypes.data) == 0
    assert orc.rel_l2(y[0], yr) < 2e-3


# --- combines: swiglu_cuda.cu:69-116, test_expert_batch_cuda.cpp:492-523 ---

def test_combine_f16_adversarial_bits(oracle_mod):
    raw = np.array([[[-3.041015625], [3.09765625]]], np.float32)  # [T=1, K=2, H=1]
    w = np.array([[1.0, 0.891144335269928]], np.float32)
    out = oracle_mod.combine_f16(raw, w, np.array([[0, 1]], np.int64))
    assert int(out[0, 0]) == 0xB480


def test_combine_f16_stable_expert_order(oracle_mod):
    rng = np.random.default_rng(5)
    raw = rng.standard_normal((2, 4, 8)).astype(np.float32)
    w = rng.random((2, 4)).astype(np.float32)
    ids = np.array([[7, 2, 7, 1], [0, 1, 2, 3]], np.int64)
    out = oracle_mod.combine_f16(raw, w, ids)
    order = [3, 1, 0, 2]  # ascending id, ties by position
    acc = np.float16(0)
    for p in order:
        acc = np.float16(np.float32(acc) + np.float32(np.float16(np.float32(np.float16(raw[0, p, 0])) * w[0, p])))
    assert out[0, 0] == acc.view(np.uint16)


def test_combine_f32_rank_order(oracle_mod):
    rng = np.random.default_rng(6)
    raw = rng.standard_normal((3, 6, 16)).astype(np.float32)
    w = rng.random((3, 6)).astype(np.float32)
    out = oracle_mod.combine_f32(raw, w)
    acc = np.zeros((3, 16), np.float32)
    for r in range(6):
        acc = (acc + (w[:, r:r + 1] * raw[:, r]).astype(np.float32)).astype(np.float32)
    assert np.array_equal(out, acc)


def test_moe_layer_raw_layout(oracle_mod):
    """raw[t, r] holds expert ids[t, r] applied to token t (engine.cpp:1080-1113)."""
    orc = oracle_mod
    layout = orc.Layout(512, 512)
    recs = orc.synthetic_records(layout, 4, seed=21, kind="normal")
    x = orc.f16_bits(np.random.default_rng(22).standard_normal((3, 512)))
    ids = np.array([[3, 1], [1, 1], [0, 2]], np.int32)
    raw = orc.moe_layer_raw(recs, layout, x, ids)
    L = orc.lib()
    for t in range(3):
        for r in range(2):
            y = np.empty((1, 512), np.float32)
            L.dee_ref_expert_f16(recs[ids[t, r]].ctypes.data, 512, 512, x[t:t + 1].ctypes.data, 1, 0.0,
                                 y.ctypes.data)
            assert np.array_equal(y[0], raw[t, r])


# --- DeepSeek-V4 router: deepseek_v4_layer_common.py:349-403 ---

def test_dsv4_router_matches_reference(oracle_mod):
    g = _load("moe_layer.npz")
    ids, w, scores = oracle_mod.route_dsv4(g["logits"], 6, bias=g["bias"])
    assert np.array_equal(ids, g["expert_ids"].astype(np.int32))
    np.testing.assert_allclose(scores + g["bias"], g["scores"], rtol=1e-6, atol=1e-6)
    np.testing.assert_allclose(w, g["routing_weights"], rtol=1e-6)
    assert abs(float(w.sum(1).mean()) - 1.5) < 1e-5


def test_dsv4_hash_router_matches_reference(oracle_mod):
    g = _load("moe_layer.npz")
    ids, w, _ = oracle_mod.route_dsv4(g["logits"], 6, tid2eid=g["tid2eid"], input_ids=g["input_ids"])
    assert np.array_equal(ids, g["hash_ids"].astype(np.int32))
    np.testing.assert_allclose(w, g["hash_weights"], rtol=1e-6)


def test_e4m3_table_matches_torch():
    import torch
    from oracle import oracle as orc
    tab = orc.e4m3_table()
    ref = torch.arange(256, dtype=torch.int32).to(torch.uint8).view(torch.float8_e4m3fn).float().numpy()
    assert np.array_equal(np.isnan(tab), np.isnan(ref))
    ok = ~np.isnan(ref)
    assert np.array_equal(tab[ok], ref[ok])


def test_official_layer_matches_reference_fixture(oracle_mod):
    """moe_layer_forward of the reference (FP32, weight before w2, clamp 10,
    F8_E4M3 shared expert) vs the oracle's restatement, same route."""
    orc = oracle_mod
    g = _load("official.npz")
    layout = orc.Layout(512, 512)
    recs = _records(orc, layout, 16, g["records_seed"], g["records_sha256"])
    shared = {k: g["sh_" + k] for k in ("w1", "s1", "w3", "s3", "w2", "s2")}
    moe, sh = orc.official_layer(recs, layout, g["x"], g["expert_ids"], g["routing_weights"], shared, 10.0)
    assert orc.rel_l2(sh, g["shared_output"]) < 1e-5
    assert orc.rel_l2(moe, g["moe_output"]) < 1e-5


def test_e4m3_encoder_matches_torch():
    """The oracle's round-to-nearest-even E4M3 encoder against torch's
    float8_e4m3fn cast (an independent implementation), incl. subnormal ties."""
    import torch
    from oracle import oracle as orc
    rng = np.random.default_rng(5)
    v = np.concatenate([rng.standard_normal(50000) * 60, rng.standard_normal(50000) * 0.005,
                        np.array([0.0, -0.0, 448.0, -448.0, 2.0 ** -9, 2.0 ** -10, 3 * 2.0 ** -11, 2.0 ** -6,
                                  1.0625, 1.1875, 2.0 ** -6 * 15 / 16])])
    v = np.clip(v, -448, 448).astype(np.float32)
    ref = torch.from_numpy(v).to(torch.float8_e4m3fn).view(torch.uint8).numpy()
    assert np.array_equal(orc.e4m3_encode(v), ref)


@pytest.mark.parametrize("block", [128, 32])
def test_act_quant_matches_reference_fixture(oracle_mod, block):
    """act_quant_inplace of the reference (UE8M0 scales) vs the oracle's
    restatement of the official kernel: identical FP16 round trips."""
    orc = oracle_mod
    g = _load("act_quant.npz")
    q, s = orc.act_quant(g["x"], block)
    y = orc.act_dequant_f32(q, s, block).astype(np.float16).view(np.uint16)
    assert np.array_equal(y, g[f"y{block}"])


def test_reference_gpu_path_library_loads(oracle_mod):
    """oracle/_ref/libdee_ref_cuda.so (the reference's FP4 decode + cuBLAS
    SwiGLU device path) resolves every symbol when loaded; its computing
    test runs on the GPU."""
    import os
    path = os.path.join(os.path.dirname(oracle_mod.__file__), "_ref", "libdee_ref_cuda.so")
    if not os.path.exists(path):
        pytest.skip("oracle/_ref/libdee_ref_cuda.so not built (reference sources absent on this machine)")
    lib = oracle_mod.ref_cuda_lib()
    assert lib is not None and hasattr(lib, "dee_refcuda_moe_layer")
