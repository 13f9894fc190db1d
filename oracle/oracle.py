"""Parity oracle for the routed-expert MoE path (TEST INFRASTRUCTURE ONLY).

Only ``tests/``, ``__graft_entry__.smoke()`` and the ``cpu_baseline`` leg of
``bench.py`` import this module.  It is the checker, never the measured or
shipped path.

It wraps two shared libraries built by ``oracle/Makefile``:

* ``oracle/libdee_oracle.so`` -- the C restatement in ``dee_oracle.c``
  (decode, router, grouping, FP16 expert chain, combines; each function
  cites the reference line it follows).
* ``oracle/_ref/libdee_ref.so`` -- the reference project's own CPU code
  (``dee.cpp/src/weight_mmap.cpp`` FP4 decode and the KT-bridge
  ``ReferenceCpuExecutor``), compiled from the reference sources.

and adds numpy restatements used to build synthetic inputs:

* ``quantize_fp4`` -- the published MXFP4 recipe the reference's
  quantisation helpers follow (``dee.cpp/scripts/deepseek_v4_layer_common.py``
  ``fast_log2_ceil``/``fast_round_scale`` :160-178 and ``round_e2m1_grid``
  :181-211): per 32-element block, scale = 2^ceil(log2(amax / 6)) as a
  UE8M0 byte, values divided by the scale, clamped to +-6 and rounded to the
  E2M1 grid with ties to the even grid entry.
* ``build_record`` -- the DEE4 record layout ``[w1][w3][w2][s1][s3][s2]``
  (``dee.cpp/include/dee/expert_store.h:28-46``,
  ``dee.cpp/kaggle/deepseek-v4-flash-0731/repack_to_dee4.py:42-55``).
"""
from __future__ import annotations

import ctypes
import os
import threading
from dataclasses import dataclass

import numpy as np

_HERE = os.path.dirname(os.path.abspath(__file__))
_LIB = None
_REF = None

E2M1_TABLE = np.array([0.0, 0.5, 1.0, 1.5, 2.0, 3.0, 4.0, 6.0,
                       0.0, -0.5, -1.0, -1.5, -2.0, -3.0, -4.0, -6.0], dtype=np.float32)


def build_libs(with_ref: bool = False) -> None:
    """Compile the oracle (and optionally the reference shim) in place."""
    import subprocess
    targets = ["all"] + (["ref"] if with_ref else [])
    subprocess.run(["make", "-s", "-C", _HERE] + targets, check=True)


def lib() -> ctypes.CDLL:
    global _LIB
    if _LIB is None:
        path = os.path.join(_HERE, "libdee_oracle.so")
        if not os.path.exists(path):
            build_libs(False)
        L = ctypes.CDLL(path)
        P = ctypes.c_void_p
        L.dee_ref_f32_to_f16.restype = ctypes.c_uint16
        L.dee_ref_f32_to_f16.argtypes = [ctypes.c_float]
        L.dee_ref_f16_to_f32.restype = ctypes.c_float
        L.dee_ref_f16_to_f32.argtypes = [ctypes.c_uint16]
        L.dee_ref_scale_device.restype = ctypes.c_float
        L.dee_ref_scale_device.argtypes = [ctypes.c_uint8]
        L.dee_ref_scale_host.restype = ctypes.c_float
        L.dee_ref_scale_host.argtypes = [ctypes.c_uint8]
        L.dee_ref_fp4_decode_f16.argtypes = [P, P, P, ctypes.c_size_t, ctypes.c_size_t]
        L.dee_ref_fp4_dequant_f32.argtypes = [P, P, ctypes.c_size_t, ctypes.c_size_t, P]
        L.dee_ref_fp4_dequant_e8m0_f32.argtypes = [P, P, ctypes.c_size_t, ctypes.c_size_t, P]
        L.dee_ref_route_topk.restype = ctypes.c_int
        L.dee_ref_route_topk.argtypes = [P, ctypes.c_int, ctypes.c_int, ctypes.c_int, P, P]
        L.dee_ref_group.restype = ctypes.c_int
        L.dee_ref_group.argtypes = [P, ctypes.c_int, ctypes.c_int, ctypes.c_int, P, P, P]
        L.dee_ref_record_bytes.restype = ctypes.c_size_t
        L.dee_ref_record_bytes.argtypes = [ctypes.c_int, ctypes.c_int]
        L.dee_ref_expert_f16.argtypes = [P, ctypes.c_int, ctypes.c_int, P, ctypes.c_int, ctypes.c_float, P]
        L.dee_ref_moe_layer.restype = ctypes.c_int
        L.dee_ref_moe_layer.argtypes = [P, ctypes.c_size_t, P, ctypes.c_int, ctypes.c_int, ctypes.c_int,
                                        ctypes.c_int, P, ctypes.c_int, P, ctypes.c_float, ctypes.c_int, P]
        L.dee_ref_combine_f32.argtypes = [P, P, ctypes.c_int, ctypes.c_int, ctypes.c_int, P]
        L.dee_ref_combine_f16.argtypes = [P, P, P, ctypes.c_int, ctypes.c_int, ctypes.c_int, P]
        L.dee_ref_num_threads.restype = ctypes.c_int
        _LIB = L
    return _LIB


_REF_CUDA = None


def ref_cuda_lib() -> ctypes.CDLL | None:
    """The reference's own GPU expert path (FP4 decode + cuBLAS SwiGLU,
    oracle/ref_cuda_shim.cu), or None when oracle/_ref was not built with it."""
    global _REF_CUDA
    if _REF_CUDA is None:
        path = os.path.join(_HERE, "_ref", "libdee_ref_cuda.so")
        if not os.path.exists(path):
            return None
        L = ctypes.CDLL(path)
        P = ctypes.c_void_p
        L.dee_refcuda_moe_layer.restype = ctypes.c_int
        L.dee_refcuda_moe_layer.argtypes = [P, ctypes.c_size_t, ctypes.c_int, ctypes.c_int, ctypes.c_int,
                                            ctypes.c_int, P, ctypes.c_int, P, ctypes.c_float, P]
        _REF_CUDA = L
    return _REF_CUDA


def ref_cuda_moe_layer_raw(d_records_ptr: int, record_bytes: int, experts: int, layout: "Layout",
                           x_f16: np.ndarray, ids: np.ndarray, swiglu_limit: float = 0.0) -> np.ndarray:
    """Raw FP32 [T, K, H] from the reference's own device path (records
    already on the GPU at d_records_ptr)."""
    L = ref_cuda_lib()
    if L is None:
        raise RuntimeError("oracle/_ref/libdee_ref_cuda.so not built")
    x_f16 = np.ascontiguousarray(x_f16, dtype=np.uint16)
    ids = np.ascontiguousarray(ids, dtype=np.int32)
    T, K = ids.shape
    raw = np.zeros((T, K, layout.hidden), dtype=np.float32)
    rc = L.dee_refcuda_moe_layer(ctypes.c_void_p(d_records_ptr), record_bytes, layout.hidden, layout.inter,
                                 experts, K, _p(x_f16), T, _p(ids), swiglu_limit, _p(raw))
    if rc != 0:
        raise RuntimeError(f"reference device path failed ({rc})")
    return raw


def ref_lib() -> ctypes.CDLL | None:
    """The reference's own CPU code, or None when oracle/_ref was not built."""
    global _REF
    if _REF is None:
        path = os.path.join(_HERE, "_ref", "libdee_ref.so")
        if not os.path.exists(path):
            return None
        L = ctypes.CDLL(path)
        P = ctypes.c_void_p
        L.dee_refimpl_fp4_dequantize.argtypes = [P, P, ctypes.c_size_t, ctypes.c_size_t, P]
        L.dee_refimpl_expert.restype = ctypes.c_int
        L.dee_refimpl_expert.argtypes = [P, ctypes.c_size_t, ctypes.c_size_t, P, ctypes.c_float,
                                         ctypes.c_float, P]
        L.dee_refimpl_moe_layer.restype = ctypes.c_int
        L.dee_refimpl_moe_layer.argtypes = [P, ctypes.c_size_t, ctypes.c_size_t, ctypes.c_size_t,
                                            ctypes.c_int, P, ctypes.c_int, P, P, ctypes.c_float,
                                            ctypes.c_int, P]
        _REF = L
    return _REF


def _p(a: np.ndarray) -> int:
    assert a.flags["C_CONTIGUOUS"]
    return a.ctypes.data


# ---------------------------------------------------------------------------
# Record layout and synthetic experts
# ---------------------------------------------------------------------------

@dataclass(frozen=True)
class Layout:
    hidden: int
    inter: int

    @property
    def ih(self) -> int:
        return self.hidden * self.inter

    @property
    def w1(self) -> int: return 0
    @property
    def w3(self) -> int: return self.ih // 2
    @property
    def w2(self) -> int: return self.ih
    @property
    def s1(self) -> int: return self.ih + self.ih // 2
    @property
    def s3(self) -> int: return self.s1 + self.ih // 32
    @property
    def s2(self) -> int: return self.s3 + self.ih // 32
    @property
    def bytes(self) -> int: return self.s2 + self.ih // 32


def quantize_fp4(w: np.ndarray) -> tuple[np.ndarray, np.ndarray]:
    """FP32 [out, in] -> (packed uint8 [out, in/2], scale uint8 [out, in/32])."""
    w = np.asarray(w, dtype=np.float32)
    out, n = w.shape
    blk = w.reshape(out, n // 32, 32)
    amax = np.abs(blk).max(axis=-1)
    amax = np.maximum(amax, np.float32(6.0 * 2.0 ** -126))
    v = (amax * np.float32(1.0 / 6.0)).astype(np.float32)
    bits = v.view(np.int32)
    e = ((bits >> 23) & 0xFF) - 127 + ((bits & 0x7FFFFF) != 0).astype(np.int32)
    s = ((e + 127).astype(np.int64) << 23).astype(np.int32).view(np.float32)
    q = np.clip(blk / s[..., None], -6.0, 6.0).astype(np.float32)
    a = np.abs(q)
    mag_idx = np.select(
        [a <= 0.25, a < 0.75, a <= 1.25, a < 1.75, a <= 2.5, a < 3.5, a <= 5.0],
        [0, 1, 2, 3, 4, 5, 6], default=7).astype(np.uint8)
    nib = mag_idx | np.where((q < 0) & (mag_idx != 0), 8, 0).astype(np.uint8)
    nib = nib.reshape(out, n)
    packed = (nib[:, 0::2] | (nib[:, 1::2] << 4)).astype(np.uint8)
    scale = (e + 127).astype(np.uint8)
    return np.ascontiguousarray(packed), np.ascontiguousarray(scale)


def build_record(layout: Layout, w1p, w1s, w3p, w3s, w2p, w2s) -> np.ndarray:
    rec = np.empty(layout.bytes, dtype=np.uint8)
    for off, arr in ((layout.w1, w1p), (layout.w3, w3p), (layout.w2, w2p),
                     (layout.s1, w1s), (layout.s3, w3s), (layout.s2, w2s)):
        a = np.ascontiguousarray(arr, dtype=np.uint8).reshape(-1)
        rec[off:off + a.size] = a
    return rec


def split_record(layout: Layout, rec: np.ndarray) -> dict[str, np.ndarray]:
    H, I = layout.hidden, layout.inter
    return {
        "w1.weight": rec[layout.w1:layout.w1 + I * H // 2].reshape(I, H // 2),
        "w3.weight": rec[layout.w3:layout.w3 + I * H // 2].reshape(I, H // 2),
        "w2.weight": rec[layout.w2:layout.w2 + I * H // 2].reshape(H, I // 2),
        "w1.scale": rec[layout.s1:layout.s1 + I * H // 32].reshape(I, H // 32),
        "w3.scale": rec[layout.s3:layout.s3 + I * H // 32].reshape(I, H // 32),
        "w2.scale": rec[layout.s2:layout.s2 + I * H // 32].reshape(H, I // 32),
    }


def synthetic_records(layout: Layout, experts: int, seed: int, std: float = 0.02,
                      kind: str = "normal") -> np.ndarray:
    """[experts, record_bytes] uint8.  kind="normal": N(0, std) weights through
    quantize_fp4.  kind="bytes": uniform random nibbles with scale bytes in
    [0x7D, 0x83) (the reference's realistic range,
    dee.cpp/scripts/deepseek_v4_expert_reference.py:433-436)."""
    rng = np.random.default_rng(seed)
    H, I = layout.hidden, layout.inter
    recs = np.empty((experts, layout.bytes), dtype=np.uint8)
    for e in range(experts):
        if kind == "normal":
            parts = []
            for shape in ((I, H), (I, H), (H, I)):
                w = rng.standard_normal(shape, dtype=np.float32) * np.float32(std)
                parts.append(quantize_fp4(w))
            (p1, s1), (p3, s3), (p2, s2) = parts
        else:
            p1 = rng.integers(0, 256, (I, H // 2), dtype=np.uint8)
            p3 = rng.integers(0, 256, (I, H // 2), dtype=np.uint8)
            p2 = rng.integers(0, 256, (H, I // 2), dtype=np.uint8)
            s1 = rng.integers(0x7D, 0x83, (I, H // 32), dtype=np.uint8)
            s3 = rng.integers(0x7D, 0x83, (I, H // 32), dtype=np.uint8)
            s2 = rng.integers(0x7D, 0x83, (H, I // 32), dtype=np.uint8)
        recs[e] = build_record(layout, p1, s1, p3, s3, p2, s2)
    return recs


# ---------------------------------------------------------------------------
# Wrappers over the C restatement
# ---------------------------------------------------------------------------

def f16_bits(x: np.ndarray) -> np.ndarray:
    return np.ascontiguousarray(np.asarray(x, dtype=np.float32).astype(np.float16).view(np.uint16))


def fp4_decode_f16(packed: np.ndarray, scale: np.ndarray) -> np.ndarray:
    out, half_in = packed.shape
    dst = np.empty((out, half_in * 2), dtype=np.uint16)
    lib().dee_ref_fp4_decode_f16(_p(np.ascontiguousarray(packed)), _p(np.ascontiguousarray(scale)),
                                 _p(dst), out, half_in * 2)
    return dst


def fp4_dequant_f32(packed: np.ndarray, scale: np.ndarray) -> np.ndarray:
    out, half_in = packed.shape
    dst = np.empty((out, half_in * 2), dtype=np.float32)
    lib().dee_ref_fp4_dequant_f32(_p(np.ascontiguousarray(packed)), _p(np.ascontiguousarray(scale)),
                                  out, half_in * 2, _p(dst))
    return dst


def route_topk(logits: np.ndarray, topk: int) -> tuple[np.ndarray, np.ndarray]:
    logits = np.ascontiguousarray(logits, dtype=np.float32)
    T, E = logits.shape
    ids = np.empty((T, topk), dtype=np.int32)
    w = np.empty((T, topk), dtype=np.float32)
    rc = lib().dee_ref_route_topk(_p(logits), T, E, topk, _p(ids), _p(w))
    if rc != 0:
        raise ValueError("router denominator or selected sum not positive and finite")
    return ids, w


def route_dsv4(logits: np.ndarray, topk: int, bias: np.ndarray | None = None,
               route_scale: float = 1.5, tid2eid: np.ndarray | None = None,
               input_ids: np.ndarray | None = None) -> tuple[np.ndarray, np.ndarray, np.ndarray]:
    """DeepSeek-V4 Gate.forward restated in numpy FP32
    (dee.cpp/scripts/deepseek_v4_layer_common.py:349-403): scores =
    sqrt(softplus(logits)) with softplus threshold 20; bias shifts only the
    selection; top-k by biased score with ties to the lower id (hash layers:
    tid2eid[input_ids]); weights = selected unbiased scores / their sum *
    route_scale.  Returns (ids int32, weights f32, unbiased scores f32)."""
    x = np.ascontiguousarray(logits, dtype=np.float32)
    with np.errstate(over="ignore"):
        sp = np.where(x > 20.0, x, np.log1p(np.exp(x.astype(np.float64))).astype(np.float32))
    scores = np.sqrt(sp.astype(np.float32)).astype(np.float32)
    T, E = scores.shape
    if tid2eid is not None:
        ids = np.asarray(tid2eid)[np.asarray(input_ids)].astype(np.int32)
    else:
        sel = scores + (bias.astype(np.float32) if bias is not None else np.float32(0))
        ids = np.lexsort((np.tile(np.arange(E), (T, 1)), -sel), axis=1)[:, :topk].astype(np.int32)
    w = np.take_along_axis(scores, ids, 1)
    s = np.zeros(T, np.float32)
    for k in range(topk):
        s = (s + w[:, k]).astype(np.float32)
    w = ((w / s[:, None]).astype(np.float32) * np.float32(route_scale)).astype(np.float32)
    return ids, w, scores


def group(ids: np.ndarray, experts: int) -> tuple[np.ndarray, np.ndarray, np.ndarray]:
    ids = np.ascontiguousarray(ids, dtype=np.int32)
    T, K = ids.shape
    counts = np.empty(experts, dtype=np.int32)
    offsets = np.empty(experts + 1, dtype=np.int32)
    perm = np.empty(T * K, dtype=np.int32)
    if lib().dee_ref_group(_p(ids), T, K, experts, _p(counts), _p(offsets), _p(perm)) != 0:
        raise ValueError("expert id out of range")
    return counts, offsets, perm


def moe_layer_raw(records: np.ndarray, layout: Layout, x_f16: np.ndarray, ids: np.ndarray,
                  swiglu_limit: float = 0.0, threads: int = 0) -> np.ndarray:
    """Raw FP32 [T, K, H] expert outputs under the live FP16 chain."""
    records = np.ascontiguousarray(records, dtype=np.uint8)
    x_f16 = np.ascontiguousarray(x_f16, dtype=np.uint16)
    ids = np.ascontiguousarray(ids, dtype=np.int32)
    T, K = ids.shape
    E = records.shape[0]
    raw = np.zeros((T, K, layout.hidden), dtype=np.float32)
    rc = lib().dee_ref_moe_layer(_p(records), records.shape[1], None, layout.hidden, layout.inter,
                                 E, K, _p(x_f16), T, _p(ids), swiglu_limit, threads, _p(raw))
    if rc != 0:
        raise ValueError("expert id out of range")
    return raw


def mxfp8_layer_raw(records: np.ndarray, layout: Layout, x_f16: np.ndarray, ids: np.ndarray, act_block: int,
                    swiglu_limit: float = 0.0) -> np.ndarray:
    """Raw FP32 [T, K, H] of the MXFP8-activation variant: x quantised by
    act_quant (E4M3, UE8M0 per act_block), the records' E2M1 weights with
    their UE8M0 scales, FP64 sums of the exact FP8 x FP4 products, the live
    FP16 SwiGLU chain (swiglu_cuda.cu:46-59), the SwiGLU output quantised by
    act_quant again, then the down projection."""
    T, K = ids.shape
    H, I = layout.hidden, layout.inter
    xq, xs = act_quant(x_f16, act_block)
    xd = act_dequant_f32(xq, xs, act_block).astype(np.float64)
    raw = np.zeros((T, K, H), dtype=np.float32)

    def w64(rec, name, slot):
        w = rec[name + ".weight"]
        f32 = dequant_fp4_f32(w, rec[name + ".scale"], _scratch("f32" + slot, (w.shape[0], w.shape[1] * 2),
                                                                  np.float32))
        f64 = _scratch("f64" + slot, f32.shape, np.float64)
        np.copyto(f64, f32)
        return f64

    def one(e):
        rec = split_record(layout, records[e])
        w1, w3, w2 = w64(rec, "w1", "a"), w64(rec, "w3", "b"), w64(rec, "w2", "c")
        t, k = np.nonzero(ids == e)
        g = (xd[t] @ w1.T).astype(np.float32).astype(np.float16).astype(np.float32)
        u = (xd[t] @ w3.T).astype(np.float32).astype(np.float16).astype(np.float32)
        if swiglu_limit > 0:
            g = np.minimum(g, np.float32(swiglu_limit))
            u = np.clip(u, -swiglu_limit, swiglu_limit).astype(np.float32)
        sv = (g / (np.float32(1.0) + np.exp(-g))).astype(np.float32).astype(np.float16).astype(np.float32)
        act = (sv * u).astype(np.float32).astype(np.float16)
        aq, as_ = act_quant(act.view(np.uint16), act_block)
        ad = act_dequant_f32(aq, as_, act_block).astype(np.float64)
        raw[t, k] = (ad @ w2.T).astype(np.float32)

    _per_expert(np.unique(ids), one)
    return raw


def combine_f32(raw: np.ndarray, weights: np.ndarray) -> np.ndarray:
    raw = np.ascontiguousarray(raw, dtype=np.float32)
    weights = np.ascontiguousarray(weights, dtype=np.float32)
    T, K, H = raw.shape
    out = np.empty((T, H), dtype=np.float32)
    lib().dee_ref_combine_f32(_p(raw), _p(weights), T, K, H, _p(out))
    return out


def combine_f16(raw: np.ndarray, weights: np.ndarray, ids: np.ndarray) -> np.ndarray:
    raw = np.ascontiguousarray(raw, dtype=np.float32)
    weights = np.ascontiguousarray(weights, dtype=np.float32)
    ids64 = np.ascontiguousarray(ids, dtype=np.int64)
    T, K, H = raw.shape
    out = np.zeros((T, H), dtype=np.uint16)
    lib().dee_ref_combine_f16(_p(raw), _p(weights), _p(ids64), T, K, H, _p(out))
    return out


def rel_l2(a: np.ndarray, b: np.ndarray) -> float:
    a = np.asarray(a, dtype=np.float64)
    b = np.asarray(b, dtype=np.float64)
    den = np.linalg.norm(b.ravel())
    return float(np.linalg.norm((a - b).ravel()) / (den if den > 0 else 1.0))


# ---------------------------------------------------------------------------
# Official DeepSeek-V4 MoE semantics (FP32), numpy restatement of
# dee.cpp/scripts/deepseek_v4_moe_reference.py:35-203
# ---------------------------------------------------------------------------

_FP4_VALUES = np.array([0.0, 0.5, 1.0, 1.5, 2.0, 3.0, 4.0, 6.0,
                        -0.0, -0.5, -1.0, -1.5, -2.0, -3.0, -4.0, -6.0], dtype=np.float32)


def e8m0_f32(b: np.ndarray) -> np.ndarray:
    """2^(b - 127) in FP32 for every byte (decode_e8m0,
    deepseek_v4_expert_reference.py:49-62)."""
    with np.errstate(over="ignore"):
        return np.float32(2.0) ** (np.asarray(b, dtype=np.float32) - np.float32(127.0))


def e4m3_table() -> np.ndarray:
    """The 256 F8_E4M3 (fn) values: 1 sign, 4 exponent (bias 7), 3 mantissa
    bits, subnormals, 0x7F/0xFF NaN, no infinities."""
    b = np.arange(256)
    sign = np.where(b & 0x80, -1.0, 1.0)
    e = (b >> 3) & 0xF
    m = b & 7
    val = np.where(e == 0, m / 8.0 * 2.0 ** -6, (1.0 + m / 8.0) * 2.0 ** (e - 7.0))
    val = sign * val
    val[(e == 15) & (m == 7)] = np.nan
    return val.astype(np.float32)


def e4m3_encode(v: np.ndarray) -> np.ndarray:
    """FP32 values already clamped to [-448, 448] -> F8_E4M3 (fn) codes,
    round to nearest, ties to even mantissa (the cast of the official
    act_quant kernel, official-source/inference/kernel.py:88-93)."""
    v = np.asarray(v, dtype=np.float64)
    a = np.abs(v)
    sign = np.where(np.signbit(v), 0x80, 0).astype(np.int64)
    out = np.zeros(a.shape, dtype=np.int64)
    sub = a < 2.0 ** -6
    # subnormals: multiples of 2^-9, rounded half to even (np.rint)
    out[sub] = np.rint(a[sub] * 2.0 ** 9).astype(np.int64)  # 8 carries into the first normal code
    norm = ~sub
    e = np.floor(np.log2(a[norm])).astype(np.int64)
    m = np.rint((a[norm] / 2.0 ** e - 1.0) * 8.0).astype(np.int64)
    e = np.where(m == 8, e + 1, e)
    m = np.where(m == 8, 0, m)
    out[norm] = ((e + 7) << 3) | m
    return (out | sign).astype(np.uint8)


def act_quant(x_f16_bits: np.ndarray, block: int) -> tuple[np.ndarray, np.ndarray]:
    """The official act_quant with UE8M0 scales (kernel.py:41-103, FP32
    compute; restated in deepseek_v4_layer_common.py:213-240): per row and
    block, amax = max(|x|, 1e-4); s = 2^ceil(log2(fp32(amax * fp32(1/448))));
    q = E4M3(clamp(x / s, -448, 448)).  FP16 bits [rows, cols] -> (codes
    [rows, cols] uint8, UE8M0 bytes [rows, cols / block] uint8)."""
    x = np.asarray(x_f16_bits, dtype=np.uint16).view(np.float16).astype(np.float32)
    rows, cols = x.shape
    xb = x.reshape(rows, cols // block, block)
    amax = np.maximum(np.abs(xb).max(axis=2), np.float32(1e-4)).astype(np.float32)
    prod = (amax * np.float32(1.0 / 448.0)).astype(np.float32)
    bits = prod.view(np.uint32)
    e = ((bits >> 23) & 0xFF).astype(np.int64) - 127 + ((bits & 0x7FFFFF) != 0)
    q = np.clip(xb * np.ldexp(np.float32(1.0), -e)[:, :, None].astype(np.float32), -448.0, 448.0)
    return e4m3_encode(q.reshape(rows, cols)), (e + 127).astype(np.uint8)


def act_dequant_f32(q: np.ndarray, scales: np.ndarray, block: int) -> np.ndarray:
    """E4M3 codes x UE8M0 block scales -> FP32."""
    return e4m3_table()[q] * np.repeat(e8m0_f32(scales), block, axis=1)


_TLS = threading.local()


def _scratch(name: str, shape: tuple, dtype) -> np.ndarray:
    """A per-thread buffer reused across calls (large fresh allocations cost a
    page fault per 4 KB; the per-expert oracles reuse theirs)."""
    buf = getattr(_TLS, name, None)
    if buf is None or buf.shape != shape or buf.dtype != np.dtype(dtype):
        buf = np.empty(shape, dtype=dtype)
        setattr(_TLS, name, buf)
    return buf


def dequant_fp4_f32(packed: np.ndarray, scale: np.ndarray, out: np.ndarray | None = None) -> np.ndarray:
    """Packed E2M1 [out, in/2] (low nibble first) x UE8M0 per 32 -> FP32 [out, in]
    (dequantize_expert_weight, deepseek_v4_expert_reference.py:85-99): each
    value times 2^(b - 127) in FP32, byte 255 giving infinity.  Computed by
    dee_ref_fp4_dequant_e8m0_f32 (C), into `out` when given."""
    p = np.ascontiguousarray(packed, dtype=np.uint8)
    s = np.ascontiguousarray(scale, dtype=np.uint8)
    rows, half = p.shape
    if out is None:
        out = np.empty((rows, half * 2), dtype=np.float32)
    assert out.shape == (rows, half * 2) and out.dtype == np.float32 and out.flags.c_contiguous
    lib().dee_ref_fp4_dequant_e8m0_f32(_p(p), _p(s), rows, half * 2, _p(out))
    return out


def _per_expert(experts, fn, threads: int = 0) -> None:
    """Run fn(e) for every expert on a thread pool (numpy releases the GIL in
    its array work); fn writes disjoint outputs."""
    from concurrent.futures import ThreadPoolExecutor
    experts = list(experts)
    n = threads if threads > 0 else min(len(experts), os.cpu_count() or 1, 16)
    if n <= 1:
        for e in experts:
            fn(e)
        return
    with ThreadPoolExecutor(max_workers=n) as pool:
        for f in [pool.submit(fn, e) for e in experts]:
            f.result()


def dequant_fp8_f32(w: np.ndarray, scale: np.ndarray) -> np.ndarray:
    """F8_E4M3 [out, in] x E8M0 per 128 x 128 tile -> FP32 (dequantize_fp8_e4m3,
    deepseek_v4_moe_reference.py:35-58)."""
    v = e4m3_table()[np.asarray(w, dtype=np.uint8)]
    s = np.repeat(np.repeat(e8m0_f32(scale), 128, axis=0), 128, axis=1)[: v.shape[0], : v.shape[1]]
    return v * s


def _silu(g: np.ndarray) -> np.ndarray:
    return (g / (np.float32(1.0) + np.exp(-g))).astype(np.float32)


def _swiglu_f32(x, w1, w3, limit):
    gate = x @ w1.T
    up = x @ w3.T
    if limit > 0:
        gate = np.minimum(gate, np.float32(limit))
        up = np.clip(up, np.float32(-limit), np.float32(limit))
    return (_silu(gate) * up).astype(np.float32)


def official_layer(records: np.ndarray, layout: Layout, x: np.ndarray, ids: np.ndarray,
                   weights: np.ndarray, shared: dict | None = None,
                   swiglu_limit: float = 10.0) -> tuple[np.ndarray, np.ndarray]:
    """FP32 moe_layer_forward (deepseek_v4_moe_reference.py:113-203) given the
    route: each selection's expert with the weight applied to the
    intermediate before w2, summed, plus the shared expert (keys w1, s1, w3,
    s3, w2, s2: F8_E4M3 bytes and E8M0 scales).  Returns (moe, shared_out)."""
    x = np.asarray(x, dtype=np.float32)
    T, K = ids.shape
    # each selection's FP32 output, then summed in rank order per token
    routed = np.zeros((T, K, x.shape[1]), dtype=np.float32)

    def one(e):
        parts = split_record(layout, records[e])
        w1, w3, w2 = (dequant_fp4_f32(parts[n + ".weight"], parts[n + ".scale"],
                                      _scratch("f32" + n, (parts[n + ".weight"].shape[0],
                                                           parts[n + ".weight"].shape[1] * 2), np.float32))
                      for n in ("w1", "w3", "w2"))
        for t, r in zip(*np.nonzero(ids == e)):
            h = _swiglu_f32(x[t:t + 1], w1, w3, swiglu_limit) * np.float32(weights[t, r])
            routed[t, r] = (h @ w2.T)[0]

    _per_expert(np.unique(ids), one)
    moe = np.zeros((T, x.shape[1]), dtype=np.float32)
    for r in range(K):
        moe += routed[:, r]
    sh = np.zeros_like(moe)
    if shared is not None:
        w1 = dequant_fp8_f32(shared["w1"], shared["s1"])
        w3 = dequant_fp8_f32(shared["w3"], shared["s3"])
        w2 = dequant_fp8_f32(shared["w2"], shared["s2"])
        sh = (_swiglu_f32(x, w1, w3, swiglu_limit) @ w2.T).astype(np.float32)
    return (moe + sh).astype(np.float32), sh
