"""ctypes binding of ``libdee_b200.so`` (the C ABI in ``include/dee_b200.h``).

The library is built in-tree by ``dee_b200.build``.  Loading fails loudly
when it is missing: there is no CPU fallback for any entry point.
"""
from __future__ import annotations

import ctypes
import os

_HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(_HERE, "libdee_b200.so")

DEE_OK = 0
DEE_ERR_INVALID = -1
DEE_ERR_CUDA = -2
DEE_ERR_RANGE = -3
DEE_ERR_UNSUPPORTED = -4
DEE_ERR_DEVICE = -5
DEE_ERR_NO_BANK = -6
DEE_ERR_SCRATCH_LIMIT = -7

# Every symbol include/dee_b200.h declares, with (restype, argtypes).
P = ctypes.c_void_p
SZ = ctypes.c_size_t
I = ctypes.c_int
U32P = ctypes.POINTER(ctypes.c_uint32)


class DeeConfig(ctypes.Structure):
    _fields_ = [
        ("hidden", ctypes.c_int),
        ("inter", ctypes.c_int),
        ("num_experts", ctypes.c_int),
        ("topk", ctypes.c_int),
        ("num_layers", ctypes.c_int),
        ("device_id", ctypes.c_int),
        ("swiglu_limit", ctypes.c_float),
        ("max_tokens", ctypes.c_int),
    ]


class DeeStoreInfo(ctypes.Structure):
    _fields_ = [
        ("start_layer", ctypes.c_int),
        ("num_layers", ctypes.c_int),
        ("experts_per_layer", ctypes.c_int),
        ("segmented", ctypes.c_int),
        ("trace_indexed", ctypes.c_int),
        ("record_bytes", ctypes.c_size_t),
        ("stored_records", ctypes.c_size_t),
        ("file_count", ctypes.c_size_t),
        ("weight_offsets", ctypes.c_size_t * 3),
        ("weight_nbytes", ctypes.c_size_t * 3),
        ("weight_out", ctypes.c_size_t * 3),
        ("weight_stored_in", ctypes.c_size_t * 3),
        ("scale_offsets", ctypes.c_size_t * 3),
        ("scale_nbytes", ctypes.c_size_t * 3),
        ("scale_out", ctypes.c_size_t * 3),
        ("scale_in", ctypes.c_size_t * 3),
    ]


class DeeStoreReadStats(ctypes.Structure):
    _fields_ = [
        ("bytes_read", ctypes.c_uint64),
        ("pread_calls", ctypes.c_uint64),
        ("short_reads", ctypes.c_uint64),
        ("records", ctypes.c_uint64),
        ("files_verified", ctypes.c_uint64),
        ("seconds", ctypes.c_double),
    ]


SIGNATURES = {
    "dee_abi_config_size": (SZ, []),
    "dee_abi_version": (I, []),
    "dee_engine_create": (I, [ctypes.POINTER(DeeConfig), ctypes.POINTER(P)]),
    "dee_engine_destroy": (None, [P]),
    "dee_last_error": (ctypes.c_char_p, [P]),
    "dee_expert_bank_attach": (I, [P, I, P, I, SZ, P]),
    "dee_expert_bank_set_slots": (I, [P, I, P, P]),
    "dee_group_by_expert_device": (I, [P, P, I, I, P, P, P, P]),
    "dee_route_topk_device": (I, [P, P, I, P, P, P]),
    "dee_route_dsv4_device": (I, [P, P, P, P, P, I, ctypes.c_float, P, P, P]),
    "dee_moe_forward_batch_device": (I, [P, I, P, I, P, I, P]),
    "dee_moe_forward_combined_device": (I, [P, I, P, I, P, I, P, P, P, P]),
    "dee_moe_forward_device": (I, [P, I, P, I, P, P, I, P, P, P, P]),
    "dee_moe_forward_routed_device": (I, [P, I, P, I, P, P, P, P, P, P]),
    "dee_shared_expert_attach": (I, [P, I, P, P, P, P, P, P, I]),
    "dee_moe_forward_official_device": (I, [P, I, P, I, P, P, P, P, P]),
    "dee_ep_pack_device": (I, [P, P, I, P, I, I, I, P, P, P, P]),
    "dee_moe_forward_rows_device": (I, [P, I, P, P, I, P, P]),
    "dee_ep_combine_device": (I, [P, P, P, P, I, P, P]),
    "dee_ep_p2p_init": (I, [P, I, I, I, P, ctypes.POINTER(ctypes.c_uint64)]),
    "dee_ep_p2p_connect": (I, [P, P, P]),
    "dee_ep_p2p_dispatch_device": (I, [P, P, P, P]),
    "dee_ep_p2p_experts_device": (I, [P, I, P]),
    "dee_ep_p2p_combine_device": (I, [P, P, P, P]),
    "dee_ep_p2p_forward_device": (I, [P, I, P, P, P, P, P]),
    "dee_offload_attach": (I, [P, P, SZ, I, P, I]),
    "dee_offload_prepare_device": (I, [P, I, P, I, P, ctypes.POINTER(ctypes.c_int)]),
    "dee_offload_stats": (I, [P, ctypes.POINTER(ctypes.c_uint64)]),
    "dee_host_alloc_pinned": (I, [SZ, ctypes.POINTER(P)]),
    "dee_host_free_pinned": (I, [P]),
    "dee_stack_embed_device": (I, [P, P, P, I, I, P, P]),
    "dee_stack_rmsnorm_device": (I, [P, P, P, ctypes.c_float, I, P, P]),
    "dee_stack_router_logits_device": (I, [P, P, P, I, I, P, P]),
    "dee_stack_residual_add_device": (I, [P, P, P, I, P]),
    "dee_stack_lm_head_argmax_device": (I, [P, P, P, I, I, P, P, P]),
    "dee_records_scramble_device": (I, [P, P, I, SZ, SZ, ctypes.c_uint64, I, P]),
    "dee_engine_sync_status": (I, [P, P, U32P]),
    "dee_journal_ids_host": (I, [P, P, I]),
    "dee_fp4_decode_device": (I, [P, P, P, SZ, SZ, P]),
    "dee_fp4_quantize_device": (I, [P, SZ, SZ, P, P, P]),
    "dee_engine_launch_count": (ctypes.c_uint64, [P]),
    "dee_act_quant_device": (I, [P, I, I, I, P, P, P]),
    "dee_moe_forward_mxfp8_device": (I, [P, I, P, I, P, I, P, P, P, I, P]),
    "dee_moe_forward_noalloc": (I, [ctypes.POINTER(DeeConfig), P, SZ, I, P, I, P, P, P, P, P]),
    "dee_engine_set_profiling": (I, [P, I]),
    "dee_engine_stage_ms": (I, [P, P, I]),
    "dee_engine_set_wait_limit_ns": (I, [P, ctypes.c_uint64]),
    "dee_wait_selftest": (I, [ctypes.c_uint64, P, P]),
    "dee_offload_debug_fail_next_copy": (I, [P]),
    "dee_store_create": (I, [ctypes.POINTER(P)]),
    "dee_store_destroy": (None, [P]),
    "dee_store_open": (I, [P, ctypes.c_char_p, I, I]),
    "dee_store_close": (None, [P]),
    "dee_store_last_error": (ctypes.c_char_p, [P]),
    "dee_store_backend": (ctypes.c_char_p, [P]),
    "dee_store_identity": (ctypes.c_char_p, [P]),
    "dee_store_get_info": (I, [P, ctypes.POINTER(DeeStoreInfo)]),
    "dee_store_stats": (I, [P, ctypes.POINTER(ctypes.c_uint64)]),
    "dee_store_lookup": (I, [P, I, I, ctypes.POINTER(ctypes.c_uint64)]),
    "dee_store_materialize": (I, [P, I, I, P, SZ, ctypes.POINTER(DeeStoreReadStats)]),
    "dee_store_read_layers": (I, [P, I, I, I, I, P, SZ, I, I, ctypes.POINTER(DeeStoreReadStats)]),
    "dee_store_upload_layers_device": (I, [P, I, I, I, I, P, SZ, SZ, I, I, P,
                                           ctypes.POINTER(DeeStoreReadStats)]),
    "dee_sha256_hex": (I, [P, SZ, ctypes.c_char_p]),
}

STAGES = ("route", "permute", "gather", "gate_up", "down", "combine", "dispatch", "experts")

_lib = None


def load(build_if_missing: bool = False) -> ctypes.CDLL:
    """Load the CUDA library; raise if it is absent (no fallback path)."""
    global _lib
    if _lib is not None:
        return _lib
    if not os.path.exists(LIB_PATH):
        if build_if_missing:
            from . import build
            build.build()
        else:
            raise RuntimeError(
                f"dee_b200 CUDA library not built ({LIB_PATH}); run `python -m dee_b200.build`")
    lib = ctypes.CDLL(LIB_PATH)
    for name, (res, args) in SIGNATURES.items():
        fn = getattr(lib, name)
        fn.restype = res
        fn.argtypes = args
    if lib.dee_abi_config_size() != ctypes.sizeof(DeeConfig):
        raise ImportError("dee_b200 ABI mismatch: dee_config size differs; rebuild the library")
    _lib = lib
    return lib
