"""dee_b200 -- B200-native routed-expert MoE layer behind the pydee boundary.

The host side mirrors the reference binding ``pydee`` (so-nerdyy/dee
``dee.cpp/pydee/pydee.cpp``, ``dee.cpp/pydee/__init__.py``): an
``EngineConfig`` with the reference field names, an ``Engine`` with
``init``/``moe_forward_batch_device``/``moe_forward_combined_device``/
``last_error_message``, and ``configure``/``new_engine`` helpers.  Every
compute call goes through the C ABI of ``libdee_b200.so``; there is no CPU
path.
"""
from __future__ import annotations

import ctypes
from dataclasses import dataclass

import numpy as np

from . import _native
from .records import RecordLayout

__all__ = ["EngineConfig", "Engine", "configure", "new_engine", "RecordLayout", "DeeError"]


class DeeError(RuntimeError):
    pass


@dataclass
class EngineConfig:
    """Fields of the reference EngineConfig (engine.h:84-156) this path reads."""
    hidden: int = 4096
    inter: int = 2048
    num_experts: int = 256
    topk: int = 6
    num_layers: int = 1
    device_id: int = 0
    swiglu_limit: float = 0.0
    max_tokens: int = 64
    use_cuda: bool = True           # accepted for signature parity; always CUDA
    cache_dtype: str = "fp4"        # packed FP4 E2M1 residency (DeviceCacheDType::Fp4E2m1)

    def to_c(self) -> _native.DeeConfig:
        return _native.DeeConfig(self.hidden, self.inter, self.num_experts, self.topk,
                                 self.num_layers, self.device_id, float(self.swiglu_limit),
                                 self.max_tokens)


def _stream_handle(stream) -> int:
    if stream is None:
        return 0
    if isinstance(stream, int):
        return stream
    return int(getattr(stream, "cuda_stream", stream))


class Engine:
    """pydee.Engine-compatible MoE engine on one CUDA device."""

    def __init__(self) -> None:
        self._lib = _native.load()
        self._h = ctypes.c_void_p()
        self.cfg: EngineConfig | None = None
        self._banks: dict[int, object] = {}
        self._shared: dict[int, tuple] = {}

    # -- lifecycle -------------------------------------------------------
    def init(self, cfg: EngineConfig) -> bool:
        c = cfg.to_c()
        rc = self._lib.dee_engine_create(ctypes.byref(c), ctypes.byref(self._h))
        if rc != _native.DEE_OK:
            self._h = ctypes.c_void_p()
            return False
        self.cfg = cfg
        return True

    def close(self) -> None:
        if self._h:
            self._lib.dee_engine_destroy(self._h)
            self._h = ctypes.c_void_p()

    def __del__(self) -> None:
        try:
            self.close()
        except Exception:
            pass

    def _check(self, rc: int, what: str) -> None:
        if rc != _native.DEE_OK:
            raise DeeError(f"{what} failed (status {rc}): {self.last_error_message()}")

    def last_error_message(self) -> str:
        if not self._h:
            return "engine not initialised"
        msg = self._lib.dee_last_error(self._h)
        return msg.decode() if msg else ""

    def hidden_dim(self) -> int:
        return self.cfg.hidden

    def inter_dim(self) -> int:
        return self.cfg.inter

    def launch_count(self) -> int:
        return int(self._lib.dee_engine_launch_count(self._h))

    def set_wait_limit(self, seconds: float) -> None:
        """Limit of this engine's waits on other ranks' flags (100 us .. 2 s):
        a rank that never arrives is reported by sync_status (bit 6) instead
        of stalling the stream."""
        self._check(self._lib.dee_engine_set_wait_limit_ns(self._h, int(seconds * 1e9)),
                    "dee_engine_set_wait_limit_ns")

    def set_profiling(self, enable: bool) -> None:
        self._check(self._lib.dee_engine_set_profiling(self._h, int(bool(enable))),
                    "dee_engine_set_profiling")

    def stage_ms(self) -> dict[str, float]:
        """Per-stage milliseconds of the most recent profiled forward."""
        buf = (ctypes.c_float * len(_native.STAGES))()
        n = self._lib.dee_engine_stage_ms(self._h, buf, len(_native.STAGES))
        if n < 0:
            self._check(n, "dee_engine_stage_ms")
        return {name: float(buf[i]) for i, name in enumerate(_native.STAGES) if buf[i] >= 0}

    # -- expert residency ------------------------------------------------
    def attach_bank(self, layer: int, records, slot_of_expert: np.ndarray | None = None) -> None:
        """records: device uint8 tensor [n_slots, record_bytes] (DEE4 layout)."""
        n_slots, record_bytes = int(records.shape[0]), int(records.shape[1])
        slots = None
        if slot_of_expert is not None:
            slots = np.ascontiguousarray(slot_of_expert, dtype=np.int32)
        rc = self._lib.dee_expert_bank_attach(
            self._h, layer, ctypes.c_void_p(records.data_ptr()), n_slots, record_bytes,
            slots.ctypes.data_as(ctypes.c_void_p) if slots is not None else None)
        self._check(rc, "dee_expert_bank_attach")
        self._banks[layer] = records  # keep the storage alive

    def set_slots(self, layer: int, slot_of_expert: np.ndarray, stream=None) -> None:
        slots = np.ascontiguousarray(slot_of_expert, dtype=np.int32)
        rc = self._lib.dee_expert_bank_set_slots(self._h, layer, slots.ctypes.data_as(ctypes.c_void_p),
                                                 ctypes.c_void_p(_stream_handle(stream)))
        self._check(rc, "dee_expert_bank_set_slots")

    # -- the reference's binding surface ---------------------------------
    def moe_forward_batch_device(self, layer: int, d_h_in_ptr: int, tokens: int,
                                 expert_ids: np.ndarray, topk: int, d_experts_out_ptr: int) -> bool:
        """pydee.Engine.moe_forward_batch_device (pydee.cpp:430-467)."""
        ids = np.ascontiguousarray(expert_ids, dtype=np.int32)
        if ids.ndim != 2 or ids.shape[0] != tokens or ids.shape[1] != topk:
            raise RuntimeError("expert_ids must have shape [tokens, topk]")
        # pydee's binding accepts only the configured topk (pydee.cpp:443-444);
        # the C entry also takes fewer, as Engine::moe_forward_batch_device does
        if topk != self.cfg.topk:
            raise RuntimeError("expert_ids topk does not match EngineConfig.topk")
        rc = self._lib.dee_moe_forward_batch_device(
            self._h, layer, ctypes.c_void_p(d_h_in_ptr), tokens, ids.ctypes.data_as(ctypes.c_void_p),
            topk, ctypes.c_void_p(d_experts_out_ptr))
        return rc == _native.DEE_OK

    def moe_forward_combined_device(self, layer: int, d_h_in_ptr: int, tokens: int,
                                    d_expert_ids_ptr: int, topk: int, d_weights_ptr: int,
                                    d_output_ptr: int, d_raw_trace_ptr: int,
                                    external_stream_ptr: int) -> bool:
        """pydee.Engine.moe_forward_combined_device (pydee.cpp:468-509)."""
        if topk != self.cfg.topk:  # pydee.cpp:479-482
            raise RuntimeError("expert_ids topk does not match EngineConfig.topk")
        rc = self._lib.dee_moe_forward_combined_device(
            self._h, layer, ctypes.c_void_p(d_h_in_ptr), tokens, ctypes.c_void_p(d_expert_ids_ptr),
            topk, ctypes.c_void_p(d_weights_ptr), ctypes.c_void_p(d_output_ptr),
            ctypes.c_void_p(d_raw_trace_ptr or 0), ctypes.c_void_p(external_stream_ptr or 0))
        return rc == _native.DEE_OK

    # -- device-resident routing and the one-call layer ------------------
    def route_topk_device(self, d_logits_ptr: int, tokens: int, d_ids_ptr: int, d_weights_ptr: int,
                          stream=None) -> None:
        rc = self._lib.dee_route_topk_device(self._h, ctypes.c_void_p(d_logits_ptr), tokens,
                                             ctypes.c_void_p(d_ids_ptr), ctypes.c_void_p(d_weights_ptr),
                                             ctypes.c_void_p(_stream_handle(stream)))
        self._check(rc, "dee_route_topk_device")

    def route_dsv4_device(self, d_logits_ptr: int, tokens: int, d_ids_ptr: int, d_weights_ptr: int, *,
                          d_bias_ptr: int = 0, d_tid2eid_ptr: int = 0, d_input_ids_ptr: int = 0,
                          route_scale: float = 1.5, stream=None) -> None:
        rc = self._lib.dee_route_dsv4_device(
            self._h, ctypes.c_void_p(d_logits_ptr), ctypes.c_void_p(d_bias_ptr or 0),
            ctypes.c_void_p(d_tid2eid_ptr or 0), ctypes.c_void_p(d_input_ids_ptr or 0), tokens,
            float(route_scale), ctypes.c_void_p(d_ids_ptr), ctypes.c_void_p(d_weights_ptr),
            ctypes.c_void_p(_stream_handle(stream)))
        self._check(rc, "dee_route_dsv4_device")

    def moe_forward_routed_device(self, layer: int, d_x_ptr: int, tokens: int, d_logits_ptr: int, d_ids_ptr: int,
                                  d_weights_ptr: int, *, d_out_ptr: int = 0, d_raw_ptr: int = 0,
                                  stream=None) -> None:
        """Route (softmax top-k of device logits [T, E] into d_ids / d_weights)
        and run the layer in one call; decode-sized batches route inside the
        grouping kernel."""
        rc = self._lib.dee_moe_forward_routed_device(
            self._h, layer, ctypes.c_void_p(d_x_ptr), tokens, ctypes.c_void_p(d_logits_ptr),
            ctypes.c_void_p(d_ids_ptr), ctypes.c_void_p(d_weights_ptr), ctypes.c_void_p(d_out_ptr or 0),
            ctypes.c_void_p(d_raw_ptr or 0), ctypes.c_void_p(_stream_handle(stream)))
        self._check(rc, "dee_moe_forward_routed_device")

    def moe_forward_device(self, layer: int, d_x_ptr: int, tokens: int, *, d_ids_ptr: int = 0,
                           h_ids: np.ndarray | None = None, d_weights_ptr: int = 0,
                           d_out_ptr: int = 0, d_raw_ptr: int = 0, stream=None) -> None:
        hid = None
        if h_ids is not None:
            hid = np.ascontiguousarray(h_ids, dtype=np.int32)
        rc = self._lib.dee_moe_forward_device(
            self._h, layer, ctypes.c_void_p(d_x_ptr), tokens, ctypes.c_void_p(d_ids_ptr or 0),
            hid.ctypes.data_as(ctypes.c_void_p) if hid is not None else None, self.cfg.topk,
            ctypes.c_void_p(d_weights_ptr or 0), ctypes.c_void_p(d_out_ptr or 0),
            ctypes.c_void_p(d_raw_ptr or 0), ctypes.c_void_p(_stream_handle(stream)))
        self._check(rc, "dee_moe_forward_device")

    def moe_forward_mxfp8_device(self, layer: int, d_x_ptr: int, tokens: int, d_ids_ptr: int, d_raw_ptr: int = 0,
                                 *, d_weights_ptr: int = 0, d_out_ptr: int = 0, act_block: int = 32,
                                 stream=None) -> None:
        """The MXFP8-activation variant of moe_forward_device: E4M3 token rows
        and SwiGLU output with UE8M0 scales per act_block (32 MX, 128 the
        official act_quant), block-scaled tcgen05 GEMMs on the FP4 records."""
        rc = self._lib.dee_moe_forward_mxfp8_device(
            self._h, layer, ctypes.c_void_p(d_x_ptr), tokens, ctypes.c_void_p(d_ids_ptr), self.cfg.topk,
            ctypes.c_void_p(d_weights_ptr or 0), ctypes.c_void_p(d_out_ptr or 0), ctypes.c_void_p(d_raw_ptr or 0),
            act_block, ctypes.c_void_p(_stream_handle(stream)))
        self._check(rc, "dee_moe_forward_mxfp8_device")

    # -- official DeepSeek-V4 semantics ---------------------------------------
    def attach_shared_expert(self, layer: int, w1, w1_scale, w3, w3_scale, w2, w2_scale) -> None:
        """Device tensors: F8_E4M3 (uint8 view) W1, W3 [inter, H], W2 [H, inter]
        and their E8M0 scale bytes [ceil(rows/128), ceil(cols/128)].  The
        tensors must stay alive while the engine uses them."""
        inter = int(w1.shape[0])
        rc = self._lib.dee_shared_expert_attach(
            self._h, layer, ctypes.c_void_p(w1.data_ptr()), ctypes.c_void_p(w1_scale.data_ptr()),
            ctypes.c_void_p(w3.data_ptr()), ctypes.c_void_p(w3_scale.data_ptr()),
            ctypes.c_void_p(w2.data_ptr()), ctypes.c_void_p(w2_scale.data_ptr()), inter)
        self._check(rc, "dee_shared_expert_attach")
        self._shared[layer] = (w1, w1_scale, w3, w3_scale, w2, w2_scale)  # keep the storage alive

    def moe_forward_official_device(self, layer: int, d_x_ptr: int, tokens: int, d_ids_ptr: int,
                                    d_weights_ptr: int, d_out_ptr: int, d_shared_out_ptr: int = 0,
                                    stream=None) -> None:
        rc = self._lib.dee_moe_forward_official_device(
            self._h, layer, ctypes.c_void_p(d_x_ptr), tokens, ctypes.c_void_p(d_ids_ptr),
            ctypes.c_void_p(d_weights_ptr), ctypes.c_void_p(d_out_ptr),
            ctypes.c_void_p(d_shared_out_ptr or 0), ctypes.c_void_p(_stream_handle(stream)))
        self._check(rc, "dee_moe_forward_official_device")

    # -- expert parallelism (see dee_b200.ep for the whole layer) -----------
    def ep_pack_device(self, d_ids_ptr: int, tokens: int, d_x_ptr: int, ranks: int,
                       experts_per_rank: int, capacity: int, d_send_rows_ptr: int,
                       d_send_expert_ptr: int, d_slot_of_pos_ptr: int, stream=None) -> None:
        rc = self._lib.dee_ep_pack_device(
            self._h, ctypes.c_void_p(d_ids_ptr), tokens, ctypes.c_void_p(d_x_ptr), ranks,
            experts_per_rank, capacity, ctypes.c_void_p(d_send_rows_ptr),
            ctypes.c_void_p(d_send_expert_ptr), ctypes.c_void_p(d_slot_of_pos_ptr),
            ctypes.c_void_p(_stream_handle(stream)))
        self._check(rc, "dee_ep_pack_device")

    def moe_forward_rows_device(self, layer: int, d_rows_ptr: int, d_expert_ptr: int, rows: int,
                                d_raw_ptr: int, stream=None) -> None:
        rc = self._lib.dee_moe_forward_rows_device(
            self._h, layer, ctypes.c_void_p(d_rows_ptr), ctypes.c_void_p(d_expert_ptr), rows,
            ctypes.c_void_p(d_raw_ptr), ctypes.c_void_p(_stream_handle(stream)))
        self._check(rc, "dee_moe_forward_rows_device")

    def ep_combine_device(self, d_back_ptr: int, d_slot_of_pos_ptr: int, d_weights_ptr: int,
                          tokens: int, d_out_ptr: int, stream=None) -> None:
        rc = self._lib.dee_ep_combine_device(
            self._h, ctypes.c_void_p(d_back_ptr), ctypes.c_void_p(d_slot_of_pos_ptr),
            ctypes.c_void_p(d_weights_ptr), tokens, ctypes.c_void_p(d_out_ptr),
            ctypes.c_void_p(_stream_handle(stream)))
        self._check(rc, "dee_ep_combine_device")

    # -- offload tier --------------------------------------------------------
    def offload_attach(self, h_records, layers: int, d_pool, pool_slots: int) -> None:
        """h_records: pinned host uint8 tensor [layers * E, record_bytes];
        d_pool: device uint8 tensor [pool_slots, record_bytes]."""
        rc = self._lib.dee_offload_attach(self._h, ctypes.c_void_p(h_records.data_ptr()),
                                          int(h_records.shape[-1]), layers, ctypes.c_void_p(d_pool.data_ptr()),
                                          pool_slots)
        self._check(rc, "dee_offload_attach")
        self._offload = (h_records, d_pool)  # keep the storage alive

    def offload_prepare_device(self, layer: int, d_ids_ptr: int, tokens: int, stream=None) -> int:
        cold = ctypes.c_int(0)
        rc = self._lib.dee_offload_prepare_device(self._h, layer, ctypes.c_void_p(d_ids_ptr), tokens,
                                                  ctypes.c_void_p(_stream_handle(stream)), ctypes.byref(cold))
        self._check(rc, "dee_offload_prepare_device")
        return cold.value

    def offload_debug_fail_next_copy(self) -> None:
        """Test hook: the next cold record copy fails as if it could not be
        queued (the reference's AsyncPrefetcher.debug_fail_next_submit)."""
        self._check(self._lib.dee_offload_debug_fail_next_copy(self._h), "dee_offload_debug_fail_next_copy")

    def offload_stats(self) -> dict:
        out = (ctypes.c_uint64 * 4)()
        self._lib.dee_offload_stats(self._h, out)
        return {"lookups": out[0], "hits": out[1], "cold_reads": out[2], "bytes": out[3]}

    # -- expert parallelism over NVLink peer memory ---------------------------
    def ep_p2p_init(self, ranks: int, rank: int, tokens: int) -> tuple[bytes, int]:
        """Allocate and export this rank's exchange block: (IPC handle, device address)."""
        handle = ctypes.create_string_buffer(64)
        block = ctypes.c_uint64(0)
        rc = self._lib.dee_ep_p2p_init(self._h, ranks, rank, tokens, handle, ctypes.byref(block))
        self._check(rc, "dee_ep_p2p_init")
        return handle.raw, block.value

    def ep_p2p_connect(self, handles: list[bytes] | None, blocks: list[int] | None = None) -> None:
        hbuf = ctypes.create_string_buffer(b"".join(handles)) if handles else None
        barr = (ctypes.c_uint64 * len(blocks))(*blocks) if blocks else None
        rc = self._lib.dee_ep_p2p_connect(self._h, hbuf, barr)
        self._check(rc, "dee_ep_p2p_connect")

    def ep_p2p_dispatch_device(self, d_x_ptr: int, d_ids_ptr: int, stream=None) -> None:
        rc = self._lib.dee_ep_p2p_dispatch_device(self._h, ctypes.c_void_p(d_x_ptr),
                                                  ctypes.c_void_p(d_ids_ptr),
                                                  ctypes.c_void_p(_stream_handle(stream)))
        self._check(rc, "dee_ep_p2p_dispatch_device")

    def ep_p2p_experts_device(self, layer: int, stream=None) -> None:
        rc = self._lib.dee_ep_p2p_experts_device(self._h, layer, ctypes.c_void_p(_stream_handle(stream)))
        self._check(rc, "dee_ep_p2p_experts_device")

    def ep_p2p_combine_device(self, d_weights_ptr: int, d_out_ptr: int, stream=None) -> None:
        rc = self._lib.dee_ep_p2p_combine_device(self._h, ctypes.c_void_p(d_weights_ptr),
                                                 ctypes.c_void_p(d_out_ptr),
                                                 ctypes.c_void_p(_stream_handle(stream)))
        self._check(rc, "dee_ep_p2p_combine_device")

    def ep_p2p_forward_device(self, layer: int, d_x_ptr: int, d_ids_ptr: int, d_weights_ptr: int,
                              d_out_ptr: int, stream=None) -> None:
        rc = self._lib.dee_ep_p2p_forward_device(self._h, layer, ctypes.c_void_p(d_x_ptr),
                                                 ctypes.c_void_p(d_ids_ptr), ctypes.c_void_p(d_weights_ptr),
                                                 ctypes.c_void_p(d_out_ptr),
                                                 ctypes.c_void_p(_stream_handle(stream)))
        self._check(rc, "dee_ep_p2p_forward_device")

    def sync_status(self, stream=None) -> int:
        st = ctypes.c_uint32(0)
        rc = self._lib.dee_engine_sync_status(self._h, ctypes.c_void_p(_stream_handle(stream)),
                                              ctypes.byref(st))
        if rc not in (_native.DEE_OK, _native.DEE_ERR_DEVICE):
            self._check(rc, "dee_engine_sync_status")
        return int(st.value)

    def journal_ids(self, tokens: int) -> np.ndarray:
        """The int32 [tokens, topk] ids the last forward consumed."""
        out = np.empty((tokens, self.cfg.topk), dtype=np.int32)
        n = self._lib.dee_journal_ids_host(self._h, out.ctypes.data_as(ctypes.c_void_p), out.size)
        if n != out.size:
            raise DeeError(f"journal ids unavailable ({n} of {out.size})")
        return out


def configure(num_experts: int, num_layers: int, hidden: int, inter: int, topk: int = 6,
              swiglu_limit: float = 0.0, device_id: int = 0, max_tokens: int = 64,
              **_ignored) -> EngineConfig:
    """pydee.configure (pydee/__init__.py:66-107) for the packed-FP4 path."""
    return EngineConfig(hidden=hidden, inter=inter, num_experts=num_experts, topk=topk,
                        num_layers=num_layers, device_id=device_id, swiglu_limit=swiglu_limit,
                        max_tokens=max_tokens)


def new_engine(cfg: EngineConfig) -> Engine:
    engine = Engine()
    if not engine.init(cfg):
        raise RuntimeError("dee_b200 engine creation failed (unsupported shape or CUDA error)")
    return engine
