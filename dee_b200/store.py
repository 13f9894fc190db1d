"""DEE4 expert stores on disk: the native reader and a writer of the three shapes.

Reader.  ``Dee4Store`` drives the native reader of ``libdee_b200``
(``dee_store_*``), which restates ``Dee4ExpertStore``
(dee.cpp/include/dee/expert_store.h:286-409, dee.cpp/src/expert_store.cpp:
786-1230): same metadata keys, same fail-closed checks and messages, same
record lookup.  Records move with parallel ``pread`` straight into pinned
host memory (``read_layers``: the offload tier's record block) or through a
pinned staging ring into HBM (``upload_layers``: a resident expert bank).

Writer.  ``write_store`` emits what the reference's builders emit
(dee.cpp/tools/phase3/p3_builder.py: ``build_segmented`` 285-460,
``build_single`` 463-578, ``_store_metadata`` 580-625;
dee.cpp/kaggle/deepseek-v4-flash-0731/repack_to_dee4.py:42-55,120-180 for
the component table and the dee4-v3-trace record index): ``metadata.json``,
the data file(s) and ``integrity.jsonl`` with one line per record.
"""
from __future__ import annotations

import ctypes
import hashlib
import json
import os
from typing import Callable, Iterable

from . import _native
from .records import RecordLayout

CODEC = "deepseek-fp4-e2m1-e8m0"
DATA_FILE = "experts.dee4"
INTEGRITY_FILE = "integrity.jsonl"
SEGMENT_TEMPLATE = "experts-bucket-{bucket:02d}.dee4"
FORMATS = ("dee4-v2", "dee4-v3-trace", "dee4-v4-segmented")


class StoreError(RuntimeError):
    """A store that failed to open or a record that could not be read."""


def sha256_hex(data) -> str:
    """SHA-256 through the native implementation (the seal function)."""
    lib = _native.load()
    buf = (ctypes.c_char * len(data)).from_buffer_copy(bytes(data)) if len(data) else None
    out = ctypes.create_string_buffer(65)
    rc = lib.dee_sha256_hex(ctypes.cast(buf, ctypes.c_void_p) if buf is not None else None, len(data), out)
    if rc != 0:
        raise StoreError(f"dee_sha256_hex failed ({rc})")
    return out.value.decode()


def layout_components(layout: RecordLayout) -> list[dict]:
    """The record's six components in DEE4 order (w1, w3, w2 weights, then
    their UE8M0 scales), with the shapes the checkpoint stores them in."""
    H, I = layout.hidden, layout.inter
    off = layout.offsets
    shapes = {"w1": (I, H), "w3": (I, H), "w2": (H, I)}
    comps = []
    for proj in ("w1", "w3", "w2"):
        rows, cols = shapes[proj]
        comps.append({"projection": proj, "kind": "weight", "dtype": "I8", "shape": [rows, cols // 2],
                      "offset": off[proj], "nbytes": rows * cols // 2})
    for proj in ("w1", "w3", "w2"):
        rows, cols = shapes[proj]
        comps.append({"projection": proj, "kind": "scale", "dtype": "F8_E8M0", "shape": [rows, cols // 32],
                      "offset": off["s" + proj[1]], "nbytes": rows * cols // 32})
    return comps


def _layout_fields(layout: RecordLayout) -> dict:
    comps = layout_components(layout)
    w = [c for c in comps if c["kind"] == "weight"]
    s = [c for c in comps if c["kind"] == "scale"]
    return {
        "record_bytes": layout.bytes,
        "group_size": 32,
        "components": comps,
        "weight_offsets": [c["offset"] for c in w],
        "weight_nbytes": [c["nbytes"] for c in w],
        "weight_out": [c["shape"][0] for c in w],
        "weight_stored_in": [c["shape"][1] for c in w],
        "scale_offsets": [c["offset"] for c in s],
        "scale_nbytes": [c["nbytes"] for c in s],
        "scale_out": [c["shape"][0] for c in s],
        "scale_in": [c["shape"][1] for c in s],
    }


def _write_json(path: str, payload: dict) -> None:
    tmp = path + ".tmp"
    with open(tmp, "w", encoding="utf-8", newline="\n") as fh:
        json.dump(payload, fh, indent=2)
        fh.write("\n")
    os.replace(tmp, path)


def write_store(out_dir: str, layout: RecordLayout, num_layers: int, experts_per_layer: int,
                layer_records: Callable[[int], object], *, fmt: str = "dee4-v4-segmented",
                start_layer: int = 0, trace_pairs: Iterable[tuple[int, int]] | None = None,
                trace_hashes: dict | None = None) -> dict:
    """Write a DEE4 store; returns its metadata.

    layer_records(layer) -> a buffer of experts_per_layer * record_bytes bytes
    (numpy uint8 [E, record_bytes] or bytes) holding layer `layer`'s records.
    fmt "dee4-v4-segmented" writes one sealed segment per layer, "dee4-v2"
    one dense file, "dee4-v3-trace" one file of the (layer, expert) pairs in
    `trace_pairs` (sorted, unique) with the record table in metadata.json.
    """
    if fmt not in FORMATS:
        raise ValueError(f"unknown DEE4 format {fmt!r}")
    rb = layout.bytes
    os.makedirs(out_dir, exist_ok=True)
    meta = {
        "format": fmt,
        "codec": CODEC,
        "source_repository": "synthetic",
        "source_revision": "dee_b200",
        "start_layer": start_layer,
        "num_layers": num_layers,
        "experts_per_layer": experts_per_layer,
        "total_experts": num_layers * experts_per_layer,
        **_layout_fields(layout),
    }
    integrity = []

    def layer_view(layer: int) -> memoryview:
        mv = memoryview(layer_records(layer)).cast("B")
        if mv.nbytes != experts_per_layer * rb:
            raise ValueError(f"layer {layer}: {mv.nbytes} bytes, expected {experts_per_layer * rb}")
        return mv

    def note(layer, expert, index, blob):
        integrity.append({"bucket": layer - start_layer, "layer": layer, "domain": "main", "expert": expert,
                          "record_index": index, "record_offset": index * rb, "record_bytes": rb,
                          "record_sha256": hashlib.sha256(blob).hexdigest(), "component_sha256": {},
                          "source_shards": ["synthetic"]})

    if fmt == "dee4-v4-segmented":
        os.makedirs(os.path.join(out_dir, "segments"), exist_ok=True)
        segments = []
        for b in range(num_layers):
            layer = start_layer + b
            mv = layer_view(layer)
            name = SEGMENT_TEMPLATE.format(bucket=b)
            with open(os.path.join(out_dir, "segments", name), "wb") as fh:
                fh.write(mv)
            for e in range(experts_per_layer):
                note(layer, e, b * experts_per_layer + e, mv[e * rb:(e + 1) * rb])
            segments.append({"file": f"segments/{name}", "bucket": b, "domain": "main",
                             "first_record": b * experts_per_layer, "record_count": experts_per_layer,
                             "bytes": experts_per_layer * rb, "sha256": hashlib.sha256(mv).hexdigest()})
        meta["segments"] = segments
        meta["data_file"] = None
    else:
        path = os.path.join(out_dir, DATA_FILE)
        data_hash = hashlib.sha256()
        if fmt == "dee4-v2":
            with open(path, "wb") as fh:
                for b in range(num_layers):
                    layer = start_layer + b
                    mv = layer_view(layer)
                    fh.write(mv)
                    data_hash.update(mv)
                    for e in range(experts_per_layer):
                        note(layer, e, b * experts_per_layer + e, mv[e * rb:(e + 1) * rb])
        else:
            pairs = sorted(set(trace_pairs or ()))
            if not pairs:
                raise ValueError("dee4-v3-trace needs a non-empty trace_pairs")
            records = []
            cached = (None, None)
            with open(path, "wb") as fh:
                for idx, (layer, e) in enumerate(pairs):
                    if cached[0] != layer:
                        cached = (layer, layer_view(layer))
                    blob = cached[1][e * rb:(e + 1) * rb]
                    fh.write(blob)
                    data_hash.update(blob)
                    note(layer, e, idx, blob)
                    records.append({"layer": layer, "expert": e, "record_index": idx})
            th = trace_hashes or {}
            meta["total_experts"] = len(records)
            meta["records"] = records
            meta["trace_journal_sha256"] = th.get("journal", hashlib.sha256(b"").hexdigest())
            meta["trace_final_chain_sha256"] = th.get("final_chain", hashlib.sha256(b"").hexdigest())
            meta["selection_sha256"] = th.get("selection", hashlib.sha256(
                json.dumps(pairs).encode()).hexdigest())
        meta["data_file"] = DATA_FILE
        meta["data_sha256"] = data_hash.hexdigest()
    meta["integrity_file"] = INTEGRITY_FILE
    with open(os.path.join(out_dir, INTEGRITY_FILE), "w", encoding="utf-8", newline="\n") as fh:
        for line in integrity:
            fh.write(json.dumps(line, sort_keys=True) + "\n")
    _write_json(os.path.join(out_dir, "metadata.json"), meta)
    return meta


VERIFY_SEALS = 1
SEAL_DROP_PAGES = 2


class Dee4Store:
    """An open DEE4 store (Dee4ExpertStore, expert_store.h:316-409).

    Opening fails closed with StoreError carrying the reader's message.
    `verify_segment_hashes` re-hashes every segment of a segmented store at
    open (Dee4OpenOptions::verify_segment_hashes, default true);
    `seal_reads_through_page_cache` drops each segment from the page cache
    after hashing it (Dee4OpenOptions::seal_reads_through_page_cache).
    `threads` host threads hash segments and read records in parallel.  A
    fill with verify=True checks the seal of every file it reads whole as the
    bytes stream in, so a store opened without verification and filled whole
    is sealed in one pass over the disk.
    """

    def __init__(self, path: str, *, verify_segment_hashes: bool = True,
                 seal_reads_through_page_cache: bool = False, threads: int = 0):
        self._lib = _native.load()
        self.threads = threads if threads > 0 else max(1, min(32, os.cpu_count() or 1))
        h = ctypes.c_void_p()
        if self._lib.dee_store_create(ctypes.byref(h)) != 0:
            raise StoreError("dee_store_create failed")
        self._h = h
        options = (VERIFY_SEALS if verify_segment_hashes else 0) | \
            (SEAL_DROP_PAGES if seal_reads_through_page_cache else 0)
        rc = self._lib.dee_store_open(h, os.fsencode(path), options, self.threads)
        if rc != 0:
            msg = self.last_error()
            self.close()
            raise StoreError(msg)
        info = _native.DeeStoreInfo()
        self._lib.dee_store_get_info(h, ctypes.byref(info))
        self.start_layer = info.start_layer
        self.num_layers = info.num_layers
        self.experts_per_layer = info.experts_per_layer
        self.segmented = bool(info.segmented)
        self.trace_indexed = bool(info.trace_indexed)
        self.record_bytes = info.record_bytes
        self.stored_records = info.stored_records
        self.file_count = info.file_count
        self.layout = {k: list(getattr(info, k)) for k in (
            "weight_offsets", "weight_nbytes", "weight_out", "weight_stored_in",
            "scale_offsets", "scale_nbytes", "scale_out", "scale_in")}

    # -- lifetime ------------------------------------------------------------
    def close(self) -> None:
        if getattr(self, "_h", None):
            self._lib.dee_store_destroy(self._h)
            self._h = None

    def __enter__(self):
        return self

    def __exit__(self, *exc):
        self.close()

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    # -- identity ------------------------------------------------------------
    def last_error(self) -> str:
        return self._lib.dee_store_last_error(self._h).decode()

    @property
    def backend(self) -> str:
        return self._lib.dee_store_backend(self._h).decode()

    @property
    def identity(self) -> str:
        return self._lib.dee_store_identity(self._h).decode()

    def stats(self) -> dict:
        out = (ctypes.c_uint64 * 4)()
        self._lib.dee_store_stats(self._h, out)
        return {"lookups": out[0], "lookup_failures": out[1], "records_read": out[2], "bytes_read": out[3]}

    def check_layout(self, layout: RecordLayout) -> None:
        """Fail loudly unless the store's records have this engine layout."""
        want = {k: v for k, v in _layout_fields(layout).items() if k in self.layout}
        if self.record_bytes != layout.bytes or want != self.layout:
            raise StoreError(f"store record layout {self.layout} (record_bytes {self.record_bytes}) does not "
                             f"match H={layout.hidden}, I={layout.inter}")

    # -- records -------------------------------------------------------------
    def lookup(self, layer: int, expert: int) -> int:
        """The record index of (layer, expert); StoreError if absent."""
        idx = ctypes.c_uint64()
        rc = self._lib.dee_store_lookup(self._h, layer, expert, ctypes.byref(idx))
        if rc != 0:
            raise StoreError(f"record (layer {layer}, expert {expert}) is not in the store")
        return idx.value

    def materialize(self, layer: int, expert: int, dst=None):
        """One record into dst (a writable buffer of record_bytes; a new
        bytearray by default)."""
        if dst is None:
            dst = bytearray(self.record_bytes)
        ptr, n = _buffer_ptr(dst)
        st = _native.DeeStoreReadStats()
        rc = self._lib.dee_store_materialize(self._h, layer, expert, ptr, n, ctypes.byref(st))
        if rc != 0:
            raise StoreError(self.last_error())
        return dst

    def layer_bytes(self, layers: int = 1) -> int:
        return layers * self.experts_per_layer * self.record_bytes

    def _experts(self, first_expert: int, experts: int | None) -> tuple[int, int]:
        return first_expert, (self.experts_per_layer - first_expert) if experts is None else experts

    def read_layers(self, first_layer: int, layers: int, dst_ptr: int, dst_bytes: int, *,
                    first_expert: int = 0, experts: int | None = None, verify: bool = False) -> dict:
        """Experts [first_expert, first_expert+experts) (default: all) of
        layers [first_layer, first_layer+layers) into host memory at dst_ptr
        as [layer][expert][record_bytes]."""
        fe, ne = self._experts(first_expert, experts)
        st = _native.DeeStoreReadStats()
        rc = self._lib.dee_store_read_layers(self._h, first_layer, layers, fe, ne, ctypes.c_void_p(dst_ptr),
                                             dst_bytes, self.threads, int(verify), ctypes.byref(st))
        if rc != 0:
            raise StoreError(self.last_error())
        return _stats(st)

    def upload_layers(self, first_layer: int, layers: int, d_ptr: int, d_bytes: int, stream=None, *,
                      first_expert: int = 0, experts: int | None = None, staging_bytes: int = 512 << 20,
                      verify: bool = False) -> dict:
        """The same records into device memory at d_ptr through pinned
        staging buffers; returns after the copies completed."""
        fe, ne = self._experts(first_expert, experts)
        st = _native.DeeStoreReadStats()
        s = getattr(stream, "cuda_stream", stream)
        rc = self._lib.dee_store_upload_layers_device(self._h, first_layer, layers, fe, ne, ctypes.c_void_p(d_ptr),
                                                      d_bytes, staging_bytes, self.threads, int(verify),
                                                      ctypes.c_void_p(s) if s else None, ctypes.byref(st))
        if rc != 0:
            raise StoreError(self.last_error())
        return _stats(st)


def _stats(st) -> dict:
    gbs = st.bytes_read / st.seconds / 1e9 if st.seconds > 0 else 0.0
    return {"bytes_read": st.bytes_read, "pread_calls": st.pread_calls, "short_reads": st.short_reads,
            "records": st.records, "files_verified": st.files_verified, "seconds": st.seconds, "gb_per_s": gbs}


def _buffer_ptr(buf):
    """(address, nbytes) of a writable buffer: bytearray, numpy array, or a
    torch tensor on the host."""
    if hasattr(buf, "data_ptr"):
        return ctypes.c_void_p(buf.data_ptr()), buf.numel() * buf.element_size()
    mv = memoryview(buf)
    if mv.readonly:
        raise ValueError("destination buffer is read-only")
    c = (ctypes.c_char * mv.nbytes).from_buffer(mv)
    return ctypes.cast(c, ctypes.c_void_p), mv.nbytes
