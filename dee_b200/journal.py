"""Route journal in the reference's schema-1 JSONL format.

Restates ``RoutedExpertJournal`` of so-nerdyy/dee
(``dee.cpp/kaggle/deepseek-v4-flash-0731/deepseek_v4_native_generate.py
:452-622``): one record per (forward_step, layer) holding the int32
``[rows, topk]`` route ids the engine consumed, canonical JSON (sorted keys,
``,``/``:`` separators, ASCII), a sha256 chain seeded with sha256(b""),
a flush per layer and an fsync when the last layer of a forward lands.
Records must arrive in ``forward_step, layer`` order.
"""
from __future__ import annotations

import hashlib
import json
import os
from pathlib import Path


class RouteJournal:
    SCHEMA_VERSION = 1
    GENESIS_SHA256 = hashlib.sha256(b"").hexdigest()
    CANONICAL_ORDER = "forward_step,layer,token_row,topk_rank"

    def __init__(self, path, *, run_id: str, n_layers: int, topk: int, fsync: bool = True) -> None:
        if n_layers <= 0 or topk <= 0:
            raise ValueError(f"a journal needs at least one layer and one selection per token (got {n_layers} layers, top-{topk})")
        self.path = Path(path)
        self.run_id = str(run_id)
        self.n_layers = int(n_layers)
        self.topk = int(topk)
        self._fsync = fsync
        self.path.parent.mkdir(parents=True, exist_ok=True)
        self._fh = open(self.path, "w", encoding="utf-8", newline="\n")
        self.chain_sha256 = self.GENESIS_SHA256
        self.record_count = 0
        self.completed_forwards = 0
        self._closed = False

    @staticmethod
    def canonical_bytes(payload: dict) -> bytes:
        return json.dumps(payload, sort_keys=True, separators=(",", ":"), ensure_ascii=True).encode("utf-8")

    def append_layer(self, *, step: int, start_pos: int, layer: int, device: str, expert_ids) -> dict:
        if self._closed:
            raise RuntimeError(f"{self.path} was already closed; open a new journal to record more layers")
        if int(step) != self.completed_forwards or int(layer) != self.record_count % self.n_layers:
            raise RuntimeError(
                f"layers must be recorded forward by forward, layer by layer: next expected is forward "
                f"{self.completed_forwards} layer {self.record_count % self.n_layers}, got forward {step} layer {layer}")
        raw = expert_ids.tolist() if hasattr(expert_ids, "tolist") else expert_ids
        if not isinstance(raw, (list, tuple)) or not raw:
            raise ValueError("expert ids must be given as a non-empty [tokens, topk] matrix")
        rows = []
        for i, r in enumerate(raw):
            row = [int(v) for v in r]
            if len(row) != self.topk:
                raise ValueError(f"token {i} carries {len(row)} expert ids, this journal records top-{self.topk}")
            if any(v < 0 for v in row):
                raise ValueError(f"token {i} carries a negative expert id")
            rows.append(row)
        payload = {
            "schema_version": self.SCHEMA_VERSION,
            "run_id": self.run_id,
            "record_index": self.record_count,
            "forward_step": int(step),
            "phase": "prefill" if int(step) == 0 else "decode",
            "start_pos": int(start_pos),
            "layer": int(layer),
            "device": str(device),
            "token_rows": len(rows),
            "topk": self.topk,
            "expert_ids_rank_order": rows,
            "canonical_order": self.CANONICAL_ORDER,
            "previous_chain_sha256": self.chain_sha256,
        }
        digest = hashlib.sha256(self.canonical_bytes(payload)).hexdigest()
        record = dict(payload, chain_sha256=digest)
        self._fh.write(self.canonical_bytes(record).decode("utf-8") + "\n")
        self._fh.flush()
        self.chain_sha256 = digest
        self.record_count += 1
        if int(layer) == self.n_layers - 1:
            if self._fsync:
                os.fsync(self._fh.fileno())
            self.completed_forwards += 1
        return record

    def close(self) -> None:
        if not self._closed:
            self._fh.flush()
            if self._fsync:
                os.fsync(self._fh.fileno())
            self._fh.close()
            self._closed = True

    def __enter__(self):
        return self

    def __exit__(self, *exc):
        self.close()


def verify_chain(path) -> tuple[int, str]:
    """Re-hash every record; returns (records, final chain sha256)."""
    prev = RouteJournal.GENESIS_SHA256
    n = 0
    with open(path, "r", encoding="utf-8") as fh:
        for line in fh:
            rec = json.loads(line)
            digest = rec.pop("chain_sha256")
            if rec["previous_chain_sha256"] != prev:
                raise ValueError(f"chain break at record {n}")
            if hashlib.sha256(RouteJournal.canonical_bytes(rec)).hexdigest() != digest:
                raise ValueError(f"hash mismatch at record {n}")
            prev = digest
            n += 1
    return n, prev
