"""Host-side arithmetic behind bench.py's roofline object, on CPU: the
algorithmic bytes of one decode layer launch, the record size they count,
and the reader of the committed ncu traffic summary."""
from __future__ import annotations

import os
import sys

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)

import bench  # noqa: E402


def test_record_bytes_are_the_dee4_record():
    from dee_b200.records import RecordLayout
    assert bench.RECORD_BYTES == RecordLayout(bench.H, bench.I).bytes == 13_369_344


def test_decode_kernel_bytes_formula():
    """u records, the b*K grouped token rows read (FP16), the SwiGLU rows
    written and read back (FP16), the FP32 rows written; with the fused
    combine those rows are read back once and b FP32 output rows written."""
    H, I, K = bench.H, bench.I, bench.K
    b, u = 8, 44
    sel = b * K
    base = u * 13_369_344 + sel * H * 2 + 2 * sel * I * 2 + sel * H * 4
    assert bench.decode_kernel_bytes(b, u, False) == base
    assert bench.decode_kernel_bytes(b, u, True) == base + sel * H * 4 + b * H * 4
    # fractional expert counts (a mean over steps) scale the record term only
    assert bench.decode_kernel_bytes(b, 44.5, True) - bench.decode_kernel_bytes(b, 44, True) == 13_369_344 / 2


def test_committed_traffic_summary():
    """The ncu summary's algorithmic figure is this formula at the captured
    launch's 45 active experts, and its DRAM bytes are within 1% of it."""
    tr = bench.profiled_traffic("traffic_decode_b8.md", "decode_layer")
    assert tr is not None
    assert tr["traffic"] == 602_853_888
    assert tr["traffic"] / tr["traffic_ratio"] == bench.decode_kernel_bytes(8, 45, True) == 604_110_848
    assert 0.99 < tr["traffic_ratio"] < 1.01
    assert bench.profiled_traffic("traffic_decode_b8.md", "no_such_kernel") is None
    assert bench.profiled_traffic("no_such_summary.md", "decode_layer") is None
