"""CPU tests of the DEE4 store reader (native) and writer.

The cases follow the reference's own store tests
(dee.cpp/tests/test_dee4_segmented.cpp: SHA-256 known answers, a small
dense segmented store with real seals resolved across segment boundaries
and read back byte for byte, every fail-closed case, and the true-geometry
46 x 256 x 13,369,344-byte universe over sparse files with the seal pass
off; dee.cpp/tests/test_expert_store.cpp for the single-file formats).
No CUDA runs here: the reads go to host memory.
"""
import hashlib
import json
import os

import numpy as np
import pytest

from dee_b200.records import RecordLayout

SMALL = RecordLayout(64, 32)   # 3,264-byte records
LAYERS, EXPERTS = 4, 4


def layer_records(layer, experts=EXPERTS, layout=SMALL):
    rng = np.random.default_rng(1000 + layer)
    return rng.integers(0, 256, size=(experts, layout.bytes), dtype=np.uint8)


def write(tmp_path, fmt="dee4-v4-segmented", **kw):
    from dee_b200.store import write_store
    d = str(tmp_path / fmt)
    meta = write_store(d, SMALL, LAYERS, EXPERTS, layer_records, fmt=fmt, **kw)
    return d, meta


def open_store(path, **kw):
    from dee_b200.store import Dee4Store
    return Dee4Store(path, **kw)


def edit_meta(d, fn):
    p = os.path.join(d, "metadata.json")
    meta = json.load(open(p))
    fn(meta)
    json.dump(meta, open(p, "w"))


def expect_fail(d, needle, **kw):
    from dee_b200.store import StoreError
    with pytest.raises(StoreError) as exc:
        open_store(d, **kw)
    assert needle in str(exc.value), str(exc.value)


# -- SHA-256 -----------------------------------------------------------------

def test_sha256_known_answers():
    from dee_b200.store import sha256_hex
    assert sha256_hex(b"") == "e3b0c44298fc1c149afbf4c8996fb92427ae41e4649b934ca495991b7852b855"
    assert sha256_hex(b"abc") == "ba7816bf8f01cfea414140de5dae2223b00361a396177a9cb410ff61f20015ad"
    assert sha256_hex(b"a" * 1_000_000) == "cdc76e5c9914fb9281a1c7e284d73e67f1809a48a497200e046d39ccc7112cd0"
    rng = np.random.default_rng(7)
    for n in (1, 55, 56, 63, 64, 65, 119, 120, 4095, 100_003):
        data = rng.integers(0, 256, n, dtype=np.uint8).tobytes()
        assert sha256_hex(data) == hashlib.sha256(data).hexdigest(), n


def test_sha256_portable_path_matches():
    """The portable compression (forced) agrees with the SHA-extension one."""
    import subprocess
    import sys
    code = ("import hashlib, numpy as np\n"
            "from dee_b200.store import sha256_hex\n"
            "rng = np.random.default_rng(3)\n"
            "for n in (0, 3, 64, 65, 1000, 65536 + 17):\n"
            "    d = rng.integers(0, 256, n, dtype=np.uint8).tobytes()\n"
            "    assert sha256_hex(d) == hashlib.sha256(d).hexdigest(), n\n"
            "print('ok')\n")
    env = dict(os.environ, DEE_SHA256_PORTABLE="1")
    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    out = subprocess.run([sys.executable, "-c", code], env=env, cwd=root, capture_output=True, text=True)
    assert out.returncode == 0 and "ok" in out.stdout, out.stderr


# -- the three formats --------------------------------------------------------

@pytest.mark.parametrize("fmt", ["dee4-v4-segmented", "dee4-v2"])
def test_dense_store_round_trip(tmp_path, fmt):
    d, meta = write(tmp_path, fmt)
    with open_store(d) as s:
        assert (s.start_layer, s.num_layers, s.experts_per_layer) == (0, LAYERS, EXPERTS)
        assert s.record_bytes == SMALL.bytes and s.stored_records == LAYERS * EXPERTS
        s.check_layout(SMALL)
        if fmt == "dee4-v4-segmented":
            assert s.backend == "dee4_segmented" and s.segmented and s.file_count == LAYERS
            seals = "".join(seg["sha256"] for seg in meta["segments"])
            assert s.identity == hashlib.sha256(seals.encode()).hexdigest()
        else:
            assert s.backend == "dee4" and not s.segmented and s.file_count == 1
            assert s.identity == meta["data_sha256"]
        # every pair, including the ones either side of a segment boundary
        for layer in range(LAYERS):
            want = layer_records(layer)
            for e in range(EXPERTS):
                assert s.lookup(layer, e) == layer * EXPERTS + e
                got = np.frombuffer(s.materialize(layer, e), dtype=np.uint8)
                assert np.array_equal(got, want[e]), (layer, e)
        # whole layers in parallel pieces
        buf = np.zeros((3, EXPERTS, SMALL.bytes), dtype=np.uint8)
        st = s.read_layers(1, 3, buf.ctypes.data, buf.nbytes)
        assert st["bytes_read"] == buf.nbytes and st["records"] == 3 * EXPERTS
        for k in range(3):
            assert np.array_equal(buf[k], layer_records(1 + k))
        # an expert-parallel rank's share: experts [1, 3) of layers 0..3
        part = np.zeros((LAYERS, 2, SMALL.bytes), dtype=np.uint8)
        s.read_layers(0, LAYERS, part.ctypes.data, part.nbytes, first_expert=1, experts=2)
        for k in range(LAYERS):
            assert np.array_equal(part[k], layer_records(k)[1:3])
        stats = s.stats()
        assert stats["lookup_failures"] == 0 and stats["bytes_read"] >= buf.nbytes


def test_out_of_range_pairs_fail_closed(tmp_path):
    from dee_b200.store import StoreError
    d, _ = write(tmp_path)
    with open_store(d) as s:
        for layer, e in ((LAYERS, 0), (-1, 0), (0, EXPERTS), (0, -1)):
            with pytest.raises(StoreError):
                s.lookup(layer, e)
            with pytest.raises(StoreError):
                s.materialize(layer, e)
        with pytest.raises(StoreError):
            s.materialize(0, 0, bytearray(SMALL.bytes - 1))
        buf = np.zeros((2, EXPERTS, SMALL.bytes), dtype=np.uint8)
        with pytest.raises(StoreError):
            s.read_layers(LAYERS - 1, 2, buf.ctypes.data, buf.nbytes)
        with pytest.raises(StoreError):
            s.read_layers(0, 2, buf.ctypes.data, buf.nbytes - 1)
        assert s.stats()["lookup_failures"] >= 8


def test_trace_store(tmp_path):
    from dee_b200.store import StoreError
    pairs = [(0, 1), (0, 3), (2, 0), (3, 2), (3, 3)]
    d, meta = write(tmp_path, "dee4-v3-trace", trace_pairs=pairs)
    with open_store(d) as s:
        assert s.backend == "dee4_trace" and s.trace_indexed and s.stored_records == len(pairs)
        assert s.identity == meta["data_sha256"]
        for idx, (layer, e) in enumerate(pairs):
            assert s.lookup(layer, e) == idx
            assert np.array_equal(np.frombuffer(s.materialize(layer, e), np.uint8), layer_records(layer)[e])
        for layer, e in ((0, 0), (1, 1), (2, 1)):
            with pytest.raises(StoreError):
                s.lookup(layer, e)
        buf = np.zeros((1, EXPERTS, SMALL.bytes), dtype=np.uint8)
        with pytest.raises(StoreError, match="not in the store"):
            s.read_layers(0, 1, buf.ctypes.data, buf.nbytes)


def test_trace_index_must_be_sorted_and_unique(tmp_path):
    d, _ = write(tmp_path, "dee4-v3-trace", trace_pairs=[(0, 1), (1, 2), (2, 0)])
    edit_meta(d, lambda m: m["records"].__setitem__(1, {"layer": 0, "expert": 1, "record_index": 1}))
    expect_fail(d, "not strictly sorted/unique")
    edit_meta(d, lambda m: m["records"].__setitem__(1, {"layer": 0, "expert": 1, "record_index": 5}))
    expect_fail(d, "trace record index is invalid")
    edit_meta(d, lambda m: m.__setitem__("selection_sha256", "xyz"))
    expect_fail(d, "trace index metadata is invalid")


# -- fail-closed open --------------------------------------------------------

def test_missing_metadata_and_bad_json(tmp_path):
    expect_fail(str(tmp_path / "nothing"), "metadata.json is missing")
    d = tmp_path / "bad"
    d.mkdir()
    (d / "metadata.json").write_text("{\"format\": \"dee4-v2\",")
    expect_fail(str(d), "JSON parse failed")
    (d / "metadata.json").write_text("[1, 2]")
    expect_fail(str(d), "JSON parse failed")


@pytest.mark.parametrize("edit,needle", [
    (lambda m: m.__setitem__("format", "dee4-v9"), "schema/codec/layout is invalid"),
    (lambda m: m.__setitem__("codec", "fp8"), "schema/codec/layout is invalid"),
    (lambda m: m.__setitem__("record_bytes", 3264.0), "schema/codec/layout is invalid"),
    (lambda m: m.__setitem__("num_layers", -4), "schema/codec/layout is invalid"),
    (lambda m: m.__setitem__("weight_offsets", [0, 1024]), "schema/codec/layout is invalid"),
    (lambda m: m.__setitem__("experts_per_layer", 0), "geometry is empty or out of range"),
    (lambda m: m["scale_offsets"].__setitem__(2, 3201), "component range escapes its record"),
    (lambda m: m["weight_out"].__setitem__(0, 31), "component shape/byte length mismatch"),
    (lambda m: m.__setitem__("data_file", "experts.dee4"), "must not name a data_file"),
    (lambda m: m.__setitem__("total_experts", 15), "segmented store metadata is invalid"),
    (lambda m: m["segments"].pop(), "segmented store metadata is invalid"),
    (lambda m: m.__setitem__("universe_sha256", "00"), "universe binding is invalid"),
    (lambda m: m["segments"][1].__setitem__("bucket", 2), "segment table is invalid"),
    (lambda m: m["segments"][2].__setitem__("first_record", 9), "segment table is invalid"),
    (lambda m: m["segments"][0].__setitem__("record_count", 3), "segment table is invalid"),
    (lambda m: m["segments"][0].__setitem__("sha256", "g" * 64), "segment table is invalid"),
    (lambda m: m["segments"][0].__setitem__("domain", 3), "segment table is invalid"),
    (lambda m: m["segments"][3].__setitem__("bytes", 1), "segment byte count is inconsistent"),
    (lambda m: m["segments"][0].__setitem__("file", "../x.dee4"), "segment path escapes the store"),
    (lambda m: m["segments"][0].__setitem__("file", "/etc/passwd"), "segment path escapes the store"),
])
def test_segmented_metadata_fails_closed(tmp_path, edit, needle):
    d, _ = write(tmp_path)
    edit_meta(d, edit)
    expect_fail(d, needle)


def test_segment_files_fail_closed(tmp_path):
    d, meta = write(tmp_path)
    seg = os.path.join(d, meta["segments"][2]["file"])
    data = open(seg, "rb").read()
    # mis-hashed: one flipped byte fails the seal, opens with verification off
    flipped = bytearray(data)
    flipped[1234] ^= 0x40
    open(seg, "wb").write(flipped)
    expect_fail(d, "experts-bucket-02.dee4 sha256 mismatch")
    with open_store(d, verify_segment_hashes=False) as s:
        assert s.materialize(2, 0)[1234] == flipped[1234]
    # mis-sized: structural, fails with or without verification
    open(seg, "wb").write(data[:-1])
    expect_fail(d, "does not match expected", verify_segment_hashes=False)
    # missing
    os.remove(seg)
    expect_fail(d, "cannot be opened", verify_segment_hashes=False)
    # upper-case seals are accepted (normalised to lower case)
    open(seg, "wb").write(data)
    edit_meta(d, lambda m: m["segments"][2].__setitem__("sha256", m["segments"][2]["sha256"].upper()))
    with open_store(d) as s:
        assert s.stored_records == LAYERS * EXPERTS


@pytest.mark.parametrize("fmt", ["dee4-v4-segmented", "dee4-v2"])
def test_fill_checks_seals_in_one_pass(tmp_path, fmt):
    """A store opened without the seal pass and filled whole with verify:
    every file is hashed as it streams in; a flipped byte fails the fill;
    a partial read (an expert-parallel share) verifies nothing."""
    from dee_b200.store import StoreError
    d, meta = write(tmp_path, fmt)
    files = LAYERS if fmt == "dee4-v4-segmented" else 1
    buf = np.zeros((LAYERS, EXPERTS, SMALL.bytes), dtype=np.uint8)
    with open_store(d, verify_segment_hashes=False) as s:
        st = s.read_layers(0, LAYERS, buf.ctypes.data, buf.nbytes, verify=True)
        assert st["files_verified"] == files and st["records"] == LAYERS * EXPERTS
        part = np.zeros((LAYERS, 2, SMALL.bytes), dtype=np.uint8)
        st = s.read_layers(0, LAYERS, part.ctypes.data, part.nbytes, first_expert=2, experts=2, verify=True)
        assert st["files_verified"] == 0
    path = os.path.join(d, meta["segments"][3]["file"] if files > 1 else "experts.dee4")
    data = bytearray(open(path, "rb").read())
    data[-5] ^= 1
    open(path, "wb").write(data)
    with open_store(d, verify_segment_hashes=False) as s:
        s.read_layers(0, LAYERS, buf.ctypes.data, buf.nbytes)           # unverified fill serves it
        with pytest.raises(StoreError, match="sha256 mismatch"):
            s.read_layers(0, LAYERS, buf.ctypes.data, buf.nbytes, verify=True)
    if files > 1:
        with open_store(d, verify_segment_hashes=False) as s:        # the sealed files before it pass
            st = s.read_layers(0, 3, buf.ctypes.data, buf.nbytes, verify=True)
            assert st["files_verified"] == 3


def test_seal_pass_can_drop_pages(tmp_path):
    d, _ = write(tmp_path)
    with open_store(d, seal_reads_through_page_cache=True) as s:
        assert s.num_layers == LAYERS


def test_single_file_fails_closed(tmp_path):
    d, meta = write(tmp_path, "dee4-v2")
    path = os.path.join(d, "experts.dee4")
    data = open(path, "rb").read()
    open(path, "wb").write(data + b"\0")
    expect_fail(d, "does not match expected")
    open(path, "wb").write(data)
    edit_meta(d, lambda m: m.__setitem__("data_sha256", "abc"))
    expect_fail(d, "schema/codec/layout is invalid")
    edit_meta(d, lambda m: (m.__setitem__("data_sha256", meta["data_sha256"]), m.pop("data_file")))
    expect_fail(d, "schema/codec/layout is invalid")


def test_json_literals_escapes_and_null(tmp_path):
    """The writer's literal null, escaped strings and unknown keys parse."""
    d, _ = write(tmp_path)
    p = os.path.join(d, "metadata.json")
    text = open(p).read()
    text = text.replace('"source_repository": "synthetic"',
                        '"source_repository": "syn\\u0074h\\"etic\\\\ \\ud83d\\ude00", "extra": [true, false, null, -1.5e3]')
    open(p, "w").write(text)
    with open_store(d) as s:
        assert s.num_layers == LAYERS


def test_engine_layout_check(tmp_path):
    from dee_b200.store import StoreError
    d, _ = write(tmp_path)
    with open_store(d) as s:
        with pytest.raises(StoreError):
            s.check_layout(RecordLayout(32, 64))


def _sparse_ok(path):
    with open(path, "wb") as fh:
        fh.truncate(1 << 30)
    ok = os.stat(path).st_blocks * 512 < (1 << 20)
    os.remove(path)
    return ok


def test_true_geometry_universe_sparse(tmp_path):
    """46 buckets x 256 experts x 13,369,344 B (146.6 GiB logical) over sparse
    segment files carrying a marker per probed record; seals off (the table
    must still be structurally exact)."""
    if not _sparse_ok(str(tmp_path / "probe")):
        pytest.skip("filesystem without sparse files")
    from dee_b200.store import _layout_fields, CODEC
    layout = RecordLayout(4096, 2048)
    rb, buckets, experts = layout.bytes, 46, 256
    assert rb == 13_369_344
    d = tmp_path / "universe"
    (d / "segments").mkdir(parents=True)
    probes = [(0, 0), (0, 255), (1, 0), (21, 137), (42, 255), (43, 0), (45, 255)]

    def marker(b, e):
        return hashlib.sha256(f"{b}:{e}".encode()).digest()

    segments = []
    for b in range(buckets):
        name = f"experts-bucket-{b:02d}.dee4"
        with open(d / "segments" / name, "wb") as fh:
            fh.truncate(experts * rb)
            for pb, pe in probes:
                if pb == b:
                    fh.seek(pe * rb + rb - 32)
                    fh.write(marker(pb, pe))
        segments.append({"file": f"segments/{name}", "bucket": b, "domain": "main" if b < 43 else "mtp",
                         "first_record": b * experts, "record_count": experts, "bytes": experts * rb,
                         "sha256": hashlib.sha256(name.encode()).hexdigest()})
    meta = {"format": "dee4-v4-segmented", "codec": CODEC, "start_layer": 0, "num_layers": buckets,
            "experts_per_layer": experts, "total_experts": buckets * experts, **_layout_fields(layout),
            "segments": segments, "data_file": None, "mtp_bucket_offset": 43}
    (d / "metadata.json").write_text(json.dumps(meta))
    with open_store(str(d), verify_segment_hashes=False) as s:
        assert s.stored_records == buckets * experts and s.file_count == buckets
        s.check_layout(layout)
        rec = bytearray(rb)
        for b, e in probes:
            assert s.lookup(b, e) == b * experts + e
            s.materialize(b, e, rec)
            assert bytes(rec[-32:]) == marker(b, e) and not any(rec[:64])
        from dee_b200.store import StoreError
        for b, e in ((46, 0), (-1, 0), (0, 256), (0, -1)):
            with pytest.raises(StoreError):
                s.lookup(b, e)
