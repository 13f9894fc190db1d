"""CPU tests of the host side: the C-ABI library, the pydee-mirror binding
and the route journal.  No CUDA compute runs here."""
import json
import os
import re

import numpy as np
import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
GOLDEN = os.path.join(ROOT, "tests", "golden")


@pytest.fixture(scope="module")
def lib():
    from dee_b200 import _native, build
    build.build()
    return _native.load()


def _header_functions():
    text = open(os.path.join(ROOT, "include", "dee_b200.h")).read()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"\b(dee_[a-z0-9_]+)\s*\(", text)))


def test_library_exports_every_declared_symbol(lib):
    from dee_b200 import _native
    names = _header_functions()
    assert len(names) >= 15
    for n in names:
        assert hasattr(lib, n), n
    assert set(names) == set(_native.SIGNATURES), "binding and header disagree"


def test_abi_guard(lib):
    import ctypes
    from dee_b200 import _native
    assert lib.dee_abi_config_size() == ctypes.sizeof(_native.DeeConfig)
    assert lib.dee_abi_version() == 1


def test_unsupported_shapes_fail_closed(lib):
    import ctypes
    from dee_b200 import _native
    h = ctypes.c_void_p()
    for cfg in (_native.DeeConfig(4096, 2000, 256, 6, 1, 0, 0.0, 8),    # I % 512
                _native.DeeConfig(4096, 2048, 512, 6, 1, 0, 0.0, 8),    # E > 256
                _native.DeeConfig(4096, 2048, 256, 0, 1, 0, 0.0, 8)):   # topk
        assert lib.dee_engine_create(ctypes.byref(cfg), ctypes.byref(h)) == _native.DEE_ERR_UNSUPPORTED
        assert not h


def test_kernel_entry_points_validate_arguments(lib):
    from dee_b200 import _native
    assert lib.dee_fp4_decode_device(None, None, None, 4, 64, None) == _native.DEE_ERR_INVALID
    assert lib.dee_fp4_decode_device(1, 1, 1, 4, 60, None) == _native.DEE_ERR_INVALID
    assert lib.dee_fp4_quantize_device(1, 4, 30, 1, 1, None) == _native.DEE_ERR_INVALID


def test_record_layout_matches_reference_sizes():
    from dee_b200.records import RecordLayout
    L = RecordLayout(4096, 2048)
    assert L.bytes == 13_369_344
    o = L.offsets
    assert (o["w3"], o["w2"], o["s1"], o["s3"], o["s2"]) == (4_194_304, 8_388_608, 12_582_912,
                                                             12_845_056, 13_107_200)


def test_journal_matches_reference_bytes(tmp_path):
    from dee_b200.journal import RouteJournal, verify_chain
    ids = np.load(os.path.join(GOLDEN, "journal_ids.npz"))
    path = tmp_path / "routed_experts.jsonl"
    with RouteJournal(path, run_id="golden-run", n_layers=3, topk=6) as j:
        i = 0
        for step in (0, 1):
            for layer in range(3):
                j.append_layer(step=step, start_pos=0 if step == 0 else 4, layer=layer, device="cuda:0",
                               expert_ids=ids[f"arr_{i}"])
                i += 1
    want = open(os.path.join(GOLDEN, "journal.jsonl"), "rb").read()
    assert path.read_bytes() == want
    n, chain = verify_chain(path)
    assert n == 6 and chain == json.loads(want.decode().splitlines()[-1])["chain_sha256"]


def test_journal_rejects_out_of_order(tmp_path):
    from dee_b200.journal import RouteJournal
    j = RouteJournal(tmp_path / "j.jsonl", run_id="r", n_layers=2, topk=2, fsync=False)
    j.append_layer(step=0, start_pos=0, layer=0, device="cpu", expert_ids=[[1, 2]])
    with pytest.raises(RuntimeError):
        j.append_layer(step=0, start_pos=0, layer=0, device="cpu", expert_ids=[[1, 2]])
    with pytest.raises(ValueError):
        j.append_layer(step=0, start_pos=0, layer=1, device="cpu", expert_ids=[[1, -2]])
    j.close()
