"""A stack whose expert records come from a DEE4 store on disk: written by
the exporter, read back by the native reader straight into HBM (resident
banks, through pinned staging buffers) or into the offload tier's pinned
host block.  The banks are byte-identical to the synthetic ones and the
decode -- route ids and tokens -- is identical."""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def torch_cuda():
    import torch
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    from dee_b200 import build
    build.build()
    return torch


def _decode(torch, st, spec, first, steps):
    B = first.shape[0]
    ids = torch.empty((steps, spec.layers, B, spec.topk), dtype=torch.int32, device="cuda")
    tok = torch.empty((steps, B), dtype=torch.int32, device="cuda")
    st.decode(first, steps, ids, tok)
    torch.cuda.synchronize()
    assert st.engine.sync_status() == 0
    return ids.cpu().numpy(), tok.cpu().numpy()


@pytest.mark.parametrize("fmt", ["dee4-v4-segmented", "dee4-v2"])
def test_stack_from_store_matches_synthetic(torch_cuda, tmp_path, fmt):
    torch = torch_cuda
    from dee_b200.stack import StackSpec, SyntheticStack, seed_tokens
    spec = StackSpec(layers=3, experts=16, hidden=512, inter=512, topk=6, vocab=1024, seed=11)
    B, steps = 4, 3
    first = torch.from_numpy(seed_tokens(spec, B)).cuda()
    src = SyntheticStack(torch, spec, tokens=B)
    path = str(tmp_path / "store")
    src.export_store(path, fmt)
    ids_r, tok_r = _decode(torch, src, spec, first, steps)

    res = SyntheticStack(torch, spec, tokens=B, store=path)
    for layer in range(spec.layers):
        assert torch.equal(res.banks[layer], src.banks[layer]), layer
    assert res.store_fill["records"] == spec.layers * spec.experts
    # one GPU reads every file whole: the seals are checked during the fill
    assert res.store_fill["files_verified"] == (spec.layers if fmt == "dee4-v4-segmented" else 1)
    ids_s, tok_s = _decode(torch, res, spec, first, steps)
    assert np.array_equal(ids_s, ids_r) and np.array_equal(tok_s, tok_r)

    off = SyntheticStack(torch, spec, tokens=B, store=path, offload_slots=20)
    ids_o, tok_o = _decode(torch, off, spec, first, steps)
    assert np.array_equal(ids_o, ids_r) and np.array_equal(tok_o, tok_r)
    assert off.engine.offload_stats()["cold_reads"] > 0


def test_full_shape_store_upload(torch_cuda, tmp_path):
    """DeepSeek-V4 records (13,369,344 B): a 2-layer x 32-expert segmented
    store uploaded whole and as an expert-parallel rank's share, byte for
    byte; the fill rate is printed (page-cache hot: the store was just
    written)."""
    torch = torch_cuda
    from dee_b200.records import RecordLayout, synthetic_bank
    from dee_b200.store import Dee4Store, write_store
    layout = RecordLayout(4096, 2048)
    L, E = 2, 32
    banks = [synthetic_bank(layout, E, seed=30 + l) for l in range(L)]
    host = [b.cpu().numpy() for b in banks]
    path = str(tmp_path / "v4")
    write_store(path, layout, L, E, lambda l: host[l])
    with Dee4Store(path) as st:
        st.check_layout(layout)
        block = torch.empty((L * E, layout.bytes), dtype=torch.uint8, device="cuda")
        fill = st.upload_layers(0, L, block.data_ptr(), block.numel(), torch.cuda.current_stream(), verify=True)
        assert fill["files_verified"] == L
        for l in range(L):
            assert torch.equal(block[l * E:(l + 1) * E], banks[l])
        print(f"store -> HBM: {fill['bytes_read'] / 1e9:.2f} GB in {fill['seconds']:.3f} s "
              f"({fill['gb_per_s']:.1f} GB/s, {fill['pread_calls']} preads)")
        half = torch.empty((L * E // 2, layout.bytes), dtype=torch.uint8, device="cuda")
        st.upload_layers(0, L, half.data_ptr(), half.numel(), None, first_expert=E // 2, experts=E // 2)
        for l in range(L):
            assert torch.equal(half[l * E // 2:(l + 1) * E // 2], banks[l][E // 2:])
