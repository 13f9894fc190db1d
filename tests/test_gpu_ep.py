"""Expert-parallel kernels on one GPU: two ranks emulated by two engines.

The all-to-alls become block copies between the ranks' buffers (a
multi-rank launch would need one GPU per rank); pack, the rows forward and
the combine are the product kernels.  Each rank's output must be bit-identical
to one engine holding all experts (the per-row results of the grouped GEMMs do
not depend on which rows share a tile), and close to the oracle.
"""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu

H, I, E, K, WORLD = 512, 512, 16, 6, 2
EPR = E // WORLD
TOL_REL_L2 = 2e-3


@pytest.fixture(scope="module")
def torch_cuda():
    import torch
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    from dee_b200 import build
    build.build()
    return torch


def _engine(E_, topk=K):
    import dee_b200
    return dee_b200.new_engine(dee_b200.EngineConfig(hidden=H, inter=I, num_experts=E_, topk=topk,
                                                     max_tokens=64))


@pytest.mark.parametrize("T", [1, 5, 8])
def test_expert_parallel_emulated_two_ranks(torch_cuda, oracle_mod, T):
    torch = torch_cuda
    orc = oracle_mod
    layout = orc.Layout(H, I)
    recs = orc.synthetic_records(layout, E, seed=77 + T, kind="normal")
    bank_all = torch.from_numpy(recs).cuda()
    full = _engine(E)
    full.attach_bank(0, bank_all)
    ranks = []
    for r in range(WORLD):
        eng = _engine(EPR)
        bank = torch.from_numpy(np.ascontiguousarray(recs[r * EPR:(r + 1) * EPR])).cuda()
        eng.attach_bank(0, bank)
        rng = np.random.default_rng(900 + 10 * T + r)
        x16 = orc.f16_bits(rng.standard_normal((T, H)))
        ids = np.stack([rng.choice(E, K, replace=False) for _ in range(T)]).astype(np.int32)
        if r == 1 and T > 1:
            ids[0] = np.arange(K) + EPR  # every selection of a token on the other rank
        w = rng.random((T, K)).astype(np.float32)
        w /= w.sum(axis=1, keepdims=True)
        ranks.append(dict(eng=eng, bank=bank, x16=x16, ids=ids, w=w,
                          dx=torch.from_numpy(x16.view(np.float16)).cuda(),
                          dids=torch.from_numpy(ids).cuda(), dw=torch.from_numpy(w).cuda()))
    C = T * K
    n = WORLD * C
    for rk in ranks:
        rk["send_rows"] = torch.empty((n, H), dtype=torch.float16, device="cuda")
        rk["send_exp"] = torch.empty((n,), dtype=torch.int32, device="cuda")
        rk["sop"] = torch.empty((T * K,), dtype=torch.int32, device="cuda")
        rk["eng"].ep_pack_device(rk["dids"].data_ptr(), T, rk["dx"].data_ptr(), WORLD, EPR, C,
                                 rk["send_rows"].data_ptr(), rk["send_exp"].data_ptr(),
                                 rk["sop"].data_ptr())
    # all-to-all: rank r receives block r of every source, in source order
    for r, rk in enumerate(ranks):
        rk["recv_rows"] = torch.cat([src["send_rows"][r * C:(r + 1) * C] for src in ranks]).contiguous()
        rk["recv_exp"] = torch.cat([src["send_exp"][r * C:(r + 1) * C] for src in ranks]).contiguous()
        rk["raw"] = torch.zeros((n, H), dtype=torch.float32, device="cuda")
        rk["eng"].moe_forward_rows_device(0, rk["recv_rows"].data_ptr(), rk["recv_exp"].data_ptr(), n,
                                          rk["raw"].data_ptr())
    for s, rk in enumerate(ranks):
        back = torch.cat([dst["raw"][s * C:(s + 1) * C] for dst in ranks]).contiguous()
        out = torch.empty((T, H), dtype=torch.float32, device="cuda")
        rk["eng"].ep_combine_device(back.data_ptr(), rk["sop"].data_ptr(), rk["dw"].data_ptr(), T,
                                    out.data_ptr())
        ref = torch.empty((T, H), dtype=torch.float32, device="cuda")
        full.moe_forward_device(0, rk["dx"].data_ptr(), T, d_ids_ptr=rk["dids"].data_ptr(),
                                d_weights_ptr=rk["dw"].data_ptr(), d_out_ptr=ref.data_ptr())
        torch.cuda.synchronize()
        for eng in (rk["eng"], full):
            assert eng.sync_status() == 0
        got, want = out.cpu().numpy(), ref.cpu().numpy()
        assert np.array_equal(got, want), float(np.abs(got - want).max())
        oracle = orc.combine_f32(orc.moe_layer_raw(recs, layout, rk["x16"], rk["ids"]), rk["w"])
        assert orc.rel_l2(got, oracle) <= TOL_REL_L2
        # the journal of a rank holds its own tokens' global ids
        assert np.array_equal(rk["eng"].journal_ids(T), rk["ids"])
    # each destination block of a sender holds its selections in position order
    sop = ranks[0]["sop"].cpu().numpy()
    exp_ = ranks[0]["send_exp"].cpu().numpy()
    ids0 = ranks[0]["ids"].reshape(-1)
    for d in range(WORLD):
        mine = [p for p in range(T * K) if ids0[p] // EPR == d]
        assert [int(sop[p]) for p in mine] == [d * C + i for i in range(len(mine))]
        assert all(exp_[d * C + i] == ids0[p] - d * EPR for i, p in enumerate(mine))
        assert (exp_[d * C + len(mine):(d + 1) * C] == -1).all()


def test_ep_pack_rejects_bad_arguments(torch_cuda):
    import dee_b200
    torch = torch_cuda
    eng = _engine(EPR)
    d = torch.zeros((8,), dtype=torch.int32, device="cuda")
    x = torch.zeros((1, H), dtype=torch.float16, device="cuda")
    with pytest.raises(dee_b200.DeeError):
        # experts_per_rank must equal the engine's num_experts
        eng.ep_pack_device(d.data_ptr(), 1, x.data_ptr(), WORLD, EPR + 1, K, d.data_ptr(),
                           d.data_ptr(), d.data_ptr())
    with pytest.raises(dee_b200.DeeError):
        eng.ep_pack_device(d.data_ptr(), 1, x.data_ptr(), 0, EPR, K, d.data_ptr(), d.data_ptr(),
                           d.data_ptr())


@pytest.mark.parametrize("T", [1, 8])
def test_expert_parallel_peer_emulated_two_ranks(torch_cuda, oracle_mod, T):
    """The NVLink path with both ranks in this process on one GPU: the blocks
    are mapped by address, and the phases of the two ranks are interleaved so
    that each bounded wait finds its flags already raised by earlier kernels
    on the stream."""
    torch = torch_cuda
    orc = oracle_mod
    layout = orc.Layout(H, I)
    recs = orc.synthetic_records(layout, E, seed=313 + T, kind="normal")
    full = _engine(E)
    bank_all = torch.from_numpy(recs).cuda()
    full.attach_bank(0, bank_all)
    ranks = []
    for r in range(WORLD):
        eng = _engine(EPR)
        bank = torch.from_numpy(np.ascontiguousarray(recs[r * EPR:(r + 1) * EPR])).cuda()
        eng.attach_bank(0, bank)
        rng = np.random.default_rng(1700 + 10 * T + r)
        x16 = orc.f16_bits(rng.standard_normal((T, H)))
        ids = np.stack([rng.choice(E, K, replace=False) for _ in range(T)]).astype(np.int32)
        w = rng.random((T, K)).astype(np.float32)
        w /= w.sum(axis=1, keepdims=True)
        _, block = eng.ep_p2p_init(WORLD, r, T)
        ranks.append(dict(eng=eng, bank=bank, x16=x16, ids=ids, w=w, block=block,
                          dx=torch.from_numpy(x16.view(np.float16)).cuda(),
                          dids=torch.from_numpy(ids).cuda(), dw=torch.from_numpy(w).cuda(),
                          out=torch.empty((T, H), dtype=torch.float32, device="cuda")))
    blocks = [rk["block"] for rk in ranks]
    for rk in ranks:
        rk["eng"].ep_p2p_connect(None, blocks)
    for step in range(2):  # two layer calls: the epoch advances
        for rk in ranks:
            rk["eng"].ep_p2p_dispatch_device(rk["dx"].data_ptr(), rk["dids"].data_ptr())
        for rk in ranks:
            rk["eng"].ep_p2p_experts_device(0)
        for rk in ranks:
            rk["eng"].ep_p2p_combine_device(rk["dw"].data_ptr(), rk["out"].data_ptr())
        torch.cuda.synchronize()
        for rk in ranks:
            assert rk["eng"].sync_status() == 0
            ref = torch.empty((T, H), dtype=torch.float32, device="cuda")
            full.moe_forward_device(0, rk["dx"].data_ptr(), T, d_ids_ptr=rk["dids"].data_ptr(),
                                    d_weights_ptr=rk["dw"].data_ptr(), d_out_ptr=ref.data_ptr())
            torch.cuda.synchronize()
            got, want = rk["out"].cpu().numpy(), ref.cpu().numpy()
            assert np.array_equal(got, want), float(np.abs(got - want).max())
            assert np.array_equal(rk["eng"].journal_ids(T), rk["ids"])


def test_rows_forward_large_receive_buffer(torch_cuda, oracle_mod):
    """A receive buffer of 2500 rows (the multi-CTA grouping) with a third of
    the rows unused (expert -1): the unused rows are left as they were, the
    others match the oracle's FP16 expert chain."""
    torch = torch_cuda
    orc = oracle_mod
    layout = orc.Layout(H, I)
    recs = orc.synthetic_records(layout, EPR, seed=4242, kind="normal")
    eng = _engine(EPR)
    bank = torch.from_numpy(recs).cuda()
    eng.attach_bank(0, bank)
    rng = np.random.default_rng(2500)
    n = 2500
    x16 = orc.f16_bits(rng.standard_normal((n, H)))
    exp_ = rng.integers(0, EPR, n).astype(np.int32)
    exp_[rng.random(n) < 0.35] = -1
    rows = torch.from_numpy(x16.view(np.float16)).cuda()
    dexp = torch.from_numpy(exp_).cuda()
    raw = torch.full((n, H), 7.0, dtype=torch.float32, device="cuda")
    eng.moe_forward_rows_device(0, rows.data_ptr(), dexp.data_ptr(), n, raw.data_ptr())
    torch.cuda.synchronize()
    assert eng.sync_status() == 0
    got = raw.cpu().numpy()
    unused = exp_ < 0
    assert (got[unused] == 7.0).all()
    want = orc.moe_layer_raw(recs, layout, x16[~unused], exp_[~unused].reshape(-1, 1))[:, 0]
    assert orc.rel_l2(got[~unused], want) <= TOL_REL_L2
