"""Expert-parallel choreography on two CPU ranks (gloo).

dee_b200.ep.ExpertParallelMoE runs its collectives for real; the three
device steps are replaced by numpy implementations of the same contracts on
top of the oracle (the CUDA kernels implementing them are tested against the
same contracts in test_gpu_ep.py).  Every rank's output must equal, bit for
bit, the single-process oracle layer over all experts.
"""
import os
import socket

import numpy as np
import pytest

H, I, E, K, T, WORLD = 512, 512, 16, 6, 5, 2
EPR = E // WORLD


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


def _inputs(orc, rank):
    layout = orc.Layout(H, I)
    recs = orc.synthetic_records(layout, E, seed=2024, kind="normal")
    rng = np.random.default_rng(100 + rank)
    x16 = orc.f16_bits(rng.standard_normal((T, H)))
    ids = np.stack([rng.choice(E, K, replace=False) for _ in range(T)]).astype(np.int32)
    w = rng.random((T, K)).astype(np.float32)
    w /= w.sum(axis=1, keepdims=True)
    return layout, recs, x16, ids, w


def _np_ops(orc, layout, recs_local, capacity):
    from dee_b200.ep import EpOps

    def pack(ids, x, send_rows, send_expert, slot_of_pos):
        ids_n, x_n = ids.numpy().reshape(-1), x.numpy()
        rows, sexp, sop = send_rows.numpy(), send_expert.numpy(), slot_of_pos.numpy()
        sexp[:] = -1
        fill = np.zeros(WORLD, dtype=np.int64)
        for p, e in enumerate(ids_n):  # ascending t*K + r within each destination
            d = int(e) // EPR
            s = int(fill[d])
            assert s < capacity
            fill[d] += 1
            rows[d * capacity + s] = x_n[p // K]
            sexp[d * capacity + s] = int(e) - d * EPR
            sop[p] = d * capacity + s

    def compute(recv_rows, recv_expert, raw, layer):
        ex, rw = recv_expert.numpy(), raw.numpy()
        live = np.flatnonzero(ex >= 0)
        if live.size:
            xr = recv_rows.numpy()[live].view(np.uint16)
            out = orc.moe_layer_raw(recs_local, layout, xr, ex[live].reshape(-1, 1).astype(np.int32))
            rw[live] = out[:, 0, :]

    def combine(back, slot_of_pos, weights, out):
        b, sop, w, o = back.numpy(), slot_of_pos.numpy(), weights.numpy(), out.numpy()
        for t in range(out.shape[0]):
            acc = np.zeros(H, dtype=np.float32)
            for r in range(K):
                acc = (acc + (np.float32(w[t, r]) * b[sop[t * K + r]]).astype(np.float32)).astype(np.float32)
            o[t] = acc

    return EpOps(pack, compute, combine)


def _rank_main(rank, port, q, exchange="fixed"):
    import sys
    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    sys.path.insert(0, root)
    import torch
    import torch.distributed as dist
    from oracle import oracle as orc
    from dee_b200.ep import ExpertParallelMoE
    try:
        dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank,
                                world_size=WORLD)
        layout, recs, x16, ids, w = _inputs(orc, rank)
        recs_local = recs[rank * EPR:(rank + 1) * EPR]
        ep = ExpertParallelMoE(torch, rank, WORLD, EPR, T, K, H, "cpu",
                               ops=_np_ops(orc, layout, recs_local, T * K), exchange=exchange)
        assert ep.counts_mode == (exchange == "counts")
        out = ep.forward(torch.from_numpy(x16.view(np.float16)), torch.from_numpy(ids),
                         torch.from_numpy(w)).numpy().copy()
        want = orc.combine_f32(orc.moe_layer_raw(recs, layout, x16, ids), w)
        q.put((rank, bool(np.array_equal(out, want)), float(np.abs(out - want).max())))
        dist.barrier()
        dist.destroy_process_group()
    except Exception as exc:  # report instead of hanging the parent
        q.put((rank, False, repr(exc)))


@pytest.mark.parametrize("exchange", ["fixed", "counts"])
def test_expert_parallel_two_ranks_match_single_process(exchange):
    """Both exchanges: equal blocks of capacity rows per rank pair, and the
    counts all-to-all followed by all-to-alls of the occupied rows only."""
    import torch.multiprocessing as mp
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_rank_main, args=(r, port, q, exchange)) for r in range(WORLD)]
    for p in procs:
        p.start()
    results = [q.get(timeout=240) for _ in range(WORLD)]
    for p in procs:
        p.join(timeout=60)
    for rank, ok, detail in sorted(results, key=lambda r: r[0]):
        assert ok, f"rank {rank}: {detail}"
