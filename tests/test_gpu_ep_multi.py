"""Expert parallelism on two real GPUs (skipped with fewer): each rank's
output through the NVLink peer path and through the NCCL all-to-all path
must equal, bit for bit, one engine holding all experts on the rank's GPU."""
import os
import socket

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

H, I, E, K, T, WORLD = 512, 512, 16, 6, 8, 2
EPR = E // WORLD


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


def _rank_main(rank, port, q):
    import sys
    from datetime import timedelta
    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    sys.path.insert(0, root)
    try:
        import torch
        import torch.distributed as dist
        import dee_b200
        from dee_b200.ep import ExpertParallelMoE, ExpertParallelPeer
        from oracle import oracle as orc
        torch.cuda.set_device(rank)
        dist.init_process_group("nccl", init_method=f"tcp://127.0.0.1:{port}", rank=rank,
                                world_size=WORLD, timeout=timedelta(seconds=60),
                                device_id=torch.device("cuda", rank))
        layout = orc.Layout(H, I)
        recs = orc.synthetic_records(layout, E, seed=4242, kind="normal")

        def engine(n_exp, records):
            eng = dee_b200.new_engine(dee_b200.EngineConfig(hidden=H, inter=I, num_experts=n_exp, topk=K,
                                                            max_tokens=64, device_id=rank))
            bank = torch.from_numpy(np.ascontiguousarray(records)).cuda()
            eng.attach_bank(0, bank)
            return eng, bank

        full, bank_full = engine(E, recs)
        local, bank_local = engine(EPR, recs[rank * EPR:(rank + 1) * EPR])
        rng = np.random.default_rng(50 + rank)
        x16 = orc.f16_bits(rng.standard_normal((T, H)))
        ids = np.stack([rng.choice(E, K, replace=False) for _ in range(T)]).astype(np.int32)
        w = rng.random((T, K)).astype(np.float32)
        w /= w.sum(axis=1, keepdims=True)
        dx = torch.from_numpy(x16.view(np.float16)).cuda()
        dids = torch.from_numpy(ids).cuda()
        dw = torch.from_numpy(w).cuda()
        ref = torch.empty((T, H), dtype=torch.float32, device="cuda")
        full.moe_forward_device(0, dx.data_ptr(), T, d_ids_ptr=dids.data_ptr(), d_weights_ptr=dw.data_ptr(),
                                d_out_ptr=ref.data_ptr())
        results = {}
        peer = ExpertParallelPeer(torch, local, rank, WORLD, T, H)
        for step in range(3):
            out = peer.forward(dx, dids, dw)
        torch.cuda.synchronize()
        results["peer_status"] = local.sync_status()
        results["peer"] = bool(np.array_equal(out.cpu().numpy(), ref.cpu().numpy()))
        local2, bank_local2 = engine(EPR, recs[rank * EPR:(rank + 1) * EPR])
        coll = ExpertParallelMoE(torch, rank, WORLD, EPR, T, K, H, "cuda", engine=local2)
        out2 = coll.forward(dx, dids, dw)
        torch.cuda.synchronize()
        results["nccl"] = bool(np.array_equal(out2.cpu().numpy(), ref.cpu().numpy()))
        # the same over the counts exchange (occupied rows only)
        coll_c = ExpertParallelMoE(torch, rank, WORLD, EPR, T, K, H, "cuda", engine=local2, exchange="counts")
        out3 = coll_c.forward(dx, dids, dw)
        torch.cuda.synchronize()
        results["nccl_counts"] = bool(np.array_equal(out3.cpu().numpy(), ref.cpu().numpy()))
        results["journal"] = bool(np.array_equal(local.journal_ids(T), ids))
        dist.barrier()
        dist.destroy_process_group()
        q.put((rank, results))
    except Exception as exc:
        q.put((rank, {"error": repr(exc)}))


def test_expert_parallel_two_gpus_match_one_engine():
    import torch
    if not torch.cuda.is_available() or torch.cuda.device_count() < WORLD:
        pytest.skip(f"needs {WORLD} GPUs")
    import torch.multiprocessing as mp
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_rank_main, args=(r, port, q)) for r in range(WORLD)]
    for p in procs:
        p.start()
    results = dict(q.get(timeout=300) for _ in range(WORLD))
    for p in procs:
        p.join(timeout=60)
    for rank in range(WORLD):
        res = results[rank]
        assert "error" not in res, res
        assert res["peer_status"] == 0 and res["peer"] and res["nccl"] and res["nccl_counts"] and \
            res["journal"], (rank, res)
