"""Expert-parallel routed-expert layer: one rank's share, over torch.distributed.

Rank r of `world` owns experts [r*epr, (r+1)*epr) (epr = experts per rank),
the official DeepSeek-V4 split (benchmark_reports/deepseek-v4-flash-0731-t4/
official-source/inference/model.py:625-626).  Its engine is configured with
num_experts = epr and holds those records.  Tokens are routed on their owner
rank with the same router as one GPU, so the route ids (and the journal) do
not depend on the GPU count.  A layer call on this rank's T tokens:

  1. pack: selections sorted by owner rank into `capacity` rows per rank
     (FP16 hidden row + the owner's local expert id, -1 unused);
  2. all-to-all of the rows and the expert ids: either equal blocks of
     `capacity` rows per rank pair (no host synchronisation, no split
     sizes: the choice for decode-sized layers, where the padded bytes cost
     less than a host round trip), or -- above `counts_rows` padded rows --
     an all-to-all of the per-destination counts, one host read of them, and
     all-to-alls of the occupied rows only;
  3. the grouped expert GEMMs over the received rows;
  4. all-to-all of the FP32 output rows back to their tokens' owners;
  5. the rank-order FP32 combine.

torch.distributed (NCCL on GPUs) is the transport; the packing, GEMMs and
combine are the engine's kernels (`ops=None`).  Tests pass other `ops` with
the same contracts to run the choreography on CPU ranks.
"""
from __future__ import annotations

from dataclasses import dataclass
from typing import Any, Callable


@dataclass
class EpOps:
    """The three device steps of a layer call.

    pack(ids, x, send_rows, send_expert, slot_of_pos)
    compute(recv_rows, recv_expert, raw, layer)
    combine(back, slot_of_pos, weights, out)
    """

    pack: Callable[..., None]
    compute: Callable[..., None]
    combine: Callable[..., None]


def engine_ops(engine, world: int, experts_per_rank: int, capacity: int,
               stream_of: Callable[[], Any]) -> EpOps:
    """EpOps over a dee_b200.Engine (device tensors, the current CUDA stream)."""

    def pack(ids, x, send_rows, send_expert, slot_of_pos):
        engine.ep_pack_device(ids.data_ptr(), ids.shape[0], x.data_ptr(), world, experts_per_rank,
                              capacity, send_rows.data_ptr(), send_expert.data_ptr(),
                              slot_of_pos.data_ptr(), stream_of())

    def compute(recv_rows, recv_expert, raw, layer):
        engine.moe_forward_rows_device(layer, recv_rows.data_ptr(), recv_expert.data_ptr(),
                                       recv_rows.shape[0], raw.data_ptr(), stream_of())

    def combine(back, slot_of_pos, weights, out):
        engine.ep_combine_device(back.data_ptr(), slot_of_pos.data_ptr(), weights.data_ptr(),
                                 out.shape[0], out.data_ptr(), stream_of())

    return EpOps(pack, compute, combine)


class ExpertParallelMoE:
    """One rank's share of an expert-parallel MoE layer with fixed T tokens per rank.

    All ranks must call forward() together with the same `tokens`; buffers
    are allocated once.  `capacity` defaults to tokens * topk, which covers
    any routing (a rank can receive at most all selections of another).
    """

    def __init__(self, torch_mod, rank: int, world: int, experts_per_rank: int, tokens: int,
                 topk: int, hidden: int, device, *, engine=None, layer: int = 0,
                 capacity: int | None = None, group=None, ops: EpOps | None = None,
                 exchange: str = "auto", counts_rows: int = 4096):
        self.torch = torch_mod
        self.dist = torch_mod.distributed
        self.rank, self.world, self.epr = rank, world, experts_per_rank
        self.tokens, self.topk, self.hidden = tokens, topk, hidden
        self.capacity = capacity if capacity is not None else tokens * topk
        self.group = group
        if ops is None:
            if engine is None:
                raise ValueError("ExpertParallelMoE needs an engine or explicit ops")
            cuda = torch_mod.cuda
            ops = engine_ops(engine, world, experts_per_rank, self.capacity,
                             lambda: cuda.current_stream())
        self.ops = ops
        self.layer = layer
        n = world * self.capacity
        t = torch_mod
        self.send_rows = t.empty((n, hidden), dtype=t.float16, device=device)
        self.send_expert = t.empty((n,), dtype=t.int32, device=device)
        self.recv_rows = t.empty((n, hidden), dtype=t.float16, device=device)
        self.recv_expert = t.empty((n,), dtype=t.int32, device=device)
        self.slot_of_pos = t.empty((tokens * topk,), dtype=t.int32, device=device)
        self.raw = t.zeros((n, hidden), dtype=t.float32, device=device)
        self.back = t.empty((n, hidden), dtype=t.float32, device=device)
        self.out = t.empty((tokens, hidden), dtype=t.float32, device=device)
        if exchange not in ("auto", "fixed", "counts"):
            raise ValueError(f"exchange must be auto, fixed or counts, not {exchange!r}")
        self.counts_mode = exchange == "counts" or (exchange == "auto" and n >= counts_rows)
        self.device = device

    def forward(self, x, ids, weights, layer: int | None = None):
        """x FP16 [T, H], ids int32 [T, K] (global expert ids), weights FP32
        [T, K] -> FP32 [T, H] (a view of an internal buffer, valid until the
        next call).  `layer` selects the engine's expert bank (default: the
        constructor's)."""
        shapes_ok = (tuple(ids.shape) == (self.tokens, self.topk) and
                     tuple(x.shape) == (self.tokens, self.hidden))
        if not shapes_ok:
            raise ValueError(f"expected x [{self.tokens}, {self.hidden}] and ids [{self.tokens}, "
                             f"{self.topk}], got {tuple(x.shape)} and {tuple(ids.shape)}")
        self.ops.pack(ids, x, self.send_rows, self.send_expert, self.slot_of_pos)
        lyr = self.layer if layer is None else layer
        if self.counts_mode:
            self._exchange_counts(lyr)
        else:
            # FP16 rows travel as int32 pairs: a bitwise view every backend moves
            i32 = self.torch.int32
            self.dist.all_to_all_single(self.recv_rows.view(i32), self.send_rows.view(i32),
                                        group=self.group)
            self.dist.all_to_all_single(self.recv_expert, self.send_expert, group=self.group)
            self.ops.compute(self.recv_rows, self.recv_expert, self.raw, lyr)
            self.dist.all_to_all_single(self.back, self.raw, group=self.group)
        self.ops.combine(self.back, self.slot_of_pos, weights, self.out)
        return self.out

    def _exchange_counts(self, layer) -> None:
        """Occupied rows only.  Pack fills each destination's block from its
        start, so block d's first send_n[d] rows are the ones to send; they
        land at the start of this rank's block on the owner, the rest of the
        owner's block is marked unused (-1), and the returned rows land where
        the fixed exchange would put them, so slot_of_pos and the combine are
        unchanged."""
        t, dist, W, C = self.torch, self.dist, self.world, self.capacity
        i32, i64 = t.int32, t.int64
        send_n = (self.send_expert.view(W, C) >= 0).sum(dim=1).to(i64)
        recv_n = t.empty_like(send_n)
        dist.all_to_all_single(recv_n, send_n, group=self.group)
        s_list, r_list = send_n.tolist(), recv_n.tolist()  # the one host read of the layer

        def rows_index(counts):
            idx = [d * C + i for d, k in enumerate(counts) for i in range(k)]
            return t.tensor(idx, dtype=i64, device=self.device)

        s_idx, r_idx = rows_index(s_list), rows_index(r_list)
        rows32 = self.send_rows.view(i32)
        recv32 = self.recv_rows.view(i32)
        send_c = rows32.index_select(0, s_idx)
        recv_c = t.empty((len(r_idx), rows32.shape[1]), dtype=i32, device=self.device)
        dist.all_to_all_single(recv_c, send_c, output_split_sizes=r_list, input_split_sizes=s_list,
                               group=self.group)
        exp_c = self.send_expert.index_select(0, s_idx)
        recv_e = t.empty(len(r_idx), dtype=i32, device=self.device)
        dist.all_to_all_single(recv_e, exp_c, output_split_sizes=r_list, input_split_sizes=s_list,
                               group=self.group)
        self.recv_expert.fill_(-1)
        recv32.index_copy_(0, r_idx, recv_c)
        self.recv_expert.index_copy_(0, r_idx, recv_e)
        self.ops.compute(self.recv_rows, self.recv_expert, self.raw, layer)
        raw_c = self.raw.index_select(0, r_idx)
        back_c = t.empty((len(s_idx), self.hidden), dtype=self.raw.dtype, device=self.device)
        dist.all_to_all_single(back_c, raw_c, output_split_sizes=s_list, input_split_sizes=r_list,
                               group=self.group)
        self.back.index_copy_(0, s_idx, back_c)


class ExpertParallelPeer:
    """The same layer over NVLink peer memory instead of a collective library.

    Every rank's engine exports an exchange block with CUDA IPC; the blocks
    are mapped once (handles exchanged with all_gather_object).  A layer call
    is one engine call: the selections are written straight into the expert
    owners' receive buffers, the down-projection epilogue writes each output
    row straight back into the token owner's return buffer, and per-source
    epoch flags (bounded waits) order the phases.  Requires peer access
    between the ranks' GPUs.
    """

    def __init__(self, torch_mod, engine, rank: int, world: int, tokens: int, hidden: int, *,
                 layer: int = 0, group=None):
        self.torch = torch_mod
        self.engine = engine
        self.layer = layer
        self.tokens = tokens
        dist = torch_mod.distributed
        err = None
        handle = None
        try:
            handle, _ = engine.ep_p2p_init(world, rank, tokens)
        except Exception as exc:
            err = f"rank {rank}: {exc}"
        handles = [None] * world
        dist.all_gather_object(handles, handle, group=group)
        if err is None and all(h is not None for h in handles):
            try:
                engine.ep_p2p_connect(handles)
            except Exception as exc:
                err = f"rank {rank}: {exc}"
        elif err is None:
            err = "a peer could not export its exchange block"
        # every rank takes the same decision
        errors = [None] * world
        dist.all_gather_object(errors, err, group=group)
        failed = [e for e in errors if e]
        if failed:
            raise RuntimeError("NVLink peer path unavailable: " + "; ".join(failed))
        self.out = torch_mod.empty((tokens, hidden), dtype=torch_mod.float32, device="cuda")

    def forward(self, x, ids, weights, layer: int | None = None):
        """x FP16 [T, H], ids int32 [T, K] (global), weights FP32 [T, K] ->
        FP32 [T, H] (an internal buffer, valid until the next call)."""
        self.engine.ep_p2p_forward_device(self.layer if layer is None else layer, x.data_ptr(), ids.data_ptr(),
                                          weights.data_ptr(), self.out.data_ptr(),
                                          self.torch.cuda.current_stream())
        return self.out
