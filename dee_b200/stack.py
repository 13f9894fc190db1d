"""A synthetic DeepSeek-V4-shaped MoE stack that drives the routed-expert
layer end to end (configurations 3 and 4 of the benchmark).

    embedding -> [RMSNorm, router logits, top-k, MoE, residual] x L
              -> RMSNorm -> LM head argmax (greedy decode)

Random-init weights with the layer's shapes: per layer a bank of E packed FP4
experts (layer 0 quantised from N(0, 0.02), later layers derived by
scrambling the packed nibbles with a per-layer hash, which keeps the scale
and value distribution), a router W_r [E, H] ~ N(0, 0.02); an FP16
embedding and LM head.  Every per-token step is computed in a fixed order
independent of the batch (the dense glue of stack.cu, the grouped GEMMs'
per-row results), so the route ids and tokens -- and the route journal --
are identical whether the b sequences are decoded on one GPU or spread over
N GPUs with expert parallelism (rank r holds experts [r*E/N, (r+1)*E/N) of
every layer and decodes sequences [r*b/N, (r+1)*b/N)).
"""
from __future__ import annotations

import ctypes
import hashlib
from dataclasses import dataclass

import numpy as np

from . import EngineConfig, _native, new_engine
from .records import RecordLayout, synthetic_bank


@dataclass
class StackSpec:
    layers: int = 43
    experts: int = 256
    hidden: int = 4096
    inter: int = 2048
    topk: int = 6
    vocab: int = 16384
    seed: int = 2026
    eps: float = 1e-6


class SyntheticStack:
    """One rank's share of the stack (world = 1: the whole stack on one GPU)."""

    def __init__(self, torch, spec: StackSpec, *, tokens: int, rank: int = 0, world: int = 1,
                 transport: str = "p2p", offload_slots: int = 0, store: str | None = None,
                 verify_store: bool = True):
        self.torch, self.spec, self.rank, self.world = torch, spec, rank, world
        self.tokens = tokens  # sequences decoded by this rank
        S = spec
        if S.experts % world:
            raise ValueError(f"{S.experts} experts do not split over {world} ranks")
        self.epr = S.experts // world
        dev = torch.device("cuda", torch.cuda.current_device())
        self._lib = _native.load()
        self.router = new_engine(EngineConfig(hidden=S.hidden, inter=S.inter, num_experts=S.experts,
                                              topk=S.topk, max_tokens=max(tokens, 8),
                                              device_id=dev.index))
        self.engine = new_engine(EngineConfig(hidden=S.hidden, inter=S.inter, num_experts=self.epr,
                                              topk=S.topk, num_layers=S.layers, max_tokens=max(tokens, 8),
                                              device_id=dev.index))
        layout = RecordLayout(S.hidden, S.inter)
        first = rank * self.epr
        self.offload = offload_slots > 0
        if self.offload and world > 1:
            raise ValueError("the offload tier runs on one GPU")
        self.store = None
        self.store_fill = None
        self.cold_reads = 0
        if store is not None:
            self._records_from_store(store, verify_store, layout, first, dev, offload_slots)
        else:
            self._synthetic_records(layout, first, dev, offload_slots)
        self._dense(dev, tokens, rank, world, transport)

    def _records_from_store(self, path, verify, layout, first, dev, offload_slots):
        """Every layer's records of this rank's experts from a DEE4 store on
        disk: straight into HBM through pinned staging buffers (resident), or
        into the offload tier's pinned host block.  With `verify` the seals
        are checked: while the fill streams whole segments in (one GPU: one
        pass over the disk), or at open when a rank reads a share of each."""
        from .store import Dee4Store, StoreError
        torch, S = self.torch, self.spec
        whole = self.world == 1
        st = Dee4Store(path, verify_segment_hashes=verify and not whole)
        st.check_layout(layout)
        if st.start_layer != 0 or st.num_layers < S.layers or st.experts_per_layer != S.experts:
            raise StoreError(f"store holds layers [{st.start_layer}, {st.start_layer + st.num_layers}) x "
                             f"{st.experts_per_layer} experts; the stack needs {S.layers} x {S.experts}")
        self.store = st
        n = S.layers * self.epr
        if not self.offload:
            block = torch.empty((n, layout.bytes), dtype=torch.uint8, device=dev)
            self.store_fill = st.upload_layers(0, S.layers, block.data_ptr(), block.numel(),
                                               torch.cuda.current_stream(), first_expert=first,
                                               experts=self.epr, verify=verify and whole)
            self.banks = [block[l * self.epr:(l + 1) * self.epr] for l in range(S.layers)]
            for layer, b in enumerate(self.banks):
                self.engine.attach_bank(layer, b)
        else:
            self.host = pinned_host_tensor(torch, n, layout.bytes)
            self.store_fill = st.read_layers(0, S.layers, self.host.data_ptr(), self.host.numel(),
                                             first_expert=first, experts=self.epr, verify=verify and whole)
            self.pool = torch.empty((offload_slots, layout.bytes), dtype=torch.uint8, device=dev)
            self.engine.offload_attach(self.host, S.layers, self.pool, offload_slots)
            self.banks = [self.pool]

    def _synthetic_records(self, layout, first, dev, offload_slots):
        torch, S = self.torch, self.spec
        base = synthetic_bank(layout, self.epr, seed=S.seed, first_expert=first)
        packed = S.hidden * S.inter * 3 // 2  # w1, w3, w2 packed bytes lead the record
        stream = torch.cuda.current_stream().cuda_stream

        def layer_bank(layer, out):
            if layer == 0:
                out.copy_(base)
                return
            rc = self._lib.dee_records_scramble_device(ctypes.c_void_p(base.data_ptr()),
                                                       ctypes.c_void_p(out.data_ptr()), self.epr, layout.bytes,
                                                       packed, layer, first, ctypes.c_void_p(stream))
            if rc != 0:
                raise RuntimeError(f"dee_records_scramble_device failed ({rc})")

        if not self.offload:
            self.banks = [base]
            for layer in range(1, S.layers):
                b = torch.empty_like(base)
                layer_bank(layer, b)
                self.banks.append(b)
            for layer, b in enumerate(self.banks):
                self.engine.attach_bank(layer, b)
        else:
            # every layer's records in pinned host memory, a shared device pool
            self.host = pinned_host_tensor(torch, S.layers * self.epr, layout.bytes)
            tmp = torch.empty_like(base)
            for layer in range(S.layers):
                layer_bank(layer, tmp)
                self.host[layer * self.epr:(layer + 1) * self.epr].copy_(tmp)
            del tmp
            self.pool = torch.empty((offload_slots, layout.bytes), dtype=torch.uint8, device=dev)
            self.engine.offload_attach(self.host, S.layers, self.pool, offload_slots)
            self.banks = [self.pool]

    def _dense(self, dev, tokens, rank, world, transport):
        torch, S = self.torch, self.spec
        g = torch.Generator(device=dev)
        g.manual_seed(S.seed)
        self.embed = torch.randn((S.vocab, S.hidden), generator=g, device=dev).to(torch.float16)
        self.lm_head = (torch.randn((S.vocab, S.hidden), generator=g, device=dev) * 0.02).to(torch.float16)
        self.w_r = torch.randn((S.layers, S.experts, S.hidden), generator=g, device=dev) * 0.02
        self.norm_w = torch.ones((S.layers + 1, S.hidden), device=dev)
        T, H = tokens, S.hidden
        self.x = torch.empty((T, H), dtype=torch.float32, device=dev)
        self.h = torch.empty((T, H), dtype=torch.float16, device=dev)
        self.logits = torch.empty((T, S.experts), dtype=torch.float32, device=dev)
        self.ids = torch.empty((T, S.topk), dtype=torch.int32, device=dev)
        self.w = torch.empty((T, S.topk), dtype=torch.float32, device=dev)
        self.out = torch.empty((T, H), dtype=torch.float32, device=dev)
        self.lm_logits = torch.empty((T, S.vocab), dtype=torch.float32, device=dev)
        self.ep = None
        self.transport = "single"
        if world > 1:
            from .ep import ExpertParallelMoE, ExpertParallelPeer
            if transport == "p2p":
                try:
                    self.ep = ExpertParallelPeer(torch, self.engine, rank, world, T, H)
                    self.transport = "p2p"
                except RuntimeError:
                    self.ep = None
            if self.ep is None:
                self.ep = ExpertParallelMoE(torch, rank, world, self.epr, T, S.topk, H, "cuda",
                                            engine=self.engine)
                self.transport = "nccl"

    def layer_records_host(self, layer: int):
        """uint8 numpy [experts of this rank, record_bytes] of one layer."""
        if self.offload:
            return self.host[layer * self.epr:(layer + 1) * self.epr].numpy()
        return self.banks[layer].cpu().numpy()

    def export_store(self, path: str, fmt: str = "dee4-v4-segmented") -> dict:
        """Write every layer's records as a DEE4 store (one GPU's full stack)."""
        from .store import write_store
        if self.world != 1:
            raise ValueError("export the stack from a one-GPU instance (a rank holds a share of the experts)")
        S = self.spec
        return write_store(path, RecordLayout(S.hidden, S.inter), S.layers, S.experts, self.layer_records_host,
                           fmt=fmt)

    def _h_ptr(self, t):
        return ctypes.c_void_p(t.data_ptr())

    def step(self, tok, next_tok, ids_log=None) -> None:
        """One greedy decode step on the current stream: tok int32 [T] ->
        next_tok int32 [T]; ids_log (int32 [L, T, K]) receives the route ids."""
        S, lib, e = self.spec, self._lib, self.engine
        st = ctypes.c_void_p(self.torch.cuda.current_stream().cuda_stream)
        T = self.tokens
        chk = e._check
        chk(lib.dee_stack_embed_device(e._h, self._h_ptr(self.embed), self._h_ptr(tok), T, S.vocab,
                                       self._h_ptr(self.x), st), "stack_embed")
        for layer in range(S.layers):
            chk(lib.dee_stack_rmsnorm_device(e._h, self._h_ptr(self.x), self._h_ptr(self.norm_w[layer]),
                                             S.eps, T, self._h_ptr(self.h), st), "stack_rmsnorm")
            chk(lib.dee_stack_router_logits_device(e._h, self._h_ptr(self.h), self._h_ptr(self.w_r[layer]), T,
                                                   S.experts, self._h_ptr(self.logits), st), "router_logits")
            if self.ep is None and not self.offload:
                # every expert resident on this GPU: routing and the layer in
                # one call (the router runs inside the grouping kernel or the
                # one-launch layer; the same ids as the router engine's)
                e.moe_forward_routed_device(layer, self.h.data_ptr(), T, self.logits.data_ptr(),
                                            self.ids.data_ptr(), self.w.data_ptr(), d_out_ptr=self.out.data_ptr(),
                                            stream=st.value)
                out = self.out
            else:
                self.router.route_topk_device(self.logits.data_ptr(), T, self.ids.data_ptr(), self.w.data_ptr(),
                                              st.value)
                if self.offload:
                    self.cold_reads += e.offload_prepare_device(layer, self.ids.data_ptr(), T, st.value)
                if self.ep is None:
                    e.moe_forward_device(layer, self.h.data_ptr(), T, d_ids_ptr=self.ids.data_ptr(),
                                         d_weights_ptr=self.w.data_ptr(), d_out_ptr=self.out.data_ptr(),
                                         stream=st.value)
                    out = self.out
                else:
                    out = self.ep.forward(self.h, self.ids, self.w, layer=layer)
            if ids_log is not None:
                ids_log[layer].copy_(self.ids)
            chk(lib.dee_stack_residual_add_device(e._h, self._h_ptr(self.x), self._h_ptr(out), T, st),
                "residual_add")
        chk(lib.dee_stack_rmsnorm_device(e._h, self._h_ptr(self.x), self._h_ptr(self.norm_w[S.layers]), S.eps,
                                         T, self._h_ptr(self.h), st), "final rmsnorm")
        chk(lib.dee_stack_lm_head_argmax_device(e._h, self._h_ptr(self.h), self._h_ptr(self.lm_head), T, S.vocab,
                                                self._h_ptr(self.lm_logits), self._h_ptr(next_tok), st),
            "lm_head_argmax")

    def decode(self, first_tokens, steps: int, ids_log=None, tok_log=None):
        """Greedy decode from first_tokens (int32 [T], device) for `steps`
        steps; ids_log int32 [steps, L, T, K] and tok_log int32 [steps, T]
        (optional, device) record every step."""
        torch = self.torch
        a = first_tokens.clone()
        b = torch.empty_like(a)
        for s in range(steps):
            self.step(a, b, None if ids_log is None else ids_log[s])
            if tok_log is not None:
                tok_log[s].copy_(b)
            a, b = b, a
        return a


class _PinnedBlock:
    """Owns an exactly sized pinned host allocation (freed with the object)."""

    def __init__(self, nbytes: int):
        self._lib = _native.load()
        self.ptr = ctypes.c_void_p()
        rc = self._lib.dee_host_alloc_pinned(nbytes, ctypes.byref(self.ptr))
        if rc != 0:
            raise MemoryError(f"pinned host allocation of {nbytes} bytes failed ({rc})")
        self.nbytes = nbytes

    def __del__(self):
        if getattr(self, "ptr", None) and self.ptr.value:
            self._lib.dee_host_free_pinned(self.ptr)
            self.ptr = ctypes.c_void_p()


def pinned_host_tensor(torch, rows: int, cols: int):
    """uint8 CPU tensor [rows, cols] in exactly rows*cols bytes of pinned memory."""
    block = _PinnedBlock(rows * cols)
    arr = np.ctypeslib.as_array((ctypes.c_uint8 * (rows * cols)).from_address(block.ptr.value))
    t = torch.from_numpy(arr).view(rows, cols)
    t._dee_block = block  # the tensor keeps the allocation alive
    return t


def seed_tokens(spec: StackSpec, batch: int) -> np.ndarray:
    """The b seeded first tokens of the greedy decode."""
    return np.random.default_rng(spec.seed + 1).integers(0, spec.vocab, batch).astype(np.int32)


def journal_bytes(ids_all: np.ndarray, *, run_id: str, prompt_len: int = 1) -> bytes:
    """The route journal of a whole decode (ids_all int32 [steps, L, b, K], all
    sequences in order) in the reference's JSONL format, as bytes."""
    import os
    import tempfile
    from .journal import RouteJournal
    steps, L, b, K = ids_all.shape
    with tempfile.TemporaryDirectory() as td:
        path = os.path.join(td, "routed_experts.jsonl")
        j = RouteJournal(path, run_id=run_id, n_layers=L, topk=K, fsync=False)
        for s in range(steps):
            for layer in range(L):
                j.append_layer(step=s, start_pos=prompt_len - 1 + s, layer=layer, device="cuda:0",
                               expert_ids=ids_all[s, layer])
        j.close()
        with open(path, "rb") as f:
            return f.read()


def sha256(b: bytes) -> str:
    return hashlib.sha256(b).hexdigest()
