"""Generate the golden fixtures in this directory from the reference itself.

Run where so-nerdyy/dee is checked out (its root in ``DEE_REFERENCE_ROOT``,
else the default of ``REF`` below):

    python tests/golden/make_golden.py

It imports the reference's Python FP32 semantics and route-journal writer and
records their outputs on small seeded inputs:

* ``quant.npz``   -- ``fp4_act_quant_inplace`` (deepseek_v4_layer_common.py
                     :246-266) on N(0, 0.02) weights: the quantise/dequantise
                     round trip every synthetic record follows.
* ``decode.npz``  -- ``dequantize_expert_weight`` (deepseek_v4_expert_reference
                     .py:85-99) on random packed bytes and scale bytes 1..254.
Synthetic expert records are not stored: the tests regenerate them with
``oracle.synthetic_records`` from the recorded seed and check the recorded
sha256 before use.

* ``expert.npz``  -- ``expert_forward`` (:102-129) FP32 outputs of three
                     packed experts, with and without the clamp at 10.
* ``moe_layer.npz`` -- ``moe_layer_forward`` (deepseek_v4_moe_reference.py
                     :113-203): the official sqrt-softplus router with bias,
                     top-6, weights, and the layer output (no shared expert).
* ``official.npz`` -- ``moe_layer_forward`` with a shared expert (F8_E4M3
                     weights, E8M0 scales per 128 x 128 tile): routed outputs
                     weighted before w2, clamp 10, shared output added.
* ``act_quant.npz`` -- ``act_quant_inplace`` (deepseek_v4_layer_common.py
                     :213-240) with UE8M0 scales, blocks of 128 and 32, on FP16
                     rows spanning seven decades of magnitude.
* ``journal.jsonl`` -- ``RoutedExpertJournal`` (kaggle/deepseek-v4-flash-0731/
                     deepseek_v4_native_generate.py:452-622) for two forwards
                     of three layers with fixed route ids.

The fixtures are small (a few hundred KB) and are committed; the tests never
read the reference at run time.
"""
from __future__ import annotations

import os
import sys
import tempfile
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
REPO = HERE.parent.parent
REF = Path(os.environ.get("DEE_REFERENCE_ROOT", Path(__file__).resolve().parents[3] / "reference")) / "dee.cpp"
sys.path.insert(0, str(REF))
sys.path.insert(0, str(REF / "kaggle" / "deepseek-v4-flash-0731"))
sys.path.insert(0, str(REPO))

import torch  # noqa: E402

from scripts import deepseek_v4_expert_reference as ds7  # noqa: E402
from scripts import deepseek_v4_layer_common as common  # noqa: E402
from scripts import deepseek_v4_moe_reference as moe  # noqa: E402

from oracle import oracle as orc  # noqa: E402


def _sha(a: np.ndarray) -> str:
    import hashlib
    return hashlib.sha256(np.ascontiguousarray(a).tobytes()).hexdigest()


def make_quant() -> None:
    rng = np.random.default_rng(101)
    w = (rng.standard_normal((64, 256)) * 0.02).astype(np.float32)
    w[3, :32] = 0.0                      # an all-zero block (amax floor)
    w[5, 40] = 1e-30                     # a tiny value
    w[7, 64:96] = np.linspace(-0.3, 0.3, 32, dtype=np.float32)  # grid ties
    wq = common.fp4_act_quant_inplace(torch.from_numpy(w.copy()), 32).numpy()
    np.savez_compressed(HERE / "quant.npz", w=w, wq=wq)


def make_decode() -> None:
    rng = np.random.default_rng(202)
    packed = rng.integers(0, 256, (32, 64), dtype=np.uint8)
    scale = rng.integers(1, 255, (32, 4), dtype=np.uint8)
    scale[0] = [1, 127, 254, 0x7D]
    w = ds7.dequantize_expert_weight(torch.from_numpy(packed), torch.from_numpy(scale)).numpy()
    np.savez_compressed(HERE / "decode.npz", packed=packed, scale=scale, w=w)


def make_expert() -> None:
    layout = orc.Layout(512, 512)
    recs = orc.synthetic_records(layout, 3, seed=303, kind="normal")
    rng = np.random.default_rng(304)
    x = rng.standard_normal((5, 512)).astype(np.float16).astype(np.float32)
    ys = {}
    for limit in (0.0, 10.0):
        out = []
        for e in range(3):
            t = {k: torch.from_numpy(v.copy()) for k, v in orc.split_record(layout, recs[e]).items()}
            y = ds7.expert_forward(torch.from_numpy(x), t["w1.weight"], t["w1.scale"],
                                   t["w2.weight"], t["w2.scale"], t["w3.weight"], t["w3.scale"],
                                   swiglu_limit=limit)
            out.append(y.numpy())
        ys[f"y_limit{int(limit)}"] = np.stack(out)
    np.savez_compressed(HERE / "expert.npz", records_seed=303, records_sha256=_sha(recs), x=x, **ys)


def make_moe_layer() -> None:
    layout = orc.Layout(512, 512)
    E = 16
    recs = orc.synthetic_records(layout, E, seed=404, kind="normal")
    rng = np.random.default_rng(405)
    x = rng.standard_normal((7, 512)).astype(np.float32)
    gate_w = (rng.standard_normal((E, 512)) * 0.05).astype(np.float32)
    bias = (rng.standard_normal(E) * 0.1).astype(np.float32)
    routed = {e: {k: torch.from_numpy(v.copy()) for k, v in orc.split_record(layout, recs[e]).items()}
              for e in range(E)}
    res = moe.moe_layer_forward(torch.from_numpy(x), torch.from_numpy(gate_w), torch.from_numpy(bias),
                                routed, None, topk=6, route_scale=1.5, score_func="sqrtsoftplus",
                                swiglu_limit=10.0)
    # the router's logits by the reference's own expression (router_scores :146)
    logits = (torch.from_numpy(x).float() @ torch.from_numpy(gate_w).float().transpose(0, 1)).numpy()
    # a hash layer (router_select with tid2eid, layer_common.py:387-392)
    tid2eid = np.stack([rng.choice(E, 6, replace=False) for _ in range(50)]).astype(np.int64)
    input_ids = rng.integers(0, 50, 7).astype(np.int64)
    _, h_idx, h_w = common.router_select(torch.from_numpy(x), torch.from_numpy(gate_w), None,
                                         tid2eid=torch.from_numpy(tid2eid),
                                         input_ids=torch.from_numpy(input_ids), topk=6,
                                         route_scale=1.5, score_func="sqrtsoftplus")
    np.savez_compressed(HERE / "moe_layer.npz", records_seed=404, records_sha256=_sha(recs), x=x,
                        gate_w=gate_w, bias=bias, logits=logits, tid2eid=tid2eid,
                        input_ids=input_ids, hash_ids=h_idx.numpy(), hash_weights=h_w.numpy(),
                        scores=res["scores"].numpy(), expert_ids=res["expert_ids"].numpy(),
                        routing_weights=res["routing_weights"].numpy(),
                        moe_output=res["moe_output"].numpy())


def make_official() -> None:
    """The official layer with a shared expert, at shapes the kernels take."""
    layout = orc.Layout(512, 512)
    E = 16
    recs = orc.synthetic_records(layout, E, seed=606, kind="normal")
    rng = np.random.default_rng(607)
    g = torch.Generator().manual_seed(608)
    x = rng.standard_normal((5, 512)).astype(np.float16).astype(np.float32)
    gate_w = (rng.standard_normal((E, 512)) * 0.05).astype(np.float32)
    bias = (rng.standard_normal(E) * 0.1).astype(np.float32)
    shared = {}
    for name, (rows, cols) in (("w1", (256, 512)), ("w3", (256, 512)), ("w2", (512, 256))):
        w8 = (torch.randn(rows, cols, generator=g) * 2.0).to(torch.float8_e4m3fn)
        sc = torch.randint(0x76, 0x7B, ((rows + 127) // 128, (cols + 127) // 128), generator=g,
                           dtype=torch.uint8)
        shared[f"{name}.weight"] = w8
        shared[f"{name}.scale"] = sc
    routed = {e: {k: torch.from_numpy(v.copy()) for k, v in orc.split_record(layout, recs[e]).items()}
              for e in range(E)}
    res = moe.moe_layer_forward(torch.from_numpy(x), torch.from_numpy(gate_w), torch.from_numpy(bias),
                                routed, shared, topk=6, route_scale=1.5, score_func="sqrtsoftplus",
                                swiglu_limit=10.0)
    np.savez_compressed(
        HERE / "official.npz", records_seed=606, records_sha256=_sha(recs), x=x,
        sh_w1=shared["w1.weight"].view(torch.uint8).numpy(), sh_s1=shared["w1.scale"].numpy(),
        sh_w3=shared["w3.weight"].view(torch.uint8).numpy(), sh_s3=shared["w3.scale"].numpy(),
        sh_w2=shared["w2.weight"].view(torch.uint8).numpy(), sh_s2=shared["w2.scale"].numpy(),
        expert_ids=res["expert_ids"].numpy(), routing_weights=res["routing_weights"].numpy(),
        shared_output=res["shared_output"].numpy(), moe_output=res["moe_output"].numpy())


def make_act_quant() -> None:
    rng = np.random.default_rng(2027)
    rows, cols = 48, 512
    mag = 10.0 ** rng.uniform(-3, 3, size=(rows, 1))
    x = torch.from_numpy((rng.standard_normal((rows, cols)) * mag).astype(np.float16))
    out = {"x": x.numpy().view(np.uint16)}
    for block in (128, 32):
        y = common.act_quant_inplace(x.clone(), block_size=block, scale_fmt="ue8m0")
        out[f"y{block}"] = y.numpy().view(np.uint16)
    np.savez_compressed(HERE / "act_quant.npz", **out)


def make_journal() -> None:
    import deepseek_v4_native_generate as gen
    rng = np.random.default_rng(505)
    with tempfile.TemporaryDirectory() as td:
        path = Path(td) / "routed_experts.jsonl"
        j = gen.RoutedExpertJournal(path, run_id="golden-run", n_layers=3, topk=6)
        ids_all = []
        for step, rows in ((0, 4), (1, 2)):
            for layer in range(3):
                ids = np.stack([rng.choice(256, 6, replace=False) for _ in range(rows)]).astype(np.int32)
                ids_all.append(ids)
                j.append_layer(step=step, start_pos=0 if step == 0 else 4, layer=layer,
                               device="cuda:0", expert_ids=ids)
        j.close()
        (HERE / "journal.jsonl").write_text(path.read_text("utf-8"), "utf-8")
    np.savez_compressed(HERE / "journal_ids.npz", *ids_all)


def main() -> None:
    torch.manual_seed(0)
    makers = {"quant": make_quant, "decode": make_decode, "expert": make_expert, "moe_layer": make_moe_layer,
              "official": make_official, "act_quant": make_act_quant, "journal": make_journal}
    for name in sys.argv[1:] or list(makers):  # default: all
        makers[name]()
    for p in sorted(HERE.iterdir()):
        if p.suffix in (".npz", ".jsonl"):
            print(p.name, p.stat().st_size)


if __name__ == "__main__":
    main()
