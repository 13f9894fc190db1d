"""DEE4 expert-record layout and device-side synthetic expert banks.

One record holds one routed expert as ``[w1][w3][w2][w1.scale][w3.scale]
[w2.scale]`` (so-nerdyy/dee ``dee.cpp/include/dee/expert_store.h:28-46``,
``dee.cpp/kaggle/deepseek-v4-flash-0731/repack_to_dee4.py:42-55``): packed
E2M1 nibbles ``[out, in/2]`` (low nibble = even column) followed by UE8M0
scales ``[out, in/32]``.  At DeepSeek-V4 shapes (H=4096, I=2048) a record is
13,369,344 bytes.
"""
from __future__ import annotations

import ctypes
from dataclasses import dataclass

from . import _native


@dataclass(frozen=True)
class RecordLayout:
    hidden: int
    inter: int

    @property
    def ih(self) -> int:
        return self.hidden * self.inter

    @property
    def offsets(self) -> dict[str, int]:
        ih = self.ih
        s1 = ih + ih // 2
        return {"w1": 0, "w3": ih // 2, "w2": ih, "s1": s1, "s3": s1 + ih // 32,
                "s2": s1 + 2 * (ih // 32)}

    @property
    def bytes(self) -> int:
        return self.ih + self.ih // 2 + 3 * (self.ih // 32)


def synthetic_bank(layout: RecordLayout, experts: int, seed: int, std: float = 0.02,
                   device: str = "cuda", first_expert: int = 0):
    """[experts, record_bytes] uint8 on the device: N(0, std) weights packed by
    the device quantiser.  Expert first_expert + e draws from its own seeded
    generator, so a record does not depend on which experts are built with
    it (a rank of an expert-parallel run builds the same records as one GPU)."""
    import torch
    H, I = layout.hidden, layout.inter
    lib = _native.load()
    bank = torch.empty((experts, layout.bytes), dtype=torch.uint8, device=device)
    gen = torch.Generator(device=device)
    off = layout.offsets
    stream = torch.cuda.current_stream().cuda_stream
    for e in range(experts):
        gen.manual_seed(seed * 1_000_003 + first_expert + e)
        rec = bank[e]
        for name, (rows, cols) in (("w1", (I, H)), ("w3", (I, H)), ("w2", (H, I))):
            w = torch.randn((rows, cols), generator=gen, device=device, dtype=torch.float32) * std
            packed = rec[off[name]: off[name] + rows * cols // 2]
            sname = "s" + name[1]
            scale = rec[off[sname]: off[sname] + rows * cols // 32]
            rc = lib.dee_fp4_quantize_device(ctypes.c_void_p(w.data_ptr()), rows, cols,
                                             ctypes.c_void_p(packed.data_ptr()),
                                             ctypes.c_void_p(scale.data_ptr()), ctypes.c_void_p(stream))
            if rc != 0:
                raise RuntimeError(f"dee_fp4_quantize_device failed ({rc})")
    return bank
