"""Device-resident quantized expert pools and per-layer slot tables.

The reference keeps, per layer, a packed pool ``(cap, *shape)`` per tensor key
plus an ``int32[num_experts]`` expert->slot table initialised to -1
(mlx_streaming/core/cache/resident_pool.py:549-558; native/ext/pool/
demand.cpp:286-310). Each expert's bytes follow the blob layout of
mlx_streaming/prep/blob_layout.py:14-32: gate{w,s,b}, up{w,s,b},
down{w,s,b}. Here every pool lives in HBM for the whole run; there is no SSD
streaming, eviction or residency miss handling in the timed path.
"""
from __future__ import annotations

from dataclasses import dataclass

import torch

from . import _lib
from ._lib import VbQuantPool, check, lib

KEYS = ("gate_w", "gate_s", "gate_b", "up_w", "up_s", "up_b",
        "down_w", "down_s", "down_b")


def stream_handle(stream=None) -> int:
    s = stream if stream is not None else torch.cuda.current_stream()
    return s.cuda_stream


def ptr(t) -> int | None:
    return None if t is None else t.data_ptr()


def blob_layout(hidden: int, inter: int, bits: int, group: int):
    """Segments ``(key, shape, dtype, nbytes, offset)`` and the row stride of
    one expert blob (blob_layout.py:18-32, affine format v1)."""
    segs, off = [], 0
    for proj, out_d, in_d in (("gate", inter, hidden), ("up", inter, hidden),
                              ("down", hidden, inter)):
        words = in_d * bits // 32
        groups = in_d // group
        for key, shape, dt, nb in ((f"{proj}_w", (out_d, words), torch.int32, out_d * words * 4),
                                   (f"{proj}_s", (out_d, groups), torch.bfloat16, out_d * groups * 2),
                                   (f"{proj}_b", (out_d, groups), torch.bfloat16, out_d * groups * 2)):
            segs.append((key, shape, dt, nb, off))
            off += nb
    return segs, off


@dataclass
class QuantPool:
    """A pool of ``cap`` expert slots in the nine-tensor MLX affine format.

    Either nine stacked tensors (``tensors``) or one uint8 blob tensor of
    shape ``[cap, stride]`` whose rows follow :func:`blob_layout`.
    """
    hidden: int
    inter: int
    bits: int
    group: int
    cap: int
    tensors: dict | None = None
    blob: torch.Tensor | None = None
    blob_slot0: int = 0

    @classmethod
    def empty_blob(cls, cap: int, hidden: int, inter: int, bits: int = 4,
                   group: int = 64, device="cuda") -> "QuantPool":
        _, stride = blob_layout(hidden, inter, bits, group)
        blob = torch.empty((cap, stride), dtype=torch.uint8, device=device)
        return cls(hidden, inter, bits, group, cap, blob=blob)

    @classmethod
    def from_tensors(cls, tensors: dict, hidden: int, inter: int, bits: int,
                     group: int) -> "QuantPool":
        cap = int(tensors["gate_w"].shape[0])
        for k in KEYS:
            assert tensors[k].is_contiguous(), k
        return cls(hidden, inter, bits, group, cap, tensors=dict(tensors))

    def view(self, first_slot: int, cap: int) -> "QuantPool":
        """A sub-pool of ``cap`` slots starting at ``first_slot`` (blob pools)."""
        assert self.blob is not None
        return QuantPool(self.hidden, self.inter, self.bits, self.group, cap,
                         blob=self.blob, blob_slot0=self.blob_slot0 + first_slot)

    @property
    def stride(self) -> int:
        return blob_layout(self.hidden, self.inter, self.bits, self.group)[1]

    def c_struct(self) -> VbQuantPool:
        s = VbQuantPool()
        if self.blob is not None:
            segs, stride = blob_layout(self.hidden, self.inter, self.bits, self.group)
            base = self.blob.data_ptr() + self.blob_slot0 * stride
            for i, (_, _, _, _, off) in enumerate(segs):
                s.ptr[i] = base + off
                s.slot_stride[i] = stride
        else:
            for i, k in enumerate(KEYS):
                t = self.tensors[k]
                s.ptr[i] = t.data_ptr()
                s.slot_stride[i] = t[0].numel() * t.element_size()
        s.cap = self.cap
        return s

    def slot_tensors(self, slot: int) -> dict:
        """The nine tensors of one slot (views for blob pools)."""
        if self.tensors is not None:
            return {k: self.tensors[k][slot] for k in KEYS}
        segs, stride = blob_layout(self.hidden, self.inter, self.bits, self.group)
        row = self.blob[self.blob_slot0 + slot]
        out = {}
        for key, shape, dt, nb, off in segs:
            out[key] = row[off:off + nb].view(dt).view(shape)
        return out

    def fill_synthetic(self, slot: int, seed: int, scale_lo=0.002, scale_hi=0.02,
                       stream=None) -> None:
        """Seeded synthetic expert: uniform 4-bit codes, scales U(lo, hi) in
        bf16 and biases = -8*scale (the benchmark configs' weight format)."""
        st = stream_handle(stream)
        t = self.slot_tensors(slot)
        for j, proj in enumerate(("gate", "up", "down")):
            w = t[f"{proj}_w"]
            check(lib.vb_synth_fill_u32(w.data_ptr(), w.numel(), _mix(seed, 3 * j), st),
                  "vb_synth_fill_u32")
            s, b = t[f"{proj}_s"], t[f"{proj}_b"]
            check(lib.vb_synth_fill_scales(s.data_ptr(), b.data_ptr(), s.numel(),
                                           _mix(seed, 3 * j + 1), scale_lo, scale_hi,
                                           -8.0, st), "vb_synth_fill_scales")

    def fill_synthetic_many(self, slots, seeds, scale_lo=0.002, scale_hi=0.02,
                            stream=None, bias_mul: float = -8.0) -> None:
        """:meth:`fill_synthetic` of every ``(slot, seed)`` pair in one launch."""
        import ctypes as C
        n = len(slots)
        assert n == len(seeds)
        if n == 0:
            return
        sl = (C.c_int32 * n)(*[int(s) for s in slots])
        sd = (C.c_uint64 * n)(*[int(s) for s in seeds])
        check(lib.vb_synth_fill_pool(C.byref(self.c_struct()), sl, sd, n, self.hidden,
                                     self.inter, self.bits, self.group, scale_lo, scale_hi,
                                     bias_mul, stream_handle(stream)), "vb_synth_fill_pool")

    def to_numpy_slot(self, slot: int) -> dict:
        """Copy one slot back to host numpy arrays (uint32 words, uint16 bf16
        bits) in the oracle's nine-array format."""
        import numpy as np
        t = self.slot_tensors(slot)
        out = {}
        for k in KEYS:
            v = t[k].contiguous().cpu()
            if k.endswith("_w"):
                out[k] = v.numpy().view(np.uint32)[None]
            else:
                out[k] = v.view(torch.int16).numpy().view(np.uint16)[None]
        return out


def _mix(seed: int, salt: int) -> int:
    z = (seed * 0x9E3779B97F4A7C15 + salt * 0xBF58476D1CE4E5B9 + 0x94D049BB133111EB) & (2**64 - 1)
    z ^= z >> 31
    return z


def expert_seed(base: int, layer: int, expert: int) -> int:
    """Seed of expert ``expert`` of layer ``layer`` in a synthetic model."""
    return _mix(_mix(base, layer + 1), expert + 7)


def make_table(num_experts: int, slots_of: dict[int, int], device="cuda") -> torch.Tensor:
    """``int32[num_experts]`` expert->slot table, -1 = not resident
    (resident_pool.py:549-558)."""
    t = torch.full((num_experts,), -1, dtype=torch.int32)
    for e, s in slots_of.items():
        t[int(e)] = int(s)
    return t.to(device)


def slot_remap(ids: torch.Tensor, table: torch.Tensor, miss_count=None,
               status=None, stream=None) -> torch.Tensor:
    """``local = table[ids]`` on the device (-1 where not resident)."""
    ids = ids.contiguous()
    assert ids.dtype in (torch.int32, torch.uint32)
    local = torch.empty(ids.shape, dtype=torch.int32, device=ids.device)
    check(lib.vb_slot_remap(ids.data_ptr(), table.data_ptr(), local.data_ptr(), ids.numel(),
                            table.numel(), ptr(miss_count), ptr(status), stream_handle(stream)),
          "vb_slot_remap")
    return local


__all__ = ["QuantPool", "blob_layout", "make_table", "slot_remap", "expert_seed",
           "KEYS", "stream_handle", "ptr", "_lib"]
