"""Drop-in mirror of the reference's ``native_moe_ext`` hot-path exports.

Same names and argument meaning as native/ext/bindings.cpp (nanobind module
``native_moe_ext``), over torch CUDA tensors instead of MLX arrays:

- ``fused_moe_slots`` (bindings.cpp:300-320; fused_moe.cpp:635-664)
- ``fused_moe_staged`` (bindings.cpp:31-50; fused_moe.cpp:605-633)
- ``fused_moe`` (bindings.cpp:15-30): only the reference's ``synthetic=True``
  bridge-test stub exists there; the real-mode path throws in the reference
  (fused_moe.cpp:577-580) and raises here as well
- ``demand_gpu_remap_only`` (bindings.cpp:230-232; demand.cpp:1954-1970) with
  the per-layer slot table state of ``real_init`` (bindings.cpp:195)
- ``pool_owned_zeros`` / ``pool_write_rows`` / ``pool_write_stacked``
  (bindings.cpp:190-192)

Errors raise ``RuntimeError`` (``VbError``) like the reference's
``std::runtime_error``; nothing falls back to another implementation.
"""
from __future__ import annotations

import torch

from ._lib import VbError, check, lib
from .pool import ptr, stream_handle
from ._lib import VbQuantPool

_NUM_EXPERTS = 512  # demand.cpp:296 (slot table size)


def _pool_struct(arrays) -> VbQuantPool:
    s = VbQuantPool()
    cap = int(arrays[0].shape[0])
    for i, t in enumerate(arrays):
        if not t.is_cuda or not t.is_contiguous():
            raise VbError("pool arrays must be contiguous CUDA tensors")
        if int(t.shape[0]) != cap:
            raise VbError("pool arrays disagree on the slot count")
        s.ptr[i] = t.data_ptr()
        s.slot_stride[i] = t[0].numel() * t.element_size()
    s.cap = cap
    return s


def _fused(x, local_slots, scores, arrays, hidden, inter, group, bits, stream):
    x = x.to(torch.float32).contiguous()
    scores = scores.to(torch.float32).contiguous()
    tokens = x.numel() // hidden
    active = scores.numel()
    if tokens <= 0 or active <= 0 or active % tokens:
        raise VbError("fused_moe: shape mismatch")
    if local_slots is not None and local_slots.numel() != active:
        raise VbError("SlotFusedMoePrimitive shape mismatch")
    k = active // tokens
    pool = _pool_struct(arrays)
    out = torch.empty(x.shape[:-1] + (hidden,), dtype=torch.float32, device=x.device)
    ws = torch.empty(lib.vb_fused_moe_workspace_size(active, inter), dtype=torch.uint8,
                     device=x.device)
    ls = None if local_slots is None else local_slots.to(torch.int32).contiguous()
    check(lib.vb_fused_moe_slots(x.data_ptr(), ptr(ls), scores.data_ptr(), pool, tokens, k,
                                 hidden, inter, group, bits, out.data_ptr(), None,
                                 ws.data_ptr(), ws.numel(), stream_handle(stream)),
          "vb_fused_moe_slots")
    return out


def fused_moe_slots(x, local_slots, scores, gate_w, gate_s, gate_b, up_w, up_s, up_b,
                    down_w, down_s, down_b, hidden, inter, group, bits, *, stream=None):
    """float32 ``[..., hidden]``: pair ``p`` uses token ``p // k`` and pool slot
    ``local_slots[p]``; ``out[t] = sum_j y[t*k+j] * scores[t*k+j]``."""
    return _fused(x, local_slots, scores,
                  (gate_w, gate_s, gate_b, up_w, up_s, up_b, down_w, down_s, down_b),
                  hidden, inter, group, bits, stream)


def fused_moe_staged(x, scores, gate_w, gate_s, gate_b, up_w, up_s, up_b, down_w, down_s,
                     down_b, hidden, inter, group, bits, *, stream=None):
    """As :func:`fused_moe_slots` with pair ``p`` using staged expert ``p``."""
    return _fused(x, None, scores,
                  (gate_w, gate_s, gate_b, up_w, up_s, up_b, down_w, down_s, down_b),
                  hidden, inter, group, bits, stream)


def fused_moe(x, expert_ids, scores, compute_dir, layer, hidden, inter, group, bits,
              num_experts, synthetic, *, stream=None):
    """The reference's real mode throws (fused_moe.cpp:577-580); its
    ``synthetic`` mode is a bridge-test stub that is not part of the hot path."""
    raise VbError("real mmap staging in fused_moe is not supported; use fused_moe_slots "
                  "or fused_moe_staged with HBM-resident pool arrays")


# --------------------------- slot tables ------------------------------------

_TABLES: dict[int, torch.Tensor] = {}
_CAPS: dict[int, int] = {}


def real_init(layer: int, cap: int, device="cuda") -> None:
    """Create layer ``layer``'s expert->slot table (all -1) with capacity
    ``cap`` (demand.cpp:286-304); re-init with a different cap raises."""
    if layer in _CAPS:
        if _CAPS[layer] != cap:
            raise ValueError(f"real region cap changed after initialization: old={_CAPS[layer]} new={cap}")
        return
    _CAPS[layer] = cap
    _TABLES[layer] = torch.full((_NUM_EXPERTS,), -1, dtype=torch.int32, device=device)


def real_table_set(layer: int, experts, slots) -> None:
    """Host-side table writes (demand.cpp:306-310)."""
    t = _TABLES[layer]
    e = torch.as_tensor(experts, dtype=torch.long, device=t.device)
    s = torch.as_tensor(slots, dtype=torch.int32, device=t.device)
    t[e] = s


def real_slot_table(layer: int) -> torch.Tensor:
    return _TABLES[layer]


def real_reset() -> None:
    _TABLES.clear()
    _CAPS.clear()


def demand_gpu_remap_only(inds, layer, side_gen, cap, use_side=True, *, stream=None):
    """``local = table[inds]`` on the device, int32 with ``inds``'s shape.

    The speculative side region of the reference is not modelled (all experts
    are HBM resident), so the result is the real region's gather."""
    real_init(layer, cap, inds.device)
    ids = inds.to(torch.int32).contiguous()
    table = _TABLES[layer]
    local = torch.empty(ids.shape, dtype=torch.int32, device=ids.device)
    check(lib.vb_slot_remap(ids.data_ptr(), table.data_ptr(), local.data_ptr(), ids.numel(),
                            table.numel(), None, None, stream_handle(stream)),
          "vb_slot_remap")
    return local


def pool_owned_zeros(shape, dtype, device="cuda") -> torch.Tensor:
    """Stable device buffer for a pool tensor (owned_pool.h)."""
    return torch.zeros(tuple(shape), dtype=dtype, device=device)


def pool_write_rows(pool_list, srcs_flat, slots) -> None:
    """Write expert rows into pool slots: ``pool_list[i][slot] = src``."""
    n = len(pool_list)
    for j, slot in enumerate(slots):
        for i in range(n):
            pool_list[i][int(slot)].copy_(srcs_flat[j * n + i], non_blocking=True)


def pool_write_stacked(pool_list, stacked_list, slots) -> None:
    """Write stacked rows ``stacked_list[i][j]`` to ``pool_list[i][slots[j]]``."""
    idx = torch.as_tensor(list(slots), dtype=torch.long, device=pool_list[0].device)
    for dst, src in zip(pool_list, stacked_list):
        dst.index_copy_(0, idx, src.to(dst.device))
