"""Mirror of mlx_streaming/core/moe/custom_kernel.py on B200.

- ``deterministic_route_reduce`` (custom_kernel.py:20-118)
- ``_custom_fused_moe_indexed`` (custom_kernel.py:226-383)
"""
from __future__ import annotations

import torch

from ._lib import VbError, check, lib
from .native_moe_ext import _pool_struct
from .pool import ptr, stream_handle


def deterministic_route_reduce(output: torch.Tensor, weighted: torch.Tensor,
                               assignment_pos: torch.Tensor, routes_per_token: int,
                               *, out: torch.Tensor | None = None, stream=None) -> torch.Tensor:
    """Add one expert group's routes to ``output`` without float atomics.

    ``assignment_pos`` holds unique flat positions in the ``[tokens, k]``
    routing table. Each token's routes are added in ascending route rank,
    rounding to ``output.dtype`` after every add. Returns a new tensor unless
    ``out`` is given (``out`` may be ``output`` itself)."""
    tokens, hidden = (int(v) for v in output.shape)
    groups = int(assignment_pos.numel())
    if output.dtype not in (torch.float32, torch.bfloat16):
        raise VbError("deterministic_route_reduce: output must be float32 or bfloat16")
    if groups == 0:
        return output if out is None else out.copy_(output)
    prev = output.contiguous()
    w = weighted.to(output.dtype).contiguous()
    pos = assignment_pos.to(torch.int32).contiguous()
    res = out if out is not None else torch.empty_like(prev)
    ws = torch.empty(lib.vb_route_reduce_workspace_size(tokens, routes_per_token),
                     dtype=torch.uint8, device=prev.device)
    dtype = 1 if output.dtype == torch.bfloat16 else 0
    check(lib.vb_route_reduce(prev.data_ptr(), w.data_ptr(), pos.data_ptr(), groups, tokens,
                              hidden, int(routes_per_token), dtype, res.data_ptr(), None,
                              ws.data_ptr(), ws.numel(), stream_handle(stream)),
          "vb_route_reduce")
    return res


def _custom_fused_moe_indexed(x, indices, gate_w, gate_s, gate_b, up_w, up_s, up_b,
                              down_w, down_s, down_b, hidden, moe_inter, group_size, bits,
                              active_mask=None, *, stream=None) -> torch.Tensor:
    """Fused expert per route pair: ``x[p]`` with expert ``indices[p]`` ->
    float32 ``[pairs, hidden]`` after down (inactive pairs give zero rows)."""
    x = x.to(torch.float32).contiguous()
    idx = indices.to(torch.int32).contiguous()
    pairs = int(idx.numel())
    if x.shape[0] != pairs:
        raise VbError("_custom_fused_moe_indexed: one x row per pair")
    mask = None
    if active_mask is not None:
        mask = active_mask.reshape(-1).to(torch.uint8).contiguous()
        if mask.numel() != pairs:
            raise ValueError("active_mask must have one value per route pair")
    pool = _pool_struct((gate_w, gate_s, gate_b, up_w, up_s, up_b, down_w, down_s, down_b))
    y = torch.empty((pairs, hidden), dtype=torch.float32, device=x.device)
    ws = torch.empty(lib.vb_fused_moe_workspace_size(pairs, moe_inter), dtype=torch.uint8,
                     device=x.device)
    check(lib.vb_fused_moe_pairs(x.data_ptr(), idx.data_ptr(), ptr(mask), pool, pairs, hidden,
                                 moe_inter, group_size, bits, y.data_ptr(), None, ws.data_ptr(),
                                 ws.numel(), stream_handle(stream)),
          "vb_fused_moe_pairs")
    return y
