"""Expert-major prefill of a sparse-MoE block on B200 (tcgen05 grouped GEMM).

Host-side mirror of the prefill branch of ``FileStreamingMoeBlock.__call__``
(mlx_streaming/core/moe/block.py:318-347) and ``_expert_major_forward``
(block.py:111-243): the whole block (router, top-k, grouped expert GLU,
canonical-order reduce, shared expert) runs in ``vb_moe_prefill``; this
module only owns the tensors and the argument struct.
"""
from __future__ import annotations

import ctypes as C

import torch

from ._lib import VbMoePrefillArgs, check, lib
from .pool import ptr, stream_handle

PREFILL_ALIGN = 1024


class PrefillWorkspace:
    """Grow-only device scratch for ``vb_moe_prefill`` (no initialisation
    needed); hands out a 1024-byte aligned pointer."""

    def __init__(self, device="cuda"):
        self.device = device
        self.buf = None

    def get(self, nbytes: int) -> tuple[int, int]:
        if self.buf is None or self.buf.numel() < nbytes + PREFILL_ALIGN:
            self.buf = None
            self.buf = torch.empty(nbytes + PREFILL_ALIGN, dtype=torch.uint8, device=self.device)
        base = self.buf.data_ptr()
        aligned = (base + PREFILL_ALIGN - 1) // PREFILL_ALIGN * PREFILL_ALIGN
        return aligned, self.buf.numel() - (aligned - base)


_WS: dict = {}


def prefill_args(blk, x2, out, ws_ptr, ws_bytes, debug=None, status=None,
                 layer_cap: int = 0, max_assignments: int = 0) -> VbMoePrefillArgs:
    T = int(x2.shape[0])
    a = VbMoePrefillArgs()
    a.tokens, a.hidden, a.inter = T, blk.hidden, blk.inter
    a.group, a.bits = blk.pool.group, blk.pool.bits
    a.num_experts, a.top_k, a.norm_topk = blk.num_experts, blk.top_k, int(blk.norm_topk_prob)
    a.layer_cap, a.max_assignments = int(layer_cap), int(max_assignments)
    a.x, a.router_w, a.router_bias = x2.data_ptr(), blk.router_w.data_ptr(), ptr(blk.router_bias)
    a.slot_table = blk.slot_table.data_ptr()
    a.pool = blk._pool_c
    if blk._shared_c is not None:
        a.shared = blk._shared_c
        a.shared_gate_w = blk.shared_gate_w.data_ptr()
    a.out = out.data_ptr()
    if debug is not None:
        a.out_inds = debug["inds"].data_ptr()
        a.out_scores = debug["scores"].data_ptr()
        if "logits" in debug:
            a.out_logits = debug["logits"].data_ptr()
    a.status = ptr(status)
    a.workspace, a.workspace_bytes = ws_ptr, ws_bytes
    return a


def moe_prefill(blk, x: torch.Tensor, out: torch.Tensor | None = None, debug: dict | None = None,
                status=None, stream=None, layer_cap: int = 0, max_assignments: int = 0,
                workspace: PrefillWorkspace | None = None) -> torch.Tensor:
    """``FileStreamingMoeBlock.__call__`` for a prefill batch (any T).

    ``x`` bf16 ``[T, H]`` (or ``[B, S, H]``). ``layer_cap``/``max_assignments``
    set the reference's reduce groups (block.py:154-155; 0 = defaults).
    """
    shape = x.shape
    x2 = x.reshape(-1, blk.hidden).contiguous()
    assert x2.dtype == torch.bfloat16
    T = int(x2.shape[0])
    if out is None:
        out = torch.empty_like(x2)
    need = lib.vb_moe_prefill_workspace_size(T, blk.hidden, blk.inter, blk.num_experts,
                                             blk.top_k)
    if workspace is None:
        workspace = _WS.setdefault(str(x2.device), PrefillWorkspace(x2.device))
    ws_ptr, ws_bytes = workspace.get(need)
    a = prefill_args(blk, x2, out, ws_ptr, ws_bytes, debug=debug, status=status,
                     layer_cap=layer_cap, max_assignments=max_assignments)
    check(lib.vb_moe_prefill(C.byref(a), stream_handle(stream)), "vb_moe_prefill")
    return out.reshape(shape)
