"""The sparse-MoE block of Qwen3-Next on B200: decode/verify and prefill.

Host-side mirror of ``FileStreamingMoeBlock`` (mlx_streaming/core/moe/
block.py:75-1683): router, top-k, pool slot indirection, expert GLU, weighted
combine and the sigmoid-gated shared expert. All arithmetic runs in the
``libvates_b200`` kernels; this module only owns tensors and arguments.
"""
from __future__ import annotations

import ctypes as C

import torch

from ._lib import VbMoeDecodeArgs, check, lib
from .pool import QuantPool, ptr, stream_handle

DECODE_SEQ_MAX = 8  # block.py:22 (_DECODE_SEQ_MAX)


class Workspace:
    """Grow-only, zero-initialised device scratch buffer shared by the calls
    of one stream (the decode kernels keep a counter in its first word and
    leave it at zero)."""

    def __init__(self, device="cuda"):
        self.device = device
        self.buf = None

    def get(self, nbytes: int) -> torch.Tensor:
        if self.buf is None or self.buf.numel() < nbytes:
            self.buf = torch.zeros(max(nbytes, 1), dtype=torch.uint8, device=self.device)
        return self.buf


class MoeBlock:
    """One Qwen3-Next sparse-MoE block with a resident expert pool.

    ``router_w`` bf16 ``[E, H]``; ``slot_table`` int32 ``[E]``; ``pool`` the
    routed experts; ``shared``/``shared_gate_w`` the shared expert (optional);
    ``router_bias`` optional f32 ``[E]`` added to the router logits.
    """

    def __init__(self, router_w, slot_table, pool: QuantPool, shared: QuantPool | None,
                 shared_gate_w=None, top_k: int = 10, norm_topk_prob: bool = True,
                 router_bias=None, workspace: Workspace | None = None):
        self.router_w = router_w
        self.slot_table = slot_table
        self.pool = pool
        self.shared = shared
        self.shared_gate_w = shared_gate_w
        self.top_k = top_k
        self.norm_topk_prob = norm_topk_prob
        self.router_bias = router_bias
        self.hidden = pool.hidden
        self.inter = pool.inter
        self.num_experts = int(router_w.shape[0])
        self.workspace = workspace or Workspace(router_w.device)
        self._pool_c = pool.c_struct()
        self._shared_c = shared.c_struct() if shared is not None else None

    def refresh(self):
        """Re-read pool pointers after the pool or table tensors changed."""
        self._pool_c = self.pool.c_struct()
        self._shared_c = self.shared.c_struct() if self.shared is not None else None

    def decode_args(self, x, out, residual=None, debug=None, status=None,
                    norm_eps: float = 0.0, timing=None, trace=None) -> VbMoeDecodeArgs:
        T = int(x.shape[0])
        need = lib.vb_moe_decode_workspace_size(T, self.hidden, self.inter,
                                                self.num_experts, self.top_k)
        ws = self.workspace.get(need)
        a = VbMoeDecodeArgs()
        a.tokens, a.hidden, a.inter = T, self.hidden, self.inter
        a.group, a.bits = self.pool.group, self.pool.bits
        a.num_experts, a.top_k, a.norm_topk = self.num_experts, self.top_k, int(self.norm_topk_prob)
        a.norm_eps = float(norm_eps)
        a.x, a.router_w, a.router_bias = x.data_ptr(), self.router_w.data_ptr(), ptr(self.router_bias)
        a.slot_table = self.slot_table.data_ptr()
        a.pool = self._pool_c
        if self._shared_c is not None:
            a.shared = self._shared_c
            a.shared_gate_w = self.shared_gate_w.data_ptr()
        a.residual = ptr(residual)
        a.out = out.data_ptr()
        if debug is not None:
            a.out_inds = debug["inds"].data_ptr()
            a.out_scores = debug["scores"].data_ptr()
            a.out_local = debug["local"].data_ptr()
        a.status = ptr(status)
        a.workspace = ws.data_ptr()
        a.workspace_bytes = ws.numel()
        if timing is not None:
            a.timing_events = C.cast(timing, C.c_void_p)
        a.trace = ptr(trace)
        return a

    def decode(self, x: torch.Tensor, out: torch.Tensor | None = None, residual=None,
               debug: dict | None = None, status=None, stream=None,
               norm_eps: float = 0.0, timing=None, trace=None) -> torch.Tensor:
        """``FileStreamingMoeBlock.__call__`` for ``T <= 8`` tokens.

        ``x`` bf16 ``[T, H]`` (or ``[B, S, H]`` with ``B*S <= 8``).
        """
        shape = x.shape
        x2 = x.reshape(-1, self.hidden).contiguous()
        assert x2.dtype == torch.bfloat16 and x2.shape[0] <= DECODE_SEQ_MAX
        if out is None:
            out = torch.empty_like(x2)
        a = self.decode_args(x2, out, residual=residual, debug=debug, status=status,
                             norm_eps=norm_eps, timing=timing, trace=trace)
        check(lib.vb_moe_decode(C.byref(a), stream_handle(stream)), "vb_moe_decode")
        return out.reshape(shape)

    @staticmethod
    def timing_events():
        """Two CUDA events (created) and the C array of their handles for the
        ``timing`` argument of :meth:`decode` (recorded before and after the
        layer kernel)."""
        evs = [torch.cuda.Event(enable_timing=True) for _ in range(2)]
        for e in evs:
            e.record()
        arr = (C.c_void_p * 2)(*[e.cuda_event for e in evs])
        return evs, arr

    def new_debug(self, T: int, device="cuda") -> dict:
        k = self.top_k
        return {"inds": torch.empty((T, k), dtype=torch.int32, device=device),
                "scores": torch.empty((T, k), dtype=torch.bfloat16, device=device),
                "local": torch.empty((T, k), dtype=torch.int32, device=device)}

    def __call__(self, x: torch.Tensor) -> torch.Tensor:
        n = x.numel() // self.hidden
        if n <= DECODE_SEQ_MAX:
            return self.decode(x)
        return self.prefill(x)

    def prefill(self, x: torch.Tensor, **kw) -> torch.Tensor:
        from .prefill import moe_prefill
        return moe_prefill(self, x, **kw)
