"""The MTP drafter's routed-expert layer over a bounded resident pool.

Mirror of ``StreamingMTPMoE`` (mlx_streaming/mtp/qwen3_next_mtp.py:70-137):
router (``gate``), precise softmax, top-k, optional renormalisation, the
routed experts from a pool of ``capacity`` slots filled on demand, the
weighted sum and the sigmoid-gated shared expert. Here the whole block is the
fused decode kernel behind ``vb_moe_decode_resident`` (blob store) or the
host-loader flow of :class:`ResidentExpertPool`; token counts above the
kernel's 8 are cut into 8-token pieces (tokens are routed independently, so
the result is the same). The reference keys the MTP experts as pool layer
100; this pool has the one layer.
"""
from __future__ import annotations

import torch

from ._lib import VbError
from .moe_block import DECODE_SEQ_MAX, MoeBlock
from .pool import QuantPool
from .residency import DeviceBlobStore, ResidentExpertPool

MTP_POOL_LAYER = 100  # qwen3_next_mtp.py:130 (the pool layer id of the MTP experts)


class StreamingMTPMoE:
    def __init__(self, router_w: torch.Tensor, shared: QuantPool | None, shared_gate_w,
                 capacity: int, *, top_k: int = 10, norm_topk_prob: bool = True,
                 loader=None, blob_store: DeviceBlobStore | None = None,
                 hidden: int = 2048, intermediate: int = 512, bits: int = 4,
                 group_size: int = 64, router_bias=None, route_first: bool = True):
        E = int(router_w.shape[0])
        self.top_k, self.norm_topk_prob = top_k, norm_topk_prob
        self.hidden = hidden
        self.route_first = route_first
        self._pool = ResidentExpertPool(capacity, loader, layers=1, num_experts=E, hidden=hidden,
                                        inter=intermediate, bits=bits, group=group_size,
                                        blob_store=blob_store, device=router_w.device)
        self.block = MoeBlock(router_w, self._pool.tables[0], self._pool.layer_pool(0), shared,
                              shared_gate_w, top_k=top_k, norm_topk_prob=norm_topk_prob,
                              router_bias=router_bias)
        self.status = torch.zeros(1, dtype=torch.int32, device=router_w.device)
        self._debug = {n: self.block.new_debug(n, router_w.device)
                       for n in range(1, DECODE_SEQ_MAX + 1)}

    @property
    def pool(self) -> ResidentExpertPool:
        return self._pool

    def __call__(self, x: torch.Tensor, stream=None) -> torch.Tensor:
        """``x`` bf16 ``[..., H]`` -> the MoE output of the same shape."""
        shape = x.shape
        x2 = x.reshape(-1, self.hidden).contiguous()
        out = torch.empty_like(x2)
        for i in range(0, x2.shape[0], DECODE_SEQ_MAX):
            n = min(DECODE_SEQ_MAX, x2.shape[0] - i)
            self._pool.decode(0, self.block, x2[i:i + n], out[i:i + n], status=self.status,
                              debug=self._debug[n], stream=stream, route_first=self.route_first)
        (stream or torch.cuda.current_stream()).synchronize()
        st = int(self.status.item())
        if st:
            raise VbError(f"MTP MoE status {st:#x}")
        return out.reshape(shape)


__all__ = ["StreamingMTPMoE", "MTP_POOL_LAYER"]
