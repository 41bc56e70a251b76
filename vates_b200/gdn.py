"""Gated-DeltaNet recurrent steps on B200 (the linear-attention layers of
Qwen3-Next: 16 key heads, 32 value heads, head dim 128).

Mirrors ``gated_delta_multistate_kernel`` (mlx_streaming/core/linear_attn/
gated_delta_multistate.py:153-198: returns ``(y, final_state, states_out)``,
the state after every token for MTP checkpoints) and ``gated_delta_blocked``
(mlx_streaming/core/attention/gdn_fused.py:100-126) over torch tensors; the
recurrence runs in ``vb_gated_delta_step`` (libvates_b200).
"""
from __future__ import annotations

import torch

from ._lib import check, lib
from .pool import ptr, stream_handle


def _step(q, k, v, g, beta, state, mask=None, with_states=False, stream=None):
    B, T, Hk, Dk = (int(d) for d in k.shape)
    Hv, Dv = (int(d) for d in v.shape[-2:])
    q, k, v = (t.contiguous().to(torch.bfloat16) for t in (q, k, v))
    g = g.contiguous().to(torch.float32)
    beta = beta.contiguous().to(torch.float32)
    if state is None:
        state = torch.zeros((B, Hv, Dv, Dk), dtype=torch.float32, device=k.device)
    state = state.contiguous().to(torch.float32)
    y = torch.empty((B, T, Hv, Dv), dtype=torch.bfloat16, device=k.device)
    out_state = torch.empty_like(state)
    states = (torch.empty((B, T, Hv, Dv, Dk), dtype=torch.float32, device=k.device)
              if with_states else None)
    m = None if mask is None else mask.contiguous().to(torch.uint8)
    check(lib.vb_gated_delta_step(q.data_ptr(), k.data_ptr(), v.data_ptr(), g.data_ptr(),
                                  int(g.dim() == 4), beta.data_ptr(), state.data_ptr(),
                                  out_state.data_ptr(), ptr(states), ptr(m), y.data_ptr(),
                                  B, T, Hk, Hv, Dk, Dv, stream_handle(stream)),
          "vb_gated_delta_step")
    return y, out_state, states


def gated_delta_multistate_kernel(q, k, v, g, beta, state, mask=None, stream=None):
    """``(y [B,T,Hv,Dv], final_state [B,Hv,Dv,Dk], states_out [B,T,Hv,Dv,Dk])``."""
    return _step(q, k, v, g, beta, state, mask, with_states=True, stream=stream)


def gated_delta_blocked(q, k, v, g, beta, state=None, block_t=32, stream=None):
    """``(y, final_state)``: the recurrence over T tokens in chunks of at most
    16 steps per launch (the state stays in registers within a chunk)."""
    T = int(k.shape[1])
    ys = []
    for t0 in range(0, T, 16):
        t1 = min(T, t0 + 16)
        y, state, _ = _step(q[:, t0:t1], k[:, t0:t1], v[:, t0:t1], g[:, t0:t1],
                            beta[:, t0:t1], state, stream=stream)
        ys.append(y)
    return torch.cat(ys, dim=1), state


__all__ = ["gated_delta_multistate_kernel", "gated_delta_blocked"]
