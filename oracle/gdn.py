"""CPU restatement of the Gated-DeltaNet recurrence (test infrastructure).

Follows the reference's gated-delta kernels: mlx_streaming/core/
linear_attn/gated_delta_multistate.py:28-130 (per-step states) and
mlx_streaming/core/attention/gdn_fused.py:13-97 (blocked scan). Per value
head hv (key head hv // (Hv // Hk)) and step t, in float32:
``S *= g``; ``kv = S @ k``; ``delta = (v - kv) * beta``; ``S += outer(delta,
k)``; ``y = bf16(S @ q)``. The dot products are float64 sums rounded once to
float32 (a stand-in for the kernels' float32 reductions, whose order the
reference leaves to the SIMD hardware).
"""
from __future__ import annotations

import numpy as np

from . import mlx_ops as M


def gated_delta(q, k, v, g, beta, state, mask=None):
    """``q, k [B,T,Hk,Dk]``, ``v [B,T,Hv,Dv]`` (bf16 values), ``g [B,T,Hv]`` or
    ``[B,T,Hv,Dk]`` and ``beta [B,T,Hv]`` float32, ``state [B,Hv,Dv,Dk]``
    float32, ``mask [B,T]`` bool or None. Returns ``(y [B,T,Hv,Dv] bf16
    values, final_state, states [B,T,Hv,Dv,Dk])``."""
    q = np.asarray(q, np.float32)
    k = np.asarray(k, np.float32)
    v = np.asarray(v, np.float32)
    g = np.asarray(g, np.float32)
    beta = np.asarray(beta, np.float32)
    S = np.array(state, np.float32, copy=True)
    B, T, Hk, Dk = k.shape
    Hv, Dv = v.shape[2:]
    rep = Hv // Hk
    y = np.zeros((B, T, Hv, Dv), np.float32)
    states = np.zeros((B, T, Hv, Dv, Dk), np.float32)
    for b in range(B):
        for t in range(T):
            if mask is not None and not mask[b, t]:
                states[b, t] = S[b]
                continue
            for hv in range(Hv):
                hk = hv // rep
                gv = g[b, t, hv] if g.ndim == 3 else g[b, t, hv][None, :]
                Sh = (S[b, hv] * gv).astype(np.float32)
                kv = (Sh.astype(np.float64) @ k[b, t, hk].astype(np.float64)).astype(np.float32)
                delta = ((v[b, t, hv] - kv) * beta[b, t, hv]).astype(np.float32)
                Sh = (Sh + (delta[:, None] * k[b, t, hk][None, :]).astype(np.float32)).astype(np.float32)
                out = (Sh.astype(np.float64) @ q[b, t, hk].astype(np.float64)).astype(np.float32)
                y[b, t, hv] = M.bf16(out)
                S[b, hv] = Sh
            states[b, t] = S[b]
    return y, S, states
