"""Gated-DeltaNet recurrent steps (vb_gated_delta_step) on the GPU vs the
CPU oracle, at the Qwen3-Next GDN layer shape: 16 key heads, 32 value heads,
head dim 128 (gated_delta_multistate.py:28-198, gdn_fused.py:13-126).

Parity bar: y within max(2e-2, 2 bf16 ulps) and mean-rel 5e-3 (the float32
reductions run in a different order from the oracle's); states within
1e-5 of their magnitude. A T-token call equals T one-token calls bit for bit
(the per-step states of the multistate kernel are the states of the
one-token chain: the reference's MTP-checkpoint property).
"""
import numpy as np
import pytest

from conftest import bf16_close
from helpers import bf16_tensor, to_np
from oracle import gdn as OG
from oracle import mlx_ops as M

pytestmark = pytest.mark.gpu

B, HK, HV, D = 1, 16, 32, 128


def _inputs(rng, T, vec_g=False):
    s = D ** -0.5
    def unit(x):
        return x / np.sqrt((x * x).mean(-1, keepdims=True) + 1e-6)
    q = M.bf16(unit(rng.standard_normal((B, T, HK, D))).astype(np.float32) * s * s)
    k = M.bf16(unit(rng.standard_normal((B, T, HK, D))).astype(np.float32) * s)
    v = M.bf16(rng.standard_normal((B, T, HV, D)).astype(np.float32))
    gshape = (B, T, HV, D) if vec_g else (B, T, HV)
    g = rng.uniform(0.85, 1.0, gshape).astype(np.float32)
    beta = (1 / (1 + np.exp(-rng.standard_normal((B, T, HV))))).astype(np.float32)
    state = (rng.standard_normal((B, HV, D, D)) * 0.1).astype(np.float32)
    return q, k, v, g, beta, state


def _t(a):
    import torch
    return torch.from_numpy(np.ascontiguousarray(a)).cuda()


@pytest.mark.parametrize("T,vec_g,masked", [(1, False, False), (4, False, False),
                                            (4, True, False), (3, False, True)])
def test_gdn_step_vs_oracle(cuda, T, vec_g, masked):
    import torch
    from vates_b200.gdn import gated_delta_multistate_kernel
    rng = np.random.default_rng(T * 10 + vec_g + 2 * masked)
    q, k, v, g, beta, state = _inputs(rng, T, vec_g)
    mask = np.array([[True, False, True][:T]]) if masked else None
    y, fin, states = gated_delta_multistate_kernel(
        bf16_tensor(q), bf16_tensor(k), bf16_tensor(v), _t(g), _t(beta), _t(state),
        mask=None if mask is None else _t(mask))
    torch.cuda.synchronize()
    ry, rfin, rstates = OG.gated_delta(q, k, v, g, beta, state, mask)
    bf16_close(to_np(y), ry, what="gdn y")
    scale = np.abs(rstates).max()
    assert np.abs(to_np(states) - rstates).max() <= 1e-5 * scale
    assert np.abs(to_np(fin) - rfin).max() <= 1e-5 * scale
    assert torch.equal(fin, states[:, -1])
    if masked:
        assert (to_np(y)[0, 1] == 0).all()


def test_gdn_multistep_equals_single_steps(cuda):
    """One T=4 call and four T=1 calls chained through the state: identical
    y and states bit for bit."""
    import torch
    from vates_b200.gdn import gated_delta_multistate_kernel
    rng = np.random.default_rng(7)
    q, k, v, g, beta, state = _inputs(rng, 4)
    Q, K, V, G, Bt = bf16_tensor(q), bf16_tensor(k), bf16_tensor(v), _t(g), _t(beta)
    y4, fin4, st4 = gated_delta_multistate_kernel(Q, K, V, G, Bt, _t(state))
    s = _t(state)
    for t in range(4):
        y1, s, _ = gated_delta_multistate_kernel(Q[:, t:t + 1], K[:, t:t + 1], V[:, t:t + 1],
                                                 G[:, t:t + 1], Bt[:, t:t + 1], s)
        assert torch.equal(y1[:, 0].view(torch.int16), y4[:, t].view(torch.int16))
        assert torch.equal(s, st4[:, t])
    assert torch.equal(s, fin4)


def test_gdn_blocked_long_sequence(cuda):
    """gated_delta_blocked over 40 tokens (three launches of up to 16 steps)
    against the oracle."""
    import torch
    from vates_b200.gdn import gated_delta_blocked
    rng = np.random.default_rng(11)
    q, k, v, g, beta, state = _inputs(rng, 40)
    y, fin = gated_delta_blocked(bf16_tensor(q), bf16_tensor(k), bf16_tensor(v), _t(g),
                                 _t(beta), _t(state))
    torch.cuda.synchronize()
    ry, rfin, _ = OG.gated_delta(q, k, v, g, beta, state)
    bf16_close(to_np(y), ry, what="gdn blocked y")
    assert np.abs(to_np(fin) - rfin).max() <= 1e-5 * np.abs(rfin).max()
