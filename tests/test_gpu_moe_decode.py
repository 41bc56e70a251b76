"""Decode / MTP-verify fused MoE block on the GPU vs the CPU oracle.

Parity bar: top-k expert ids and slot gathers exact
(up to bf16 ties at the k-th probability), route scores bit-exact, block
output within max-abs 2e-2 (or one bf16 ulp of the reference value) and
mean-rel 5e-3 in bf16.
"""
import numpy as np
import pytest

from conftest import bf16_close, bf16_steps, block_scale
from helpers import (bf16_tensor, oracle_route_and_host, pool_to_torch, random_pool_np,
                     routes_agree, routes_agree_logits, to_np)
from oracle import mlx_ops as M
from oracle import moe as OM

pytestmark = pytest.mark.gpu


def _check_block(blk, x, norm_eps=0.0, residual=None, k=10):
    """GPU block vs the oracle: the oracle routes from the router weights
    alone (its top-k never depends on the GPU's), the route sets must agree up
    to bf16 ties at the k-th probability and the scores of equal sets bit for
    bit; the block output is checked on the oracle's own routing and, teacher
    forced, on the GPU's routing."""
    import torch
    T = x.shape[0]
    status = torch.zeros(1, dtype=torch.int32, device="cuda")
    dbg = blk.new_debug(T)
    out = blk.decode(x, debug=dbg, status=status, norm_eps=norm_eps, residual=residual)
    torch.cuda.synchronize()
    assert int(status.item()) == 0
    g_inds, g_scores, g_local = to_np(dbg["inds"]), to_np(dbg["scores"]), to_np(dbg["local"])
    xr = to_np(x)
    res = None if residual is None else to_np(residual)
    host, r_probs, r_inds, r_scores = oracle_route_and_host(blk, xr, g_inds, k, norm_eps)
    assert (routes_agree(g_inds, r_probs, r_inds, k) |
            routes_agree_logits(g_inds, host["logits"], r_inds, host["logit_tol"])).all(), \
        "top-k differs beyond bf16 ties and logit rounding"
    same = np.array([set(a) == set(b) for a, b in zip(g_inds.tolist(), r_inds.tolist())])
    # Scores per expert id: bit-identical, except that a CUDA expf / numpy exp
    # ulp difference next to a bf16 rounding midpoint may move one by a bf16
    # step (and the renormalised scores of that token with it).
    for t in np.nonzero(same)[0]:
        gs = dict(zip(g_inds[t].tolist(), g_scores[t].tolist()))
        rs = dict(zip(r_inds[t].tolist(), r_scores[t].tolist()))
        ids = sorted(gs)
        assert bf16_steps([gs[e] for e in ids], [rs[e] for e in ids]).max() <= 1, \
            f"token {t}: route scores differ"
    ref = OM.moe_block_decode(xr, host, k=k, norm_eps=norm_eps, residual=res)
    assert np.array_equal(ref["inds"], r_inds)
    if same.all():
        bf16_close(to_np(out), ref["out"], scale=block_scale(ref, res), what="block output")
    # Teacher forcing on the GPU's routing isolates the expert path.
    assert np.array_equal(g_local, host["full_table"][g_inds])
    ref_tf = OM.moe_block_decode(xr, host, k=k, norm_eps=norm_eps, residual=res,
                                 route=(g_inds, g_scores))
    return bf16_close(to_np(out), ref_tf["out"], scale=block_scale(ref_tf, res),
                      what="teacher-forced block output")


@pytest.mark.parametrize("T", [1, 4])
def test_decode_block_full_size(cuda, T):
    """Config 0/1 block shape: H=2048, I=512, E=512, k=10, 4-bit g64."""
    from vates_b200.synth import config0, input_tokens
    blk, x = config0(seed=0)
    if T != 1:
        x = input_tokens(5, T)
    _check_block(blk, x)


@pytest.mark.parametrize("T,group,norm", [(3, 64, False), (8, 128, True), (2, 64, False),
                                           (5, 64, True)])
def test_decode_block_small_shapes(cuda, T, group, norm):
    import torch
    from vates_b200.moe_block import MoeBlock
    from vates_b200.pool import QuantPool, make_table
    H, I, E, k = (1024 if group == 128 else 512), 128, 64, 6
    rng = np.random.default_rng(T * 10 + group)
    pool_np = random_pool_np(rng, E, H, I, 4, group)
    pool = QuantPool.from_tensors(pool_to_torch(pool_np), H, I, 4, group)
    sh = QuantPool.from_tensors(pool_to_torch(random_pool_np(rng, 1, H, I, 4, group)), H, I, 4, group)
    wsg = bf16_tensor(rng.standard_normal(H).astype(np.float32) * 0.02)
    perm = rng.permutation(E)
    table = make_table(E, {int(e): int(s) for s, e in enumerate(perm)})
    # pool slot s holds expert perm[s]: reorder rows so the table is consistent
    wr = bf16_tensor(rng.standard_normal((E, H)).astype(np.float32) * 0.05)
    blk = MoeBlock(wr, table, pool, sh, wsg, top_k=k)
    x = bf16_tensor(rng.standard_normal((T, H)).astype(np.float32) * (3.0 if norm else 1.0))
    residual = bf16_tensor(rng.standard_normal((T, H)).astype(np.float32)) if norm else None
    _check_block(blk, x, norm_eps=1e-6 if norm else 0.0, residual=residual, k=k)


def test_decode_block_without_shared_expert(cuda):
    import torch
    from vates_b200.moe_block import MoeBlock
    from vates_b200.pool import QuantPool, make_table
    H, I, E, k, T = 512, 256, 32, 4, 3
    rng = np.random.default_rng(7)
    pool_np = random_pool_np(rng, E, H, I)
    pool = QuantPool.from_tensors(pool_to_torch(pool_np), H, I, 4, 64)
    table = make_table(E, {e: e for e in range(E)})
    wr = bf16_tensor(rng.standard_normal((E, H)).astype(np.float32) * 0.05)
    blk = MoeBlock(wr, table, pool, None, None, top_k=k)
    x = bf16_tensor(rng.standard_normal((T, H)).astype(np.float32))
    dbg = blk.new_debug(T)
    out = blk.decode(x, debug=dbg)
    g_inds, g_scores = to_np(dbg["inds"]), to_np(dbg["scores"])
    # oracle: routed part only
    layer = {"wr": to_np(wr), "table": np.arange(E, dtype=np.int32), "pool": pool_np,
             "hidden": H, "inter": I, "group": 64, "bits": 4}
    xr = to_np(x)
    ys = np.zeros((T, k, H), np.float32)
    for t in range(T):
        for j in range(k):
            wg, wu, wd = OM.dequant_expert(pool_np, int(g_inds[t, j]), H, I, 64, 4)
            ys[t, j] = OM.expert_mlp_decode(xr[t:t + 1], wg, wu, wd)[0][0]
    routed = M.bf16(M.bf16(ys * g_scores[:, :, None]).astype(np.float64).sum(1).astype(np.float32))
    bf16_close(to_np(out), routed, what="routed-only output")
    _, _, r_inds, r_scores = OM.router(M.bf16(xr), layer["wr"], k)
    assert [set(a) for a in r_inds.tolist()] == [set(a) for a in g_inds.tolist()]


def test_decode_miss_sets_status(cuda):
    import torch
    from vates_b200.synth import config0
    blk, x = config0(seed=0)
    dbg = blk.new_debug(1)
    blk.decode(x, debug=dbg)
    routed = to_np(dbg["inds"])[0]
    table = blk.slot_table.clone()
    blk.slot_table[int(routed[0])] = -1
    status = torch.zeros(1, dtype=torch.int32, device="cuda")
    dbg2 = blk.new_debug(1)
    blk.decode(x, debug=dbg2, status=status)
    torch.cuda.synchronize()
    assert int(status.item()) & 1  # VB_STATUS_MISS
    assert to_np(dbg2["local"])[0][list(routed).index(routed[0])] == -1
    blk.slot_table.copy_(table)


def test_decode_is_deterministic(cuda):
    import torch
    from vates_b200.synth import config0, input_tokens
    blk, _ = config0(seed=0)
    x = input_tokens(3, 4)
    a = blk.decode(x).clone()
    b = blk.decode(x).clone()
    assert torch.equal(a.view(torch.int16), b.view(torch.int16))


def test_stack_layers_match_oracle(cuda):
    """Config 1 structure at 3 layers: per-layer slot tables into one packed
    pool, h <- h + MoE(rmsnorm(h)), checked layer by layer."""
    from vates_b200.synth import DecodeStack
    st = DecodeStack(seed=1, layers=3, cap=64, T=4)
    st.ensure_resident()
    st.step()
    import torch
    torch.cuda.synchronize()
    for l, blk in enumerate(st.blocks):
        dbg = blk.new_debug(4)
        blk.decode(st.hs[l], debug=dbg, residual=st.hs[l], norm_eps=st.norm_eps)
        inds = to_np(dbg["inds"])
        host, probs, r_inds, _ = oracle_route_and_host(blk, to_np(st.hs[l]), inds, 10,
                                                       st.norm_eps)
        assert (routes_agree(inds, probs, r_inds, 10) |
                routes_agree_logits(inds, host["logits"], r_inds, host["logit_tol"])).all(), \
            f"layer {l}: top-k"
        ref = OM.moe_block_decode(to_np(st.hs[l]), host, k=10, norm_eps=st.norm_eps,
                                  residual=to_np(st.hs[l]),
                                  route=(inds, to_np(dbg["scores"])))
        bf16_close(to_np(st.hs[l + 1]), ref["out"], scale=block_scale(ref, to_np(st.hs[l])),
                   what=f"layer {l}")


def test_decode_bounded_wait_runs_out(cuda):
    """A grid barrier that cannot complete: the arrival counter of the
    workspace is preset so that all but one CTA wait for one arrival too
    many. Every wait gives up after its bound (about 2 s), the call returns
    VB_STATUS_TIMEOUT in the status word, and the context stays usable: the
    next call on a cleared workspace is correct."""
    import torch
    from vates_b200.moe_block import Workspace
    from vates_b200.synth import config0, input_tokens
    blk, _ = config0(seed=0)
    x = input_tokens(21, 4)
    ref = blk.decode(x).clone()
    G = torch.cuda.get_device_properties(0).multi_processor_count
    blk.workspace = Workspace()
    ws = blk.workspace.get(1 << 21)
    ws.view(torch.int64)[0] = 5 * G + G - 1  # (n + 1) G - 1 arrivals so far
    status = torch.zeros(1, dtype=torch.int32, device="cuda")
    blk.decode(x, status=status)
    torch.cuda.synchronize()
    assert int(status.item()) & 4  # VB_STATUS_TIMEOUT
    blk.workspace = Workspace()  # zero-filled again
    status.zero_()
    again = blk.decode(x, status=status)
    torch.cuda.synchronize()
    assert int(status.item()) == 0
    assert torch.equal(again.view(torch.int16), ref.view(torch.int16))
