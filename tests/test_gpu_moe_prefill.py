"""Expert-major prefill (tcgen05 grouped GEMM) on the GPU vs the CPU oracle.

Parity bar: router logits within one bf16 ulp of the oracle's (the router
GEMM accumulates in the tensor core's fp32 order, so a logit next to a
rounding midpoint can round the other way); from the GPU's logits the
oracle's softmax/top-k gives the same expert ids (up to bf16 ties at the
k-th probability) and bit-exact scores; top-k ids agree with the oracle's
own routing up to ties; with the
GPU's routes fed to the oracle (teacher forcing) the block output is within
max-abs 2e-2 or 3 bf16 ulps of the reduce chain's scale (sum of |route|),
at most 0.5% of elements beyond one such ulp, and mean-rel 5e-3. The prefill
reduce rounds to bf16 after each of the k adds (custom_kernel.py:63-77), one
more ulp of headroom than the decode path, which sums the k routes exactly.
"""
import numpy as np
import pytest

from conftest import bf16_close
from helpers import (bf16_tensor, logit_tolerance, pool_to_torch, random_pool_np, routes_agree,
                     routes_agree_logits, to_np)
from oracle import mlx_ops as M
from oracle import moe as OM

pytestmark = pytest.mark.gpu


def _case(T, H, I, E, k, group=64, seed=0, shared=True, bias=False, layer_cap=0,
          max_assignments=0, missing=()):
    import torch
    from vates_b200.moe_block import MoeBlock
    from vates_b200.pool import QuantPool, make_table
    from vates_b200.prefill import moe_prefill

    rng = np.random.default_rng(seed)
    pool_np = random_pool_np(rng, E, H, I, 4, group)
    pool = QuantPool.from_tensors(pool_to_torch(pool_np), H, I, 4, group)
    sh_np = random_pool_np(rng, 1, H, I, 4, group) if shared else None
    sh = QuantPool.from_tensors(pool_to_torch(sh_np), H, I, 4, group) if shared else None
    wsg_np = M.bf16(rng.standard_normal(H).astype(np.float32) * 0.02)
    wr_np = M.bf16(rng.standard_normal((E, H)).astype(np.float32) * 0.02)
    perm = rng.permutation(E)
    slot_of = {int(e): int(s) for s, e in enumerate(perm)}
    for e in missing:
        slot_of.pop(int(e))
    table = make_table(E, slot_of)
    lb = (np.log(1.0 / np.arange(1, E + 1) ** 1.1)[rng.permutation(E)].astype(np.float32)
          if bias else None)
    blk = MoeBlock(bf16_tensor(wr_np), table, pool, sh, bf16_tensor(wsg_np) if shared else None,
                   top_k=k, router_bias=None if lb is None else torch.from_numpy(lb).cuda())
    x = bf16_tensor(rng.standard_normal((T, H)).astype(np.float32))
    dbg = {"inds": torch.empty((T, k), dtype=torch.int32, device="cuda"),
           "scores": torch.empty((T, k), dtype=torch.bfloat16, device="cuda"),
           "logits": torch.empty((T, E), dtype=torch.bfloat16, device="cuda")}
    status = torch.zeros(1, dtype=torch.int32, device="cuda")
    out = moe_prefill(blk, x, debug=dbg, status=status, layer_cap=layer_cap,
                      max_assignments=max_assignments)
    torch.cuda.synchronize()
    xr = to_np(x)
    g_inds, g_scores = to_np(dbg["inds"]), to_np(dbg["scores"])
    r_logits, probs, r_inds, _ = OM.router(xr, wr_np, k, True, logit_bias=lb)
    assert (routes_agree(g_inds, probs, r_inds, k) |
            routes_agree_logits(g_inds, r_logits, r_inds,
                                logit_tolerance(xr, wr_np, r_logits))).all(), \
        "top-k differs beyond bf16 ties and logit rounding"
    g_logits = to_np(dbg["logits"])
    # One bf16 ulp of the logit, or, where the bias cancels the product and
    # the logit lands near zero, the float32 summation-order error of the
    # dot product (bounded relative to sum |x_i w_i|, not to the result).
    dot_abs = np.abs(xr) @ np.abs(wr_np).T
    tol = np.maximum(M.bf16_ulp(np.abs(r_logits)), dot_abs * np.float32(2.0 ** -16))
    assert (np.abs(g_logits - r_logits) <= tol).all(), "router logits"
    f_probs, f_inds, f_scores = OM.route_from_logits(g_logits, k, True)
    assert routes_agree(g_inds, f_probs, f_inds, k).all(), "top-k on the GPU logits"
    for t in range(T):
        if set(g_inds[t].tolist()) == set(f_inds[t].tolist()):
            assert dict(zip(g_inds[t].tolist(), g_scores[t].tolist())) == \
                dict(zip(f_inds[t].tolist(), f_scores[t].tolist())), t
    # Teacher forcing on the GPU's routes; experts without a slot add nothing.
    keep = np.isin(g_inds, list(slot_of.keys()))
    # (a route with a zero score adds exact zeros, like a skipped route)
    routed, absacc = OM.expert_major_forward(
        xr, g_inds, np.where(keep, g_scores, 0).astype(np.float32),
        lambda e: (pool_np, slot_of.get(int(e), 0)), H, I, group, 4,
        layer_cap=layer_cap if layer_cap > 0 else E,
        max_assignments=max_assignments if max_assignments > 0 else 32768, abs_sum=True)
    # Rounding scale: every partial sum of the bf16 reduce chain is bounded
    # by the sum of |route| values, and a flipped intermediate rounding is
    # worth one ulp of that partial sum.
    ref, scale = routed, absacc
    if shared:
        sh_term = OM.shared_prefill(xr, sh_np, wsg_np, H, I, group, 4)
        ref = M.bf16(routed + sh_term)
        scale = np.maximum(absacc, np.abs(sh_term))
    st = int(status.item())
    return to_np(out), ref, scale, st


@pytest.mark.parametrize("T,H,I,E,k,group", [(256, 1024, 256, 16, 4, 64),
                                             (300, 2048, 512, 32, 10, 64),
                                             (130, 1024, 256, 8, 2, 128)])
def test_prefill_block(cuda, T, H, I, E, k, group):
    got, ref, scale, st = _case(T, H, I, E, k, group, seed=T + E)
    assert st == 0
    bf16_close(got, ref, scale=scale, max_ulps=3, what="prefill block output")


def test_prefill_groups_order_and_zipf_bias(cuda):
    """Small reduce groups (several per layer) and a Zipf router bias: the
    add order of every token's routes follows the groups."""
    got, ref, scale, st = _case(384, 1024, 256, 32, 8, 64, seed=7, bias=True, layer_cap=3,
                                max_assignments=200)
    assert st == 0
    bf16_close(got, ref, scale=scale, max_ulps=3, what="grouped prefill output")


def test_prefill_heavy_experts_and_partial_tiles(cuda):
    """Enough tokens that the Zipf-biased experts run several 128-row tiles
    each (pre-dequantized bf16 weights, last tile partial) next to light
    experts on the in-kernel dequantization path: covers the gathered A rows
    of every tile row position, full 32-row output chunks (TMA stores) and
    partial ones."""
    got, ref, scale, st = _case(1536, 1024, 256, 24, 6, 64, seed=11, bias=True)
    assert st == 0
    bf16_close(got, ref, scale=scale, max_ulps=3, what="prefill output (heavy experts)")


def test_prefill_without_shared_expert(cuda):
    got, ref, scale, st = _case(200, 1024, 256, 16, 4, seed=3, shared=False)
    assert st == 0
    bf16_close(got, ref, scale=scale, max_ulps=3, what="prefill output (no shared expert)")


def test_prefill_missing_expert_flags_status(cuda):
    got, ref, scale, st = _case(128, 1024, 256, 16, 4, seed=5, missing=(0, 1, 2, 3, 4, 5, 6, 7))
    assert st & 1  # VB_STATUS_MISS
    bf16_close(got, ref, scale=scale, max_ulps=3, what="prefill output with skipped routes")


def test_prefill_config2_full_size(cuda):
    """The benchmark's prefill layer itself: 32,768 tokens, 512 experts,
    top-10 with the Zipf(1.1) router bias (49 experts above 384 rows, 48 of
    them pre-dequantized, 10+ reduce groups). Every token's routes against
    the oracle's own routing (up to bf16 ties) and its scores bit for bit
    from the GPU's logits; the block output of a seeded sample of 512 tokens
    (the tokens with the most light-expert routes among them) against the
    oracle's grouped, canonical-order reduce over the whole batch's groups."""
    import torch
    from vates_b200.prefill import moe_prefill
    from vates_b200.synth import config2, layer_to_host
    blk, x = config2(seed=2)
    T, k, E, H, I = 32768, 10, 512, 2048, 512
    dbg = {"inds": torch.empty((T, k), dtype=torch.int32, device="cuda"),
           "scores": torch.empty((T, k), dtype=torch.bfloat16, device="cuda"),
           "logits": torch.empty((T, E), dtype=torch.bfloat16, device="cuda")}
    status = torch.zeros(1, dtype=torch.int32, device="cuda")
    out = moe_prefill(blk, x, debug=dbg, status=status)
    torch.cuda.synchronize()
    assert int(status.item()) == 0
    xr = to_np(x)
    wr = blk.router_w.float().cpu().numpy()
    lb = blk.router_bias.cpu().numpy()
    g_inds, g_scores, g_logits = to_np(dbg["inds"]), to_np(dbg["scores"]), to_np(dbg["logits"])
    r_logits, probs, r_inds, _ = OM.router(xr, wr, k, True, logit_bias=lb)
    tol = logit_tolerance(xr, wr, r_logits)
    assert (np.abs(g_logits - r_logits) <= tol).all(), "router logits"
    # Against the oracle's own routing: the sets agree, or differ only among
    # experts whose logits sit within the rounding tolerance of the k-th.
    agree = routes_agree_logits(g_inds, r_logits, r_inds, tol)
    assert agree.all(), f"{int((~agree).sum())} tokens: top-k beyond logit rounding"
    print(f"tokens whose set differs from the oracle's by logit rounding: "
          f"{int((np.sort(g_inds, 1) != np.sort(r_inds, 1)).any(1).sum())} of {T}")
    del tol
    f_probs, f_inds, f_scores = OM.route_from_logits(g_logits, k, True)
    assert routes_agree(g_inds, f_probs, f_inds, k).all(), "top-k on the GPU logits"
    gi, fi = np.sort(g_inds, 1), np.sort(f_inds, 1)
    same = (gi == fi).all(1)
    assert same.mean() > 0.99
    go = np.argsort(g_inds, 1)
    fo = np.argsort(f_inds, 1)
    gs = np.take_along_axis(g_scores, go, 1)[same]
    fs = np.take_along_axis(f_scores, fo, 1)[same]
    # The softmax exponentials of the GPU (CUDA expf) and of the oracle
    # (numpy's float32 exp) may differ by an ulp, which moves a bf16
    # probability next to a rounding midpoint by one bf16 ulp (and with it
    # the renormalised scores of that token): scores agree bit for bit for
    # nearly every token and within one bf16 step everywhere.
    from conftest import bf16_steps
    steps = bf16_steps(gs, fs)
    assert steps.max() <= 1, "route scores beyond one bf16 step"
    exact = (steps == 0).all(1).mean()
    print(f"tokens with bit-identical scores: {exact:.5f}")
    assert exact >= 0.999, f"route scores bit-identical for only {exact:.4%} of tokens"
    counts = np.bincount(g_inds.reshape(-1), minlength=E)
    assert (counts >= 384).sum() >= 48 and len(OM.expert_groups(counts, E)) >= 10
    heavy = counts >= 384
    rng = np.random.default_rng(2024)
    light_routes = (~heavy[g_inds]).sum(1)
    sample = np.unique(np.concatenate([rng.choice(T, 448, replace=False),
                                       np.argsort(-light_routes, kind="stable")[:64]]))
    host = layer_to_host(blk, np.unique(g_inds[sample]))
    routed, absacc = OM.expert_major_rows(
        xr[sample], g_inds[sample], g_scores[sample], counts,
        lambda e: (host["pool"], int(host["table"][e])), H, I, 64, 4, layer_cap=E, abs_sum=True)
    sh_term = OM.shared_prefill(xr[sample], host["shared"], host["wsg"], H, I, 64, 4)
    ref = M.bf16(routed + sh_term)
    scale = np.maximum(absacc, np.abs(sh_term))
    got = to_np(out)
    bf16_close(got[sample], ref, scale=scale, max_ulps=3, what="config-2 prefill sample")
    assert np.isfinite(got).all()
