"""Shared builders for the GPU parity tests (host numpy -> device tensors)."""
import numpy as np

from oracle import mlx_ops as M

KEYS = ("gate_w", "gate_s", "gate_b", "up_w", "up_s", "up_b", "down_w", "down_s", "down_b")


def random_pool_np(rng, cap, H, I, bits=4, group=64, lo=0.002, hi=0.02, gaussian=False):
    """Nine-array pool in the oracle format. ``gaussian`` quantizes N(0, 0.1)
    weights with the MLX rule (like the reference's tests) instead of drawing
    uniform codes with bias -8*scale."""
    out = {}
    for name, (o, i) in (("gate", (I, H)), ("up", (I, H)), ("down", (H, I))):
        if gaussian:
            w = M.bf16((rng.standard_normal((cap, o, i)) * 0.1).astype(np.float32))
            q, s, b = M.mlx_affine_quantize(w, group, bits)
        else:
            q = rng.integers(0, 2 ** 32, size=(cap, o, i * bits // 32), dtype=np.uint64).astype(np.uint32)
            s = M.bf16_bits(rng.uniform(lo, hi, (cap, o, i // group)).astype(np.float32))
            b = M.bf16_bits(M.bf16_from_bits(s) * np.float32(-8))
        out[name + "_w"], out[name + "_s"], out[name + "_b"] = q, s, b
    return out


def pool_to_torch(pool_np, device="cuda"):
    import torch
    out = {}
    for k in KEYS:
        a = np.ascontiguousarray(pool_np[k])
        if k.endswith("_w"):
            out[k] = torch.from_numpy(a.view(np.int32)).to(device)
        else:
            out[k] = torch.from_numpy(a.view(np.int16)).to(device).view(torch.bfloat16)
    return out


def bf16_tensor(a, device="cuda"):
    import torch
    return torch.from_numpy(np.ascontiguousarray(M.bf16(a))).to(torch.bfloat16).to(device)


def to_np(t):
    import torch
    if t.dtype == torch.bfloat16:
        return t.float().cpu().numpy()
    return t.cpu().numpy()


def routes_agree(gpu_inds, ref_probs, ref_inds, k):
    """Per token: True when the GPU's expert set equals the oracle's, or
    differs only inside a tie at the k-th probability (bf16 ties are common
    with 512 experts)."""
    ok = []
    for t in range(gpu_inds.shape[0]):
        g, r = set(gpu_inds[t].tolist()), set(ref_inds[t].tolist())
        if g == r:
            ok.append(True)
            continue
        p = ref_probs[t]
        kth = np.sort(p)[::-1][k - 1]
        ok.append(all(p[e] >= kth for e in g))
    return np.array(ok)


def logit_tolerance(x, wr, logits):
    """Per-logit bound on how far a float32 router GEMM/GEMV may land from
    the oracle's exactly-rounded bf16 logit: one bf16 ulp of the logit (a
    value next to a rounding midpoint can round either way), or the float32
    summation-order error of the dot product where the logit is small
    (bounded relative to sum |x_i w_i|)."""
    x = np.asarray(x, np.float32)
    wr = np.asarray(wr, np.float32)
    dot_abs = np.abs(x) @ np.abs(wr).T
    return np.maximum(M.bf16_ulp(np.abs(logits)), dot_abs * np.float32(2.0 ** -16))


def routes_agree_logits(gpu_inds, ref_logits, ref_inds, tol):
    """Per token: True when the GPU's expert set equals the oracle's, or
    when every expert the GPU picked outside the oracle's set lies within
    the logit tolerance of the oracle's weakest pick (its logit, rounded
    either way, can order either way against it: the selection follows the
    bf16 probabilities, a monotone function of the logits)."""
    g = np.sort(np.asarray(gpu_inds), 1)
    r = np.sort(np.asarray(ref_inds), 1)
    ok = (g == r).all(1)
    for t in np.nonzero(~ok)[0]:
        rs = set(r[t].tolist())
        weakest = min(ref_logits[t, j] - tol[t, j] for j in rs)
        ok[t] = all(ref_logits[t, e] + tol[t, e] >= weakest for e in g[t] if e not in rs)
    return ok


def oracle_route_and_host(blk, x, gpu_inds, k, norm_eps=0.0):
    """The oracle's own routing of ``x`` through ``blk``'s router weights
    (block.py:253, 321-329; rmsnorm first when ``norm_eps > 0``), and a host
    copy of the layer holding the union of the GPU's and the oracle's routed
    experts, so that the oracle can evaluate either routing.

    Returns ``(host, probs, inds, scores)``; ``host["full_table"]`` is the
    block's slot table, ``host["logits"]`` the oracle's logits and
    ``host["logit_tol"]`` their :func:`logit_tolerance`."""
    from oracle import moe as OM
    from vates_b200.synth import layer_to_host
    xb = M.bf16(np.asarray(x, np.float32))
    if norm_eps > 0:
        xb = OM.rmsnorm_unit(xb, norm_eps)
    wr = blk.router_w.float().cpu().numpy()
    lb = None if blk.router_bias is None else blk.router_bias.cpu().numpy()
    logits, probs, inds, scores = OM.router(xb, wr, k, blk.norm_topk_prob, lb)
    experts = np.union1d(np.asarray(gpu_inds).reshape(-1), inds.reshape(-1))
    host = layer_to_host(blk, experts)
    host["full_table"] = blk.slot_table.cpu().numpy()
    host["logits"] = logits
    host["logit_tol"] = logit_tolerance(xb, wr, logits)
    return host, probs, inds, scores
