"""CPU restatement of the Vates fused quantized MoE hot path (test infrastructure).

Covers router -> top-k -> slot gather -> gate/up -> SwiGLU -> down -> weighted
combine -> sigmoid-gated shared expert, the native extension's float32
``fused_moe_slots`` semantics, the deterministic route reduce and the
expert-major prefill grouping. Each function cites the reference lines it
restates (paths relative to the AMOS144/Vates project root).

Expert pools use the reference's nine-array layout (native_moe.py:57-72,
fused_moe.cpp:635-664): ``gate_w/up_w [cap, I, H*b/32] uint32``,
``down_w [cap, H, I*b/32] uint32`` and ``*_s``/``*_b`` as ``uint16`` bf16 bits
``[cap, out, in/g]``.
"""
from __future__ import annotations

import numpy as np

from . import mlx_ops as M

PROJ_KEYS = ("gate_w", "gate_s", "gate_b", "up_w", "up_s", "up_b",
             "down_w", "down_s", "down_b")


def dequant_expert(pool: dict, slot: int, hidden: int, inter: int,
                   group: int, bits: int, to_bf16: bool = False):
    """Dequantize one pool slot's three projections to float32 matrices."""
    f = M.dequantize_bf16 if to_bf16 else M.dequantize
    wg = f(pool["gate_w"][slot], pool["gate_s"][slot], pool["gate_b"][slot],
           hidden, group, bits)
    wu = f(pool["up_w"][slot], pool["up_s"][slot], pool["up_b"][slot],
           hidden, group, bits)
    wd = f(pool["down_w"][slot], pool["down_s"][slot], pool["down_b"][slot],
           inter, group, bits)
    return wg, wu, wd


# ----------------------------------------------------------------------------
# Router (block.py:253, 321-329)
# ----------------------------------------------------------------------------


def router(x, wr, k: int, norm_topk: bool = True, logit_bias=None):
    """Router GEMV + precise softmax + top-k + renormalisation.

    - ``raw_gates = self.gate(x)`` (block.py:253): bf16 Linear, float32
      accumulation, bf16 output (``logit_bias`` is the optional Linear bias,
      added in float32 before that rounding);
    - ``softmax(precise=True)`` -> bf16 (block.py:321);
    - ``argpartition`` top-k (block.py:323); ties broken by lower expert id;
    - ``take_along_axis`` then ``scores / sum(scores)`` (block.py:324-329),
      each op rounded to bf16.

    Returns ``(logits, probs, inds int32 [T,k], scores)`` (bf16 values as f32).
    """
    acc = M.matvec_f32(wr, x)
    if logit_bias is not None:
        acc = (acc + np.asarray(logit_bias, np.float32)).astype(np.float32)
    logits = M.bf16(acc)
    probs, inds, scores = route_from_logits(logits, k, norm_topk)
    return logits, probs, inds, scores


def route_from_logits(logits, k: int, norm_topk: bool = True):
    """The router after the gate Linear (block.py:321-329): bf16 logits ->
    (probs, inds, scores)."""
    probs = M.bf16(M.softmax_precise(np.asarray(logits, np.float32)))
    inds = M.topk_desc(probs, k)
    scores = np.take_along_axis(probs, inds, axis=-1)
    if norm_topk:
        denom = M.bf16(scores.astype(np.float64).sum(-1, keepdims=True).astype(np.float32))
        scores = M.bf16(scores / denom)
    return probs, inds, scores


def slot_remap(ids, table):
    """``local = table[ids]`` (-1 = not resident): resident_pool.py:560-569,
    demand.cpp:1201-1232 without leases (the table is read-only per step)."""
    ids = np.asarray(ids, np.int64)
    return np.asarray(table, np.int32)[ids]


# ----------------------------------------------------------------------------
# Decode block (MLX dtype chain; block.py:245-1013, compute.py:145-199)
# ----------------------------------------------------------------------------


def expert_mlp_decode(x_rows, wg, wu, wd):
    """``down(silu(gate(x)) * up(x))`` with MLX's decode (qmv) chain.

    gate/up/down are ``gather_qmm`` calls (compute.py:170) that accumulate in
    float32 over float32-dequantized weights and emit bf16; SwiGLU keeps bf16
    per op (:func:`mlx_ops.swiglu_bf16`).
    """
    g = M.bf16(M.matvec_f32(wg, x_rows))
    u = M.bf16(M.matvec_f32(wu, x_rows))
    h = M.swiglu_bf16(g, u)
    return M.bf16(M.matvec_f32(wd, h)), g, u, h


def rmsnorm_unit(x, eps: float):
    """Unit-weight RMSNorm with float32 math: ``bf16(x / sqrt(mean(x^2)+eps))``.

    Stands in for the decoder's post-attention norm in front of the MoE block
    (mlx-lm ``nn.RMSNorm`` / ``mx.fast.rms_norm``, weight 1).
    """
    x = np.asarray(x, np.float32)
    ss = (x.astype(np.float64) ** 2).sum(-1, keepdims=True).astype(np.float32)
    ms = (ss / np.float32(x.shape[-1])).astype(np.float32)
    inv = (np.float32(1) / np.sqrt((ms + np.float32(eps)).astype(np.float32))).astype(np.float32)
    return M.bf16(x * inv)


def moe_block_decode(x, layer: dict, k: int = 10, norm_topk: bool = True,
                     route=None, norm_eps: float = 0.0, residual=None):
    """One ``FileStreamingMoeBlock.__call__`` for a short sequence (T <= 8).

    ``layer`` holds ``wr [E,H]``, ``table [E] int32``, ``pool`` (nine arrays),
    ``shared`` (nine arrays with a single slot 0), ``wsg [H]`` and the dims
    ``hidden, inter, group, bits``. ``route`` may carry ``(inds, scores)`` to
    evaluate the expert part on a given routing (teacher forcing).

    Chain (block.py:1008-1013): ``y = sum_j bf16(y_j * s_j)`` accumulated in
    float32 and rounded to bf16, then ``y + bf16(sigmoid(x.w_sg) * shared(x))``.
    """
    x = M.bf16(np.asarray(x, np.float32))
    if norm_eps > 0:
        x = rmsnorm_unit(x, norm_eps)
    H, I, G, B = layer["hidden"], layer["inter"], layer["group"], layer["bits"]
    if route is None:
        logits, probs, inds, scores = router(x, layer["wr"], k, norm_topk,
                                             layer.get("logit_bias"))
    else:
        inds, scores = route
        logits = probs = None
    local = slot_remap(inds, layer["table"])
    if (local < 0).any():
        raise KeyError("routed expert not resident in the slot table")
    T = x.shape[0]
    ys = np.zeros((T, k, H), np.float32)
    cache = {}
    for t in range(T):
        for j in range(k):
            slot = int(local[t, j])
            if slot not in cache:
                cache[slot] = dequant_expert(layer["pool"], slot, H, I, G, B)
            wg, wu, wd = cache[slot]
            ys[t, j] = expert_mlp_decode(x[t:t + 1], wg, wu, wd)[0][0]
    weighted = M.bf16(ys * scores[:, :, None])
    routed = M.bf16(weighted.astype(np.float64).sum(1).astype(np.float32))
    sh = layer["shared"]
    swg, swu, swd = dequant_expert(sh, 0, H, I, G, B)
    ysh = expert_mlp_decode(x, swg, swu, swd)[0]
    sg = M.bf16(M.matvec_f32(np.asarray(layer["wsg"], np.float32)[None, :], x))
    gate = M.bf16(M.sigmoid_f32(sg))
    shared_term = M.bf16(gate * ysh)
    out = M.bf16(routed + shared_term)
    if residual is not None:
        out = M.bf16(M.bf16(np.asarray(residual, np.float32)) + out)
    return {"out": out, "logits": logits, "probs": probs, "inds": inds,
            "scores": scores, "local": local, "routed": routed,
            "shared": shared_term}


# ----------------------------------------------------------------------------
# Native extension float32 semantics (fused_moe.cpp:160-298)
# ----------------------------------------------------------------------------


def fused_moe_pairs_f32(x, pair_slots, pool, hidden, inter, group, bits,
                        k: int, active_mask=None):
    """Per-pair fused expert output in float32 (``fused_moe_slots_pairs``,
    fused_moe.cpp:221-283; ``_custom_fused_moe_indexed`` custom_kernel.py:239-339
    with ``k=1`` and ``x`` already one row per pair).

    Pair ``p`` uses token ``p // k`` and pool slot ``pair_slots[p]``; rows of an
    inactive pair are zero (custom_kernel.py:243-248).
    """
    x = np.asarray(x, np.float32)
    P = len(pair_slots)
    y = np.zeros((P, hidden), np.float32)
    cache = {}
    for p in range(P):
        if active_mask is not None and not active_mask[p]:
            continue
        slot = int(pair_slots[p])
        if slot not in cache:
            cache[slot] = dequant_expert(pool, slot, hidden, inter, group, bits)
        wg, wu, wd = cache[slot]
        xt = x[p // k][None, :]
        g = M.matvec_f32(wg, xt)
        u = M.matvec_f32(wu, xt)
        act = M.swiglu_f32(g, u)
        y[p] = M.matvec_f32(wd, act)[0]
    return y


def reduce_pairs_f32(pair_y, scores, k: int):
    """``out[t,c] = sum_j pair_y[t*k+j, c] * scores[t*k+j]`` (fused_moe.cpp:284-298)."""
    P, H = pair_y.shape
    s = np.asarray(scores, np.float64).reshape(P // k, k, 1)
    return (pair_y.astype(np.float64).reshape(P // k, k, H) * s).sum(1).astype(np.float32)


# ----------------------------------------------------------------------------
# Deterministic route reduce + expert-major prefill (custom_kernel.py:20-118,
# block.py:111-243)
# ----------------------------------------------------------------------------


def route_reduce(previous, weighted, assignment_pos, k: int, out_bf16: bool):
    """``deterministic_route_reduce`` (custom_kernel.py:20-118).

    Rows of ``weighted`` are sorted by their flat route position; for every
    destination token, starting from ``previous[token]``, the rows are added in
    ascending route rank with a rounding to the output dtype after each add
    (custom_kernel.py:63-77). Untouched tokens keep ``previous``.
    """
    out = np.array(previous, np.float32, copy=True)
    pos = np.asarray(assignment_pos, np.int64)
    if pos.size == 0:
        return out
    order = np.argsort(pos, kind="stable")
    rnd = M.bf16 if out_bf16 else (lambda v: np.asarray(v, np.float32))
    vals = rnd(np.asarray(weighted, np.float32))
    for i in order:
        t = int(pos[i]) // k
        out[t] = rnd(out[t] + vals[i])
    return out


def expert_groups(counts, layer_cap: int, max_assignments: int = 32768,
                  max_group_experts: int = 128):
    """Grouping rule of ``_expert_major_forward`` (block.py:154-172).

    Experts are visited in id order, skipping empty ones; a group closes when
    it already holds ``min(layer_cap, 128)`` experts or when adding the next
    expert would exceed ``max_assignments`` routes. Returns a list of
    ``(experts, assignment_count)``.
    """
    cap = min(int(layer_cap), int(max_group_experts))
    groups, active, count_sum = [], [], 0
    for e, c in enumerate(counts):
        c = int(c)
        if c == 0:
            continue
        if active and (len(active) >= cap or count_sum + c > max_assignments):
            groups.append((active, count_sum))
            active, count_sum = [], 0
        active.append(e)
        count_sum += c
    if active:
        groups.append((active, count_sum))
    return groups


def expert_mlp_prefill(x_rows, wg_b, wu_b, wd_b):
    """Expert MLP on the prefill (``gather_qmm`` matrix) path: bf16-rounded
    dequantized weights, float32 accumulation, bf16 outputs per op."""
    g = M.bf16(M.matvec_f32(wg_b, x_rows))
    u = M.bf16(M.matvec_f32(wu_b, x_rows))
    h = M.swiglu_bf16(g, u)
    return M.bf16(M.matvec_f32(wd_b, h))


def expert_major_forward(x, inds, scores, pool_of_expert, hidden, inter, group,
                         bits, layer_cap: int = 512, max_assignments: int = 32768,
                         abs_sum: bool = False):
    """``FileStreamingMoeBlock._expert_major_forward`` (block.py:111-243).

    ``pool_of_expert(e)`` returns ``(pool, slot)`` holding expert ``e``.
    Routed contributions are accumulated group by group with
    :func:`route_reduce` into a bf16 zero buffer; the order of additions
    follows the group sequence and, within a group, the route rank.
    With ``abs_sum`` also returns the per-element sum of |weighted route|,
    the bound on every partial sum of the reduce chain (its rounding scale).
    """
    x = M.bf16(np.asarray(x, np.float32))
    T, k = inds.shape
    route_ids = inds.reshape(-1).astype(np.int64)
    route_scores = scores.reshape(-1)
    counts = np.bincount(route_ids, minlength=512)
    order = np.argsort(route_ids, kind="stable")
    output = np.zeros((T, hidden), np.float32)
    absacc = np.zeros((T, hidden), np.float32)
    prefix = 0
    for experts, count in expert_groups(counts, layer_cap, max_assignments):
        pos = order[prefix:prefix + count]
        ys = np.zeros((count, hidden), np.float32)
        for e in experts:
            sel = np.nonzero(route_ids[pos] == e)[0]
            pool, slot = pool_of_expert(e)
            wg, wu, wd = dequant_expert(pool, slot, hidden, inter, group, bits,
                                        to_bf16=True)
            ys[sel] = expert_mlp_prefill(x[pos[sel] // k], wg, wu, wd)
        weighted = M.bf16(ys * route_scores[pos][:, None])
        output = route_reduce(output, weighted, pos, k, out_bf16=True)
        if abs_sum:
            np.add.at(absacc, pos // k, np.abs(weighted))
        prefix += count
    return (output, absacc) if abs_sum else output


def shared_prefill(x, shared, wsg, hidden, inter, group, bits):
    """``sigmoid(shared_expert_gate(x)) * shared_expert(x)`` (block.py:102-109)
    on the prefill (matrix) path."""
    x = M.bf16(np.asarray(x, np.float32))
    wg, wu, wd = dequant_expert(shared, 0, hidden, inter, group, bits, to_bf16=True)
    ysh = expert_mlp_prefill(x, wg, wu, wd)
    sg = M.bf16(M.matvec_f32(np.asarray(wsg, np.float32)[None, :], x))
    return M.bf16(M.bf16(M.sigmoid_f32(sg)) * ysh)


def expert_major_rows(x_rows, rows_inds, rows_scores, counts, pool_of_expert, hidden,
                      inter, group, bits, layer_cap: int = 512,
                      max_assignments: int = 32768, abs_sum: bool = False):
    """:func:`expert_major_forward` evaluated for a subset of the batch's tokens.

    ``counts`` is the route histogram of the WHOLE batch (after dropping
    non-resident routes), which fixes the reduce groups (block.py:154-172);
    ``x_rows``/``rows_inds``/``rows_scores`` are the selected tokens. A token's
    output depends only on its own routes and on the groups: its weighted
    rows are added to a bf16 zero row group by group, and inside a group in
    ascending flat route position, i.e. ascending route rank ``j``
    (custom_kernel.py:63-77 via block.py:206-224), rounding after every add.
    This equals the corresponding rows of :func:`expert_major_forward` over
    the whole batch at a cost proportional to the selected tokens.
    """
    x = M.bf16(np.asarray(x_rows, np.float32))
    n, k = rows_inds.shape
    group_of = np.full(len(counts), -1, np.int64)
    for gi, (experts, _) in enumerate(expert_groups(counts, layer_cap, max_assignments)):
        group_of[experts] = gi
    ys = np.zeros((n, k, hidden), np.float32)
    ids = rows_inds.astype(np.int64)
    for e in np.unique(ids):
        sel = np.nonzero(ids == e)
        pool, slot = pool_of_expert(int(e))
        wg, wu, wd = dequant_expert(pool, slot, hidden, inter, group, bits, to_bf16=True)
        ys[sel] = expert_mlp_prefill(x[sel[0]], wg, wu, wd)
    weighted = M.bf16(ys * np.asarray(rows_scores, np.float32)[:, :, None])
    out = np.zeros((n, hidden), np.float32)
    absacc = np.zeros((n, hidden), np.float32)
    for t in range(n):
        order = sorted(range(k), key=lambda j: (group_of[ids[t, j]], j))
        for j in order:
            if group_of[ids[t, j]] < 0:
                continue  # a route outside every group (not resident) adds nothing
            out[t] = M.bf16(out[t] + weighted[t, j])
            absacc[t] += np.abs(weighted[t, j])
    return (out, absacc) if abs_sum else out
