"""CPU oracle pinned against the reference's own goldens and tests."""
import json
import os

import numpy as np
import pytest

from conftest import GOLDEN
from oracle import isoquant as IQ
from oracle import mlx_ops as M
from oracle import moe as OM


# ----------------------------------------------------------------- bf16 / packing

def test_bf16_round_to_nearest_even():
    vals = np.array([1.0, 1.00390625, 1.0078125, 1.01171875, -2.5, 3.0e38], np.float32)
    got = M.bf16(vals)
    # 1 + 2^-8 is a tie -> even (1.0); 1 + 3*2^-8 ties to 1 + 2^-6
    assert got[0] == 1.0 and got[1] == 1.0 and got[2] == np.float32(1.0078125)
    assert got[3] == np.float32(1.015625)
    assert got[4] == -2.5


@pytest.mark.parametrize("bits", [2, 3, 4, 5, 6, 8])
def test_pack_unpack_roundtrip(bits):
    rng = np.random.default_rng(bits)
    dim = 256
    codes = rng.integers(0, 1 << bits, size=(7, dim)).astype(np.uint8)
    words = M.pack_codes(codes, bits)
    assert words.shape == (7, dim * bits // 32)
    assert np.array_equal(M.unpack_codes(words, dim, bits), codes)


def test_pack_is_lsb_first_bitstream_with_straddling():
    # 3-bit field 10 starts at bit 30 and straddles into word 1
    # (fused_moe.cpp:137-142).
    codes = np.zeros((1, 32), np.uint8)
    codes[0, 10] = 0b101
    w = M.pack_codes(codes, 3)
    assert w[0, 0] == (1 << 30) and w[0, 1] == 1


def test_kv_packed_widths_golden():
    with open(os.path.join(GOLDEN, "kv_packed_widths.json")) as f:
        g = json.load(f)
    assert M.packed_words(g["head_dim"], g["k_bits"]) == g["k_words"] == 32
    assert M.packed_words(g["head_dim"], g["v_bits"]) == g["v_words"] == 24


@pytest.mark.parametrize("bits", [3, 4, 8])
def test_mlx_quantize_properties(bits):
    rng = np.random.default_rng(11)
    w = M.bf16(rng.standard_normal((16, 256)).astype(np.float32))
    q, s, b = M.mlx_affine_quantize(w, 64, bits)
    codes = M.unpack_codes(q, 256, bits)
    assert codes.max() <= (1 << bits) - 1
    deq = M.dequantize(q, s, b, 256, 64, bits)
    # Anchoring the grid on the larger edge (zero exact) may clip the far edge
    # by up to about one step; bf16 rounding of scale/bias adds a little more.
    step = np.abs(np.repeat(M.bf16_from_bits(s), 64, axis=-1))
    assert np.all(np.abs(deq - w) <= 1.1 * step + 1e-2 * np.abs(w) + 1e-6)
    assert np.mean(np.abs(deq - w)) <= 0.35 * np.mean(step)


def test_mlx_quantize_zero_on_grid():
    # The grid is anchored on the larger-magnitude edge (bias = edge, exact in
    # bf16) with zero on the float32 grid; after the scale is rounded to bf16
    # a zero input dequantizes to within |q0| scale-roundings of zero.
    w = np.zeros((1, 64), np.float32)
    w[0, :32] = np.linspace(-1.0, 0.5, 32, dtype=np.float32)
    w = M.bf16(w)
    q, s, b = M.mlx_affine_quantize(w, 64, 4)
    assert M.bf16_from_bits(b)[0, 0] == np.float32(-1.0)
    deq = M.dequantize(q, s, b, 64, 64, 4)
    assert np.all(np.abs(deq[0, 32:]) <= 2 ** -7)


def test_k4_error_below_v3_error():
    # test_kv_quant.py:263-277: 4-bit K error < 3-bit V error on N(0,1)
    rng = np.random.default_rng(0)
    x = M.bf16(rng.standard_normal((2, 10, 256)).astype(np.float32))
    e4 = np.abs(IQ.kv_dequantize(IQ.kv_quantize(x, 64, 4), 256, 64, 4) - x).mean()
    e3 = np.abs(IQ.kv_dequantize(IQ.kv_quantize(x, 64, 3), 256, 64, 3) - x).mean()
    assert e4 < e3


# ----------------------------------------------------------------- SO(4)

@pytest.mark.parametrize("dim,seed", [(256, 0), (256, 1), (16, 3), (256, 5), (64, 0)])
def test_so4_matches_reference_golden(dim, seed):
    blocks = np.load(os.path.join(GOLDEN, f"so4_d{dim}_seed{seed}_blocks.npy"))
    R = IQ.build_block_so4(dim, seed)
    assert np.array_equal(IQ.so4_blocks(R).view(np.uint32), blocks.view(np.uint32))


def test_so4_orthonormal_and_proper():
    # test_kv_quant.py:225-236
    R = IQ.build_block_so4(256, 0)
    assert np.abs(R @ R.T - np.eye(256)).max() < 1e-4
    R16 = IQ.build_block_so4(16, 3)
    for b in range(4):
        assert abs(np.linalg.det(R16[4 * b:4 * b + 4, 4 * b:4 * b + 4]) - 1.0) < 1e-3


def test_rotate_last_matches_dense_bf16_matmul():
    rng = np.random.default_rng(3)
    x = M.bf16(rng.standard_normal((5, 256)).astype(np.float32))
    R = IQ.build_block_so4(256, 0)
    got = IQ.rotate_last(x, R)
    dense = M.bf16((x.astype(np.float64) @ M.bf16(R).astype(np.float64)).astype(np.float32))
    assert np.abs(got - dense).max() <= np.abs(dense).max() * 2 ** -7


# ----------------------------------------------------------------- route reduce

def test_route_reduce_rank_order_golden():
    with open(os.path.join(GOLDEN, "route_reduce_rank_order.json")) as f:
        g = json.load(f)
    got = OM.route_reduce(np.array(g["previous"], np.float32), np.array(g["weighted"], np.float32),
                          np.array(g["assignment_pos"]), g["routes_per_token"], out_bf16=False)
    assert np.array_equal(got, np.array(g["expected"], np.float32))


def test_route_reduce_matches_bf16_scatter_chain():
    # test_expert_major_prefill.py:106-132, restated: scatter-add rank by rank
    tokens, routes, hidden = 17, 4, 8
    prev = M.bf16((np.arange(tokens * hidden) % 31).reshape(tokens, hidden).astype(np.float32) / 31)
    pos = (np.arange(37) * 11) % (tokens * routes)
    weighted = M.bf16((np.arange(37 * hidden) % 43).reshape(37, hidden).astype(np.float32) / 43)
    ref = prev.copy()
    for rank in range(routes):
        for i, p in enumerate(pos):
            if p % routes == rank:
                ref[p // routes] = M.bf16(ref[p // routes] + weighted[i])
    got = OM.route_reduce(prev, weighted, pos, routes, out_bf16=True)
    assert np.array_equal(got.view(np.uint32), ref.view(np.uint32))


def test_expert_groups_rule():
    # block.py:154-172: cap 2 experts per group -> [(0,1),(2,3)]
    counts = np.zeros(8, int)
    counts[[0, 1, 2, 3]] = [2, 2, 1, 1]
    groups = OM.expert_groups(counts, layer_cap=2)
    assert [tuple(g) for g, _ in groups] == [(0, 1), (2, 3)]
    groups = OM.expert_groups([5, 5, 5], layer_cap=512, max_assignments=10)
    assert [tuple(g) for g, _ in groups] == [(0, 1), (2,)]


# ----------------------------------------------------------------- router / MoE

def test_topk_tie_break_lower_id():
    v = np.array([[0.1, 0.3, 0.3, 0.2, 0.3]], np.float32)
    assert OM.M.topk_desc(v, 2).tolist() == [[1, 2]]


def _tiny_layer(seed=0, H=128, I=64, E=16, bits=4, group=64):
    rng = np.random.default_rng(seed)

    def proj(cap, out_d, in_d):
        w = rng.integers(0, 2 ** 32, size=(cap, out_d, in_d * bits // 32), dtype=np.uint64).astype(np.uint32)
        s = M.bf16_bits(rng.uniform(0.002, 0.02, (cap, out_d, in_d // group)).astype(np.float32))
        b = M.bf16_bits(M.bf16_from_bits(s) * -8)
        return w, s, b

    def pool(cap):
        d = {}
        for name, (o, i) in (("gate", (I, H)), ("up", (I, H)), ("down", (H, I))):
            d[name + "_w"], d[name + "_s"], d[name + "_b"] = proj(cap, o, i)
        return d

    return {"wr": M.bf16(rng.standard_normal((E, H)).astype(np.float32) * 0.02),
            "wsg": M.bf16(rng.standard_normal(H).astype(np.float32) * 0.02),
            "table": np.arange(E, dtype=np.int32), "pool": pool(E), "shared": pool(1),
            "hidden": H, "inter": I, "group": group, "bits": bits}


def test_decode_block_scores_normalised_and_combine_linear():
    layer = _tiny_layer()
    x = M.bf16(np.random.default_rng(1).standard_normal((2, 128)).astype(np.float32))
    r = OM.moe_block_decode(x, layer, k=4)
    assert r["inds"].shape == (2, 4)
    assert np.allclose(r["scores"].sum(-1), 1.0, atol=2e-2)
    # teacher forcing with the same route reproduces the output bit-exactly
    r2 = OM.moe_block_decode(x, layer, k=4, route=(r["inds"], r["scores"]))
    assert np.array_equal(r["out"], r2["out"])


def test_native_pairs_match_reduce():
    layer = _tiny_layer(bits=6, group=32, H=64, I=32, E=3)
    rng = np.random.default_rng(0)
    x = (rng.standard_normal((5, 64)) * 0.1).astype(np.float32)
    idx = np.array([0, 1, 2, 1, 0])
    y = OM.fused_moe_pairs_f32(x, idx, layer["pool"], 64, 32, 32, 6, k=1)
    assert y.shape == (5, 64) and np.isfinite(y).all()
    # one token with 5 routes and weights summing the pairs
    y5 = OM.fused_moe_pairs_f32(x[:1], idx, layer["pool"], 64, 32, 32, 6, k=5)
    out = OM.reduce_pairs_f32(y5, np.full(5, 0.2, np.float32), 5)
    assert np.allclose(out, y5.mean(0, keepdims=True), atol=1e-5)


def test_expert_major_matches_token_major_weighted_sum():
    # test_expert_major_prefill.py:33-60 restated through the oracle's
    # grouping + route reduce with the probe expert y_e(x) = x + (e + 1).
    x = np.array([[1.0, 2.0], [3.0, 4.0], [5.0, 6.0]], np.float32)
    inds = np.array([[0, 3], [1, 0], [3, 2]])
    scores = np.array([[0.25, 0.75], [0.6, 0.4], [0.1, 0.9]], np.float32)
    T, k = inds.shape
    route_ids = inds.reshape(-1)
    order = np.argsort(route_ids, kind="stable")
    counts = np.bincount(route_ids, minlength=4)
    out = np.zeros((T, 2), np.float32)
    prefix = 0
    for experts, count in OM.expert_groups(counts, layer_cap=2):
        pos = order[prefix:prefix + count]
        ys = x[pos // k] + (route_ids[pos] + 1)[:, None]
        weighted = ys * scores.reshape(-1)[pos][:, None]
        out = OM.route_reduce(out, weighted, pos, k, out_bf16=False)
        prefix += count
    expected = np.array([[sum((v + e + 1) * s for e, s in zip(r, sc)) for v in row]
                         for row, r, sc in zip(x, inds, scores)], np.float32)
    assert np.allclose(out, expected, atol=1e-6)


def test_expert_major_rows_equal_whole_batch_rows():
    """The per-token restatement (used at the 32K-token size) reproduces the
    whole-batch reduce bit for bit on the selected tokens, with several reduce
    groups per layer."""
    from helpers import random_pool_np
    rng = np.random.default_rng(4)
    T, H, I, E, k = 96, 128, 64, 12, 4
    pool = random_pool_np(rng, E, H, I, 4, 64)
    x = M.bf16(rng.standard_normal((T, H)).astype(np.float32))
    inds = np.stack([rng.choice(E, k, replace=False) for _ in range(T)]).astype(np.int32)
    scores = M.bf16(rng.uniform(0.05, 0.3, (T, k)).astype(np.float32))
    full = OM.expert_major_forward(x, inds, scores, lambda e: (pool, e), H, I, 64, 4,
                                   layer_cap=3, max_assignments=40)
    sel = np.array([0, 5, 17, 42, 95])
    counts = np.bincount(inds.reshape(-1), minlength=E)
    rows = OM.expert_major_rows(x[sel], inds[sel], scores[sel], counts, lambda e: (pool, e),
                                H, I, 64, 4, layer_cap=3, max_assignments=40)
    assert len(OM.expert_groups(counts, 3, 40)) > 3
    assert np.array_equal(rows, full[sel])


def test_gdn_oracle_states_and_chain():
    """The oracle's per-step states end in its final state, masked steps keep
    the state, and a T-step run equals T one-step runs."""
    from oracle import gdn as OG
    rng = np.random.default_rng(3)
    B, T, Hk, Hv, D = 1, 3, 2, 4, 16
    q = M.bf16(rng.standard_normal((B, T, Hk, D)).astype(np.float32) * 0.1)
    k = M.bf16(rng.standard_normal((B, T, Hk, D)).astype(np.float32) * 0.2)
    v = M.bf16(rng.standard_normal((B, T, Hv, D)).astype(np.float32))
    g = rng.uniform(0.8, 1.0, (B, T, Hv)).astype(np.float32)
    beta = rng.uniform(0.1, 0.9, (B, T, Hv)).astype(np.float32)
    s0 = (rng.standard_normal((B, Hv, D, D)) * 0.1).astype(np.float32)
    y, fin, states = OG.gated_delta(q, k, v, g, beta, s0)
    assert np.array_equal(states[:, -1], fin)
    s = s0
    for t in range(T):
        y1, s, _ = OG.gated_delta(q[:, t:t + 1], k[:, t:t + 1], v[:, t:t + 1], g[:, t:t + 1],
                                  beta[:, t:t + 1], s)
        assert np.array_equal(y1[:, 0], y[:, t]) and np.array_equal(s, states[:, t])
    ym, finm, sm = OG.gated_delta(q, k, v, g, beta, s0, mask=np.array([[True, False, True]]))
    assert np.array_equal(sm[:, 1], sm[:, 0]) and (ym[:, 1] == 0).all()
