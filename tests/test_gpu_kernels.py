"""GPU parity of the slot gather, native-extension fused MoE (float32), route
reduce and IsoQuant kernels against the CPU oracle."""
import json
import os

import numpy as np
import pytest

from conftest import GOLDEN, bf16_close, f32_close
from helpers import bf16_tensor, pool_to_torch, random_pool_np, to_np
from oracle import isoquant as IQ
from oracle import mlx_ops as M
from oracle import moe as OM

pytestmark = pytest.mark.gpu


# ------------------------------------------------------------------ slot gather

def test_slot_remap_exact_with_misses_and_bounds(cuda):
    import torch
    from vates_b200.native_moe_ext import demand_gpu_remap_only, real_reset, real_table_set
    from vates_b200.pool import slot_remap
    rng = np.random.default_rng(0)
    table_np = np.full(512, -1, np.int32)
    experts = rng.permutation(512)[:192]
    table_np[experts] = np.arange(192)
    table = torch.from_numpy(table_np).cuda()
    ids = rng.integers(0, 512, size=(4, 10)).astype(np.int32)
    ids[0, 0] = 700  # out of range -> -1 + BOUNDS
    miss = torch.zeros(1, dtype=torch.int32, device="cuda")
    status = torch.zeros(1, dtype=torch.int32, device="cuda")
    local = slot_remap(torch.from_numpy(ids).cuda(), table, miss, status)
    ref = np.where(ids < 512, table_np[np.minimum(ids, 511)], -1)
    assert np.array_equal(to_np(local), ref)
    assert int(miss.item()) == int((ref < 0).sum())
    assert int(status.item()) & 2
    real_reset()
    real_table_set_layer = 3
    from vates_b200.native_moe_ext import real_init
    real_init(real_table_set_layer, 192)
    real_table_set(real_table_set_layer, experts.tolist(), list(range(192)))
    ids2 = torch.from_numpy(rng.integers(0, 512, size=(1, 1, 10)).astype(np.int32)).cuda()
    loc2 = demand_gpu_remap_only(ids2, real_table_set_layer, 0, 192, use_side=False)
    assert np.array_equal(to_np(loc2), table_np[to_np(ids2)])


# ------------------------------------------------------ native fused MoE (f32)

def test_custom_fused_moe_indexed_matches_three_projections(cuda):
    """test_fused_moe_runtime.py:36-67 restated: 6-bit, group 32, H=64, I=32,
    3 experts, 5 pairs, indices [0,1,2,1,0], atol 1e-3."""
    import torch
    from vates_b200.custom_kernel import _custom_fused_moe_indexed
    rng = np.random.default_rng(0)
    pool_np = random_pool_np(rng, 3, 64, 32, bits=6, group=32, gaussian=True)
    x = (rng.standard_normal((5, 64)) * 0.1).astype(np.float32)
    idx = np.array([0, 1, 2, 1, 0], np.uint32)
    pt = pool_to_torch(pool_np)
    got = _custom_fused_moe_indexed(torch.from_numpy(x).cuda(), torch.from_numpy(idx.astype(np.int32)).cuda(),
                                    *[pt[k] for k in ("gate_w", "gate_s", "gate_b", "up_w", "up_s",
                                                      "up_b", "down_w", "down_s", "down_b")],
                                    64, 32, 32, 6)
    ref = OM.fused_moe_pairs_f32(x, idx, pool_np, 64, 32, 32, 6, k=1)
    assert np.abs(to_np(got) - ref).max() <= 1e-3
    mask = torch.tensor([1, 0, 1, 1, 0], dtype=torch.uint8, device="cuda")
    got_m = _custom_fused_moe_indexed(torch.from_numpy(x).cuda(), torch.from_numpy(idx.astype(np.int32)).cuda(),
                                      *[pt[k] for k in ("gate_w", "gate_s", "gate_b", "up_w", "up_s",
                                                        "up_b", "down_w", "down_s", "down_b")],
                                      64, 32, 32, 6, active_mask=mask)
    g = to_np(got_m)
    assert np.all(g[[1, 4]] == 0)
    assert np.abs(g[[0, 2, 3]] - ref[[0, 2, 3]]).max() <= 1e-3


@pytest.mark.parametrize("bits,group,H,I", [(4, 64, 2048, 512), (3, 64, 256, 128), (8, 128, 256, 256),
                                             (2, 32, 128, 64), (5, 64, 128, 128)])
def test_fused_moe_slots_and_staged(cuda, bits, group, H, I):
    import torch
    from vates_b200.native_moe_ext import fused_moe_slots, fused_moe_staged
    rng = np.random.default_rng(bits * 7 + H)
    cap, T, k = 12, 2, 4
    pool_np = random_pool_np(rng, cap, H, I, bits, group)
    pt = pool_to_torch(pool_np)
    arrays = [pt[k_] for k_ in ("gate_w", "gate_s", "gate_b", "up_w", "up_s", "up_b",
                                "down_w", "down_s", "down_b")]
    x = rng.standard_normal((T, H)).astype(np.float32)
    slots = rng.integers(0, cap, size=T * k).astype(np.int32)
    scores = rng.uniform(0, 1, T * k).astype(np.float32)
    got = fused_moe_slots(torch.from_numpy(x).cuda(), torch.from_numpy(slots).cuda(),
                          torch.from_numpy(scores).cuda(), *arrays, H, I, group, bits)
    ref = OM.reduce_pairs_f32(OM.fused_moe_pairs_f32(x, slots, pool_np, H, I, group, bits, k=k),
                              scores, k)
    scale = max(1.0, float(np.abs(ref).max()))
    f32_close(to_np(got) / scale, ref / scale, atol=1e-4, mean_rel=1e-4, what="fused_moe_slots")
    # staged: pair p uses slot p
    P = T * k
    stg = {k_: v[:P] for k_, v in pt.items()}
    got_s = fused_moe_staged(torch.from_numpy(x).cuda(), torch.from_numpy(scores).cuda(),
                             *[stg[k_] for k_ in ("gate_w", "gate_s", "gate_b", "up_w", "up_s",
                                                  "up_b", "down_w", "down_s", "down_b")],
                             H, I, group, bits)
    ref_s = OM.reduce_pairs_f32(OM.fused_moe_pairs_f32(x, np.arange(P), pool_np, H, I, group, bits, k=k),
                                scores, k)
    f32_close(to_np(got_s) / scale, ref_s / scale, atol=1e-4, mean_rel=1e-4, what="fused_moe_staged")


# ------------------------------------------------------------------ route reduce

def test_route_reduce_golden_rank_order(cuda):
    import torch
    from vates_b200.custom_kernel import deterministic_route_reduce
    g = json.load(open(os.path.join(GOLDEN, "route_reduce_rank_order.json")))
    out = deterministic_route_reduce(torch.tensor(g["previous"], device="cuda"),
                                     torch.tensor(g["weighted"], device="cuda"),
                                     torch.tensor(g["assignment_pos"], dtype=torch.int32, device="cuda"),
                                     g["routes_per_token"])
    assert to_np(out).tolist() == g["expected"]


def test_route_reduce_bf16_chain_bits(cuda):
    import torch
    from vates_b200.custom_kernel import deterministic_route_reduce
    tokens, routes, hidden = 17, 4, 8
    prev = M.bf16((np.arange(tokens * hidden) % 31).reshape(tokens, hidden).astype(np.float32) / 31)
    pos = ((np.arange(37) * 11) % (tokens * routes)).astype(np.int32)
    w = M.bf16((np.arange(37 * hidden) % 43).reshape(37, hidden).astype(np.float32) / 43)
    ref = OM.route_reduce(prev, w, pos, routes, out_bf16=True)
    got = deterministic_route_reduce(bf16_tensor(prev), bf16_tensor(w),
                                     torch.from_numpy(pos).cuda(), routes)
    assert np.array_equal(to_np(got).view(np.uint32), ref.view(np.uint32))
    # large random case, four repeats bit-identical
    rng = np.random.default_rng(1)
    tokens, routes, hidden, G = 4096, 10, 256, 9000
    pos = rng.permutation(tokens * routes)[:G].astype(np.int32)
    w = M.bf16(rng.standard_normal((G, hidden)).astype(np.float32))
    prev = M.bf16(rng.standard_normal((tokens, hidden)).astype(np.float32))
    ref = OM.route_reduce(prev, w, pos, routes, out_bf16=True)
    outs = [to_np(deterministic_route_reduce(bf16_tensor(prev), bf16_tensor(w),
                                             torch.from_numpy(pos).cuda(), routes))
            for _ in range(4)]
    for o in outs:
        assert np.array_equal(o.view(np.uint32), ref.view(np.uint32))


# ------------------------------------------------------------------ IsoQuant

@pytest.mark.parametrize("dim,kbits,vbits", [(256, 4, 3), (128, 8, 8), (64, 4, 2), (256, 5, 6)])
def test_kv_quant_append_codes_bit_exact(cuda, dim, kbits, vbits):
    """Packed codes and bf16 scale/bias bit-exact given identical rotated
    inputs; the fused rotation is bit-exact with the oracle's rotate_last."""
    import torch
    from vates_b200.quant_kv import AsymmetricQuantizedKVCache, so4_blocks, build_block_so4
    rng = np.random.default_rng(dim + kbits)
    B, Hh, n = 1, 2, 300
    k = M.bf16(rng.standard_normal((B, Hh, n, dim)).astype(np.float32))
    v = M.bf16(rng.standard_normal((B, Hh, n, dim)).astype(np.float32))
    Rk, Rv = build_block_so4(dim, 0), build_block_so4(dim, 1)
    cache = AsymmetricQuantizedKVCache(64, kbits, vbits)
    kq, vq = cache.update_and_fetch(bf16_tensor(k), bf16_tensor(v), rk=so4_blocks(Rk),
                                    rv=so4_blocks(Rv))
    kr = IQ.rotate_last(k, Rk.numpy())
    vr = IQ.rotate_last(v, Rv.numpy())
    for got, src, bits in ((kq, kr, kbits), (vq, vr, vbits)):
        w, s, b = IQ.kv_quantize(src, 64, bits)
        assert got[0].shape[-1] == dim * bits // 32
        assert np.array_equal(to_np(got[0]).view(np.uint32), w)
        assert np.array_equal(to_np(got[1].view(torch.int16)).view(np.uint16), s)
        assert np.array_equal(to_np(got[2].view(torch.int16)).view(np.uint16), b)
    # growth across the 256-step boundary (test_kv_quant.py:81-92)
    for _ in range(5):
        kq, vq = cache.update_and_fetch(bf16_tensor(k[:, :, :1]), bf16_tensor(v[:, :, :1]))
    assert cache.offset == 305 and kq[0].shape[-2] == 305
    w1, _, _ = IQ.kv_quantize(k[:, :, :1], 64, kbits)
    assert np.array_equal(to_np(kq[0][:, :, 304:305]).view(np.uint32), w1)


def test_so4_rotate_bit_exact(cuda):
    import torch
    from vates_b200.quant_kv import build_block_so4, rotate_last
    rng = np.random.default_rng(5)
    x = M.bf16(rng.standard_normal((3, 7, 256)).astype(np.float32))
    R = build_block_so4(256, 5)
    got = rotate_last(bf16_tensor(x), R)
    ref = IQ.rotate_last(x, R.numpy())
    assert np.array_equal(to_np(got), ref)
    back = rotate_last(got, R, transpose=True)
    assert np.abs(to_np(back) - x).max() < 2e-2


@pytest.mark.parametrize("L,S,causal", [(1, 40, False), (1, 4100, False), (4, 40, True),
                                         (4, 3000, True), (2, 1000, True)])
def test_kv_attention_vs_oracle(cuda, L, S, causal):
    import torch
    from vates_b200.quant_kv import (AsymmetricQuantizedKVCache, asym_quantized_sdpa,
                                     build_block_so4, so4_blocks)
    rng = np.random.default_rng(S + L)
    nq, nkv, D = 16, 2, 256
    k = M.bf16(rng.standard_normal((1, nkv, S, D)).astype(np.float32))
    v = M.bf16(rng.standard_normal((1, nkv, S, D)).astype(np.float32))
    q = M.bf16(rng.standard_normal((1, nq, L, D)).astype(np.float32))
    Rv = build_block_so4(D, 1)
    cache = AsymmetricQuantizedKVCache(64, 4, 3)
    kq, vq = cache.update_and_fetch(bf16_tensor(k), bf16_tensor(v))
    out = asym_quantized_sdpa(bf16_tensor(q), kq, vq, D ** -0.5, "causal" if causal else None,
                              64, 4, 3, rv=so4_blocks(Rv))
    kq_np = tuple(np.ascontiguousarray(a) for a in (to_np(kq[0]).view(np.uint32),
                                                   to_np(kq[1].view(torch.int16)).view(np.uint16),
                                                   to_np(kq[2].view(torch.int16)).view(np.uint16)))
    vq_np = tuple(np.ascontiguousarray(a) for a in (to_np(vq[0]).view(np.uint32),
                                                   to_np(vq[1].view(torch.int16)).view(np.uint16),
                                                   to_np(vq[2].view(torch.int16)).view(np.uint16)))
    ref = IQ.attention_layer_decode(q, kq_np, vq_np, Rv.numpy(), D ** -0.5, causal=causal)
    bf16_close(to_np(out), ref, what="kv attention")
    # mechanism check against dense attention (test_kv_quant.py:140-157): cos > 0.9
    if not causal:
        kd = k.reshape(1, nkv, 1, S, D)
        vd = v.reshape(1, nkv, 1, S, D)
        qd = q.reshape(1, nkv, nq // nkv, L, D) * D ** -0.5
        s = np.einsum("bhrld,bhxsd->bhrls", qd, kd)
        p = np.exp(s - s.max(-1, keepdims=True))
        p /= p.sum(-1, keepdims=True)
        dense = np.einsum("bhrls,bhxsd->bhrld", p, vd).reshape(1, nq, L, D)
        # the kernel applied R_v^T to attention over unrotated V: undo it
        got_unrot = IQ.rotate_last(to_np(out), Rv.numpy())
        cos = float((got_unrot * dense).sum() / (np.linalg.norm(got_unrot) * np.linalg.norm(dense)))
        assert cos > 0.9


@pytest.mark.parametrize("L,S,causal,nq,nkv", [(40, 40, True, 16, 2), (200, 300, True, 16, 2),
                                               (33, 150, False, 16, 2), (130, 130, True, 8, 2),
                                               (64, 1000, True, 16, 2), (5, 260, True, 16, 2),
                                               (300, 700, True, 16, 1)])
def test_prefill_attention_vs_oracle(cuda, L, S, causal, nq, nkv):
    """tcgen05 prefill attention (_tiled_asymmetric_attention,
    expert_major.py:32-95) against the oracle's MLX dtype chain, with the
    inverse V rotation fused; L > 4 also goes through asym_quantized_sdpa."""
    import torch
    from vates_b200.quant_kv import (AsymmetricQuantizedKVCache, asym_quantized_sdpa,
                                     build_block_so4, so4_blocks, tiled_asymmetric_attention)
    rng = np.random.default_rng(1000 + S + L)
    D = 256
    k = M.bf16(rng.standard_normal((1, nkv, S, D)).astype(np.float32))
    v = M.bf16(rng.standard_normal((1, nkv, S, D)).astype(np.float32))
    q = M.bf16(rng.standard_normal((1, nq, L, D)).astype(np.float32))
    Rv = build_block_so4(D, 2)
    cache = AsymmetricQuantizedKVCache(64, 4, 3)
    kq, vq = cache.update_and_fetch(bf16_tensor(k), bf16_tensor(v))
    status = torch.zeros(1, dtype=torch.int32, device="cuda")
    out = tiled_asymmetric_attention(bf16_tensor(q), kq, vq, scale=D ** -0.5,
                                     mask="causal" if causal else None, group_size=64, k_bits=4,
                                     v_bits=3, rv=so4_blocks(Rv), status=status)
    torch.cuda.synchronize()
    assert int(status.item()) == 0
    kq_np = tuple(np.ascontiguousarray(a) for a in (to_np(kq[0]).view(np.uint32),
                                                   to_np(kq[1].view(torch.int16)).view(np.uint16),
                                                   to_np(kq[2].view(torch.int16)).view(np.uint16)))
    vq_np = tuple(np.ascontiguousarray(a) for a in (to_np(vq[0]).view(np.uint32),
                                                   to_np(vq[1].view(torch.int16)).view(np.uint16),
                                                   to_np(vq[2].view(torch.int16)).view(np.uint16)))
    ref = IQ.attention_layer_decode(q, kq_np, vq_np, Rv.numpy(), D ** -0.5, causal=causal)
    bf16_close(to_np(out), ref, what="prefill attention")
    again = asym_quantized_sdpa(bf16_tensor(q), kq, vq, D ** -0.5, "causal" if causal else None,
                                64, 4, 3, rv=so4_blocks(Rv))
    assert torch.equal(again.view(torch.int16), out.view(torch.int16))


# ------------------------------------------------------------------ dequantized weights

@pytest.mark.parametrize("bits,group,gaussian", [(4, 64, False), (4, 64, True), (4, 128, True),
                                                 (3, 64, True), (2, 32, True), (5, 64, True),
                                                 (6, 64, False), (8, 128, True)])
def test_dequantize_bit_exact(cuda, bits, group, gaussian):
    """Dequantized weights bit for bit (fused_moe.cpp:131-145 qvalue): the
    float32 value q*s + b and its bf16 rounding, against the oracle, for
    benchmark-format weights (uniform codes, bias -8*scale) and for weights
    quantized with the MLX rule. The 4-bit bf16 output comes from the device
    routine that feeds every prefill GEMM."""
    import ctypes as C
    import torch
    from vates_b200._lib import check, lib
    from vates_b200.pool import stream_handle
    rng = np.random.default_rng(bits * 1000 + group)
    rows, cols = 96, 512
    if gaussian:
        w = M.bf16((rng.standard_normal((rows, cols)) * 0.1).astype(np.float32))
        q, s, b = M.mlx_affine_quantize(w, group, bits)
    else:
        q = rng.integers(0, 2 ** 32, size=(rows, cols * bits // 32), dtype=np.uint64).astype(np.uint32)
        s = M.bf16_bits(rng.uniform(0.002, 0.02, (rows, cols // group)).astype(np.float32))
        b = M.bf16_bits(M.bf16_from_bits(s) * np.float32(-8))
    dq = torch.from_numpy(q.view(np.int32)).cuda()
    ds = torch.from_numpy(s.view(np.int16)).cuda()
    db = torch.from_numpy(b.view(np.int16)).cuda()
    o32 = torch.empty((rows, cols), dtype=torch.float32, device="cuda")
    o16 = torch.empty((rows, cols), dtype=torch.int16, device="cuda")
    for out, is_bf16 in ((o32, 0), (o16, 1)):
        check(lib.vb_dequantize(dq.data_ptr(), ds.data_ptr(), db.data_ptr(), rows, cols, group,
                                bits, is_bf16, out.data_ptr(), stream_handle()), "vb_dequantize")
    torch.cuda.synchronize()
    ref = M.dequantize(q, s, b, cols, group, bits)
    assert np.array_equal(o32.cpu().numpy().view(np.uint32), ref.view(np.uint32))
    ref16 = M.bf16_bits(M.dequantize_bf16(q, s, b, cols, group, bits))
    assert np.array_equal(o16.cpu().numpy().view(np.uint16), ref16)


def test_dequantize_synthetic_expert_bit_exact(cuda):
    """The benchmark pool's own expert bytes (counter-hash codes, 2048-wide
    rows) dequantized on the device equal the oracle's bf16 weights."""
    import torch
    from vates_b200._lib import check, lib
    from vates_b200.pool import QuantPool, expert_seed, stream_handle
    pool = QuantPool.empty_blob(2, 2048, 512, 4, 64)
    pool.fill_synthetic_many([0, 1], [expert_seed(0, 0, 17), expert_seed(0, 0, 401)])
    for slot in (0, 1):
        t = pool.slot_tensors(slot)
        host = pool.to_numpy_slot(slot)
        for proj, cols in (("gate", 2048), ("up", 2048), ("down", 512)):
            rows = t[f"{proj}_w"].shape[0]
            out = torch.empty((rows, cols), dtype=torch.int16, device="cuda")
            check(lib.vb_dequantize(t[f"{proj}_w"].data_ptr(), t[f"{proj}_s"].data_ptr(),
                                    t[f"{proj}_b"].data_ptr(), rows, cols, 64, 4, 1,
                                    out.data_ptr(), stream_handle()), "vb_dequantize")
            ref = M.bf16_bits(M.dequantize_bf16(host[f"{proj}_w"][0], host[f"{proj}_s"][0],
                                                host[f"{proj}_b"][0], cols, 64, 4))
            assert np.array_equal(out.cpu().numpy().view(np.uint16), ref), (slot, proj)


def test_synth_pool_one_launch_matches_per_tensor_fill(cuda):
    import torch
    from vates_b200.pool import QuantPool, expert_seed
    a = QuantPool.empty_blob(5, 2048, 512, 4, 64)
    b = QuantPool.empty_blob(5, 2048, 512, 4, 64)
    seeds = [expert_seed(3, 2, e) for e in (0, 9, 100, 511, 100_000)]
    for s, sd in enumerate(seeds):
        a.fill_synthetic(s, sd)
    b.fill_synthetic_many(range(5), seeds)
    torch.cuda.synchronize()
    assert torch.equal(a.blob, b.blob)


@pytest.mark.parametrize("L", [1, 4])
def test_kv_attention_128k_vs_oracle(cuda, L):
    """The benchmark's attention layer: 131,072 keys, 16 query / 2 kv heads,
    head_dim 256, K4/V3 after the seeded SO(4) rotations (K seed 0, V seed
    1), one query (L=1) and the four causal MTP-verify queries (L=4): packed
    codes bit-exact against the oracle's quantize of the oracle's rotation,
    output against the oracle's MLX chain with the inverse V rotation."""
    import torch
    from vates_b200.quant_kv import (AsymmetricQuantizedKVCache, asym_quantized_sdpa,
                                     build_block_so4, so4_blocks)
    S, nq, nkv, D = 131072, 16, 2, 256
    rng = np.random.default_rng(131072 + L)
    k = M.bf16(rng.standard_normal((1, nkv, S, D), dtype=np.float32))
    v = M.bf16(rng.standard_normal((1, nkv, S, D), dtype=np.float32))
    q = M.bf16(rng.standard_normal((1, nq, L, D), dtype=np.float32))
    Rk, Rv = build_block_so4(D, 0), build_block_so4(D, 1)
    cache = AsymmetricQuantizedKVCache(64, 4, 3)
    kq, vq = cache.update_and_fetch(bf16_tensor(k), bf16_tensor(v), rk=so4_blocks(Rk),
                                    rv=so4_blocks(Rv))
    qr = IQ.rotate_last(q, Rk.numpy())
    out = asym_quantized_sdpa(bf16_tensor(qr), kq, vq, D ** -0.5, "causal" if L > 1 else None,
                              64, 4, 3, rv=so4_blocks(Rv))
    torch.cuda.synchronize()
    packs = []
    for got, src, R, bits in ((kq, k, Rk, 4), (vq, v, Rv, 3)):
        w, s, b = IQ.kv_quantize(IQ.rotate_last(src, R.numpy()), 64, bits)
        gw = to_np(got[0]).view(np.uint32)
        gs = to_np(got[1].view(torch.int16)).view(np.uint16)
        gb = to_np(got[2].view(torch.int16)).view(np.uint16)
        assert np.array_equal(gw, w) and np.array_equal(gs, s) and np.array_equal(gb, b)
        packs.append((np.ascontiguousarray(gw), np.ascontiguousarray(gs), np.ascontiguousarray(gb)))
    del k, v
    ref = IQ.attention_layer_decode(qr, packs[0], packs[1], Rv.numpy(), D ** -0.5,
                                    causal=L > 1)
    bf16_close(to_np(out), ref, what=f"128K-key attention, L={L}")
