"""Pool fill and residency on the GPU: blob bytes land in the right slots
(host copies and the device gather), the device slot tables follow the native
state, and a decode over a pool smaller than the expert count, with misses
loaded between kernel runs, gives bit-identical outputs to a fully resident
pool."""
import numpy as np
import pytest

from conftest import bf16_close, block_scale
from helpers import KEYS, bf16_tensor, pool_to_torch, random_pool_np, routes_agree, to_np
from oracle import moe as OM
from oracle.residency import ResidencyOracle

pytestmark = pytest.mark.gpu

H, I, G, BITS = 512, 128, 64, 4


def _blobs_np(pool_np, E):
    """expert_blob_v1 rows (prep/blob_layout.py:14-32) of every expert."""
    rows = []
    for e in range(E):
        rows.append(np.concatenate([np.ascontiguousarray(pool_np[k][e]).view(np.uint8).reshape(-1)
                                    for k in KEYS]))
    return np.stack(rows)


def _slot_bytes(pool, slot):
    import torch
    t = pool.slot_tensors(slot)
    return np.concatenate([t[k].contiguous().view(torch.uint8).cpu().numpy().reshape(-1)
                           for k in KEYS])


@pytest.mark.parametrize("source", ["pinned", "pageable", "device"])
def test_pool_fill_blob_and_stacked_pools(cuda, source):
    import torch
    from vates_b200.pool import QuantPool
    from vates_b200.residency import fill_slots
    rng = np.random.default_rng(1)
    E = 12
    pool_np = random_pool_np(rng, E, H, I, BITS, G)
    blobs = _blobs_np(pool_np, E)
    experts, slots = [5, 1, 9, 11], [3, 0, 7, 2]

    def src(e):
        t = torch.from_numpy(blobs[e].copy())
        if source == "pinned":
            return t.pin_memory()
        if source == "device":
            return t.cuda()
        return t

    blob_pool = QuantPool.empty_blob(8, H, I, BITS, G)
    blob_pool.blob.zero_()
    stacked = QuantPool.from_tensors({k: torch.zeros_like(v[:8]) for k, v in
                                      pool_to_torch(pool_np).items()}, H, I, BITS, G)
    for p in (blob_pool, stacked):
        fill_slots(p, slots, [src(e) for e in experts])
        torch.cuda.synchronize()
        for e, s in zip(experts, slots):
            assert np.array_equal(_slot_bytes(p, s), blobs[e])
        untouched = [s for s in range(8) if s not in slots]
        assert all(not _slot_bytes(p, s).any() for s in untouched)


def test_blob_gather_into_slots(cuda):
    import torch
    from vates_b200.pool import QuantPool
    from vates_b200.residency import DeviceBlobStore
    rng = np.random.default_rng(2)
    E = 10
    pool_np = random_pool_np(rng, E, H, I, BITS, G)
    blobs = _blobs_np(pool_np, E)
    store = DeviceBlobStore(torch.from_numpy(np.stack([blobs, blobs[::-1].copy()])).cuda())
    big = QuantPool.empty_blob(12, H, I, BITS, G)
    big.blob.zero_()
    view = big.view(4, 6)
    place = [(7, 0), (2, 5), (9, 3)]
    store.fill(1, view, place)      # layer 1 holds the experts in reverse order
    torch.cuda.synchronize()
    for e, s in place:
        assert np.array_equal(_slot_bytes(big, 4 + s), blobs[E - 1 - e])
    assert not any(_slot_bytes(big, s).any() for s in range(12) if s not in (4, 9, 7))


def _loader(blobs):
    import torch
    pinned = [torch.from_numpy(b.copy()).pin_memory() for b in blobs]
    return lambda layer, e: pinned[e]


def test_acquire_and_acquire_gpu(cuda):
    import torch
    from vates_b200.residency import ResidentExpertPool
    rng = np.random.default_rng(3)
    E = 16
    pool_np = random_pool_np(rng, E, H, I, BITS, G)
    blobs = _blobs_np(pool_np, E)
    rp = ResidentExpertPool(4, _loader(blobs), layers=2, num_experts=E, hidden=H, inter=I)
    pool, slots = rp.acquire(0, [2, 5, 2])
    assert slots[0] == slots[2] and rp.misses == 2
    _, slots2 = rp.acquire(0, [2, 5])
    assert slots2 == slots[:2] and rp.hits == 2
    inds = torch.tensor([[5, 7, 9]], dtype=torch.int32, device="cuda")
    lp, loc = rp.acquire_gpu(0, inds, E)
    torch.cuda.synchronize()
    table = rp.tables[0].cpu().numpy()
    assert loc.cpu().numpy().tolist() == [table[[5, 7, 9]].tolist()]
    assert (table[[5, 7, 9]] >= 0).all() and rp.gpu_fallback == 1
    for e in (5, 7, 9, 2):
        if table[e] >= 0:
            assert np.array_equal(_slot_bytes(lp, int(table[e])), blobs[e])
    rp.acquire_gpu(0, inds, E)
    assert rp.gpu_fastpath == 1
    # layer 1 is independent and its pool rows follow layer 0's
    _, s1 = rp.acquire(1, [0])
    torch.cuda.synchronize()
    assert np.array_equal(_slot_bytes(rp.pool, 4 + s1[0]), blobs[0])
    with pytest.raises(ValueError):
        rp.acquire(0, [0, 1, 2, 3, 4])


@pytest.mark.parametrize("T,cap,source,route_first", [(1, 16, "host", False),
                                                     (4, 32, "host", False),
                                                     (2, 16, "device", True),
                                                     (4, 32, "device", False)])
def test_decode_with_misses_matches_full_pool(cuda, T, cap, source, route_first):
    """Decode steps over a pool of ``cap`` < E slots: every routed miss is
    loaded (host flow, or the native vb_moe_decode_resident from an HBM blob
    store) and the block run once all are resident; outputs are
    bit-identical to the same block over all E experts, and the manager's
    state follows the oracle."""
    import torch
    from vates_b200.moe_block import MoeBlock
    from vates_b200.pool import QuantPool, make_table
    from vates_b200.residency import DeviceBlobStore, ResidentExpertPool
    E, k, L = 64, 6, 2
    rng = np.random.default_rng(10 + T)
    pools_np = [random_pool_np(rng, E, H, I, BITS, G) for _ in range(L)]
    blobs = [_blobs_np(p, E) for p in pools_np]
    sh = QuantPool.from_tensors(pool_to_torch(random_pool_np(rng, 1, H, I, BITS, G)), H, I, BITS, G)
    wsg = bf16_tensor(rng.standard_normal(H).astype(np.float32) * 0.02)
    wrs = [bf16_tensor(rng.standard_normal((E, H)).astype(np.float32) * 0.05) for _ in range(L)]
    full = [MoeBlock(wrs[l], make_table(E, {e: e for e in range(E)}),
                     QuantPool.from_tensors(pool_to_torch(pools_np[l]), H, I, BITS, G), sh, wsg,
                     top_k=k) for l in range(L)]
    if source == "device":
        store = DeviceBlobStore(torch.from_numpy(np.stack(blobs)).cuda())
        rp = ResidentExpertPool(cap, None, layers=L, num_experts=E, hidden=H, inter=I,
                                blob_store=store)
    else:
        pinned = [[torch.from_numpy(b.copy()).pin_memory() for b in bl] for bl in blobs]
        rp = ResidentExpertPool(cap, lambda l, e: pinned[l][e], layers=L, num_experts=E,
                                hidden=H, inter=I)
    res = [MoeBlock(wrs[l], rp.tables[l], rp.layer_pool(l), sh, wsg, top_k=k) for l in range(L)]
    orc = ResidencyOracle(L, cap, E)
    status = torch.zeros(1, dtype=torch.int32, device="cuda")
    runs = []
    xs = [bf16_tensor(rng.standard_normal((T, H)).astype(np.float32)) for _ in range(12)]
    for step in range(12):
        x = xs[step // 2 * 2]       # every input twice in a row: the repeat hits
        for l in range(L):
            want = full[l].decode(x).clone()
            out = torch.empty_like(x)
            dbg = res[l].new_debug(T)
            runs.append(rp.decode(l, res[l], x, out, status=status, debug=dbg,
                                  route_first=route_first))
            torch.cuda.synchronize()
            assert int(status.item()) == 0
            assert torch.equal(out.view(torch.int16), want.view(torch.int16)), f"step {step} layer {l}"
            orc.demand(l, dbg["inds"].reshape(-1).cpu().tolist())
            assert rp.state.table(l) == orc.L[l].table
    repeats = [runs[s * L + l] for s in range(1, 12, 2) for l in range(L)]
    if route_first:
        assert all(r == 2 for r in runs)
    else:
        assert 2 in runs and all(r == 1 for r in repeats)
    assert rp.state.table(0) == rp.tables[0].cpu().tolist()
    assert rp.misses > 0 and rp.hits > 0


def test_route_only_launch(cuda):
    """VB_DECODE_ROUTE_ONLY writes the routing outputs of the whole-block
    call, leaves out untouched, and the workspace stays usable."""
    import ctypes as C
    import torch
    from vates_b200._lib import VB_DECODE_ROUTE_ONLY, check, lib
    from vates_b200.moe_block import MoeBlock
    from vates_b200.pool import QuantPool, make_table, stream_handle
    E, k, T = 64, 6, 3
    rng = np.random.default_rng(5)
    pool = QuantPool.from_tensors(pool_to_torch(random_pool_np(rng, E, H, I, BITS, G)), H, I, BITS, G)
    table = make_table(E, {e: e for e in range(0, E, 2)})  # odd experts not resident
    wr = bf16_tensor(rng.standard_normal((E, H)).astype(np.float32) * 0.05)
    blk = MoeBlock(wr, table, pool, None, None, top_k=k)
    x = bf16_tensor(rng.standard_normal((T, H)).astype(np.float32))
    st_full = torch.zeros(1, dtype=torch.int32, device="cuda")
    d_full = blk.new_debug(T)
    ref = blk.decode(x, debug=d_full, status=st_full).clone()
    out = torch.full_like(x, 7.0)
    d_ro = blk.new_debug(T)
    st_ro = torch.zeros(1, dtype=torch.int32, device="cuda")
    a = blk.decode_args(x, out, debug=d_ro, status=st_ro)
    a.flags = VB_DECODE_ROUTE_ONLY
    check(lib.vb_moe_decode(C.byref(a), stream_handle()), "vb_moe_decode")
    torch.cuda.synchronize()
    for key in ("inds", "scores", "local"):
        assert torch.equal(d_ro[key].view(torch.int16) if key == "scores" else d_ro[key],
                           d_full[key].view(torch.int16) if key == "scores" else d_full[key])
    assert int(st_ro.item()) == int(st_full.item())
    assert bool((out == 7.0).all())
    again = blk.decode(x).clone()
    assert torch.equal(again.view(torch.int16), ref.view(torch.int16))


@pytest.mark.parametrize("T,source", [(1, "device"), (11, "host"), (4, "host")])
def test_mtp_moe_matches_full_pool(cuda, T, source):
    """The MTP drafter's MoE (StreamingMTPMoE, qwen3_next_mtp.py:70-137) over
    a pool smaller than the experts (room for one 8-token piece's routes):
    bit-identical to the block over all experts, token counts above 8 in
    pieces."""
    import torch
    from vates_b200.moe_block import MoeBlock
    from vates_b200.mtp import StreamingMTPMoE
    from vates_b200.pool import QuantPool, make_table
    from vates_b200.residency import DeviceBlobStore
    E, k = 64, 6
    cap = max(16, k * min(T, 8))
    rng = np.random.default_rng(20 + T)
    pool_np = random_pool_np(rng, E, H, I, BITS, G)
    blobs = _blobs_np(pool_np, E)
    sh_np = random_pool_np(rng, 1, H, I, BITS, G)
    sh = QuantPool.from_tensors(pool_to_torch(sh_np), H, I, BITS, G)
    wsg = bf16_tensor(rng.standard_normal(H).astype(np.float32) * 0.02)
    wr = bf16_tensor(rng.standard_normal((E, H)).astype(np.float32) * 0.05)
    layer = {"wr": to_np(wr), "wsg": to_np(wsg), "table": np.arange(E, dtype=np.int32),
             "pool": pool_np, "shared": sh_np, "hidden": H, "inter": I, "group": G,
             "bits": BITS}
    full = MoeBlock(wr, make_table(E, {e: e for e in range(E)}),
                    QuantPool.from_tensors(pool_to_torch(pool_np), H, I, BITS, G), sh, wsg, top_k=k)
    if source == "device":
        mtp = StreamingMTPMoE(wr, sh, wsg, cap, top_k=k, hidden=H, intermediate=I,
                              blob_store=DeviceBlobStore(torch.from_numpy(blobs[None]).cuda()))
    else:
        mtp = StreamingMTPMoE(wr, sh, wsg, cap, top_k=k, hidden=H, intermediate=I,
                              loader=_loader(blobs))
    for step in range(6):
        x = bf16_tensor(rng.standard_normal((1, T, H)).astype(np.float32))
        got = mtp(x)
        want = torch.cat([full.decode(x[0, i:i + 8]) for i in range(0, T, 8)])
        torch.cuda.synchronize()
        assert torch.equal(got[0].view(torch.int16), want.view(torch.int16)), f"step {step}"
        # against the oracle (StreamingMTPMoE.__call__, qwen3_next_mtp.py:114-137)
        # with its own routing: route sets agree up to bf16 ties, and every
        # token whose set is the oracle's matches its output
        for i in range(0, T, 8):
            n = min(8, T - i)
            g_inds = to_np(mtp._debug[n]["inds"])
            ref = OM.moe_block_decode(to_np(x[0, i:i + n]), layer, k=k)
            assert routes_agree(g_inds, ref["probs"], ref["inds"], k).all(), f"step {step}"
            same = np.array([set(a) == set(b) for a, b in zip(g_inds.tolist(),
                                                              ref["inds"].tolist())])
            if same.any():
                bf16_close(to_np(got[0, i:i + n])[same], ref["out"][same],
                           scale=block_scale(ref)[same], what=f"MTP MoE step {step} vs oracle")
    assert mtp.pool.misses > 0
