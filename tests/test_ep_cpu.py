"""Expert-parallel prefill orchestration on CPU ranks (gloo, world size 2).

The collective schedule of ``vates_b200.ep.ep_prefill`` runs unchanged; the
compute steps use a restated backend built on the oracle. The EP result on
two ranks must equal, bit for bit, the oracle's single-device prefill
(``_expert_major_forward`` + shared expert): every route value is computed
the same way and the reduce order (reference group, route rank) is a
property of the whole batch, shared through the all-reduced histogram.
"""
import os

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from helpers import random_pool_np
from oracle import mlx_ops as M
from oracle import moe as OM

T, H, I, E, K = 48, 256, 128, 12, 3
LAYER_CAP, MAX_ASSIGN = 4, 40


def _layer(seed=11):
    rng = np.random.default_rng(seed)
    pool = random_pool_np(rng, E, H, I, 4, 64)
    shared = random_pool_np(rng, 1, H, I, 4, 64)
    wr = M.bf16(rng.standard_normal((E, H)).astype(np.float32) * 0.05)
    wsg = M.bf16(rng.standard_normal(H).astype(np.float32) * 0.05)
    x = M.bf16(rng.standard_normal((T, H)).astype(np.float32))
    return pool, shared, wr, wsg, x


def _bf(a):
    return torch.from_numpy(np.ascontiguousarray(a, np.float32)).to(torch.bfloat16)


class OracleEpBackend:
    """The compute steps of ep_prefill restated on the CPU with the oracle."""

    def __init__(self, pool, shared, wr, wsg, owner, rank):
        self.pool, self.shared, self.wr, self.wsg = pool, shared, wr, wsg
        self.owner, self.rank = owner, rank

    def num_experts(self):
        return E

    def has_shared(self):
        return True

    def route(self, x):
        xr = x.float().numpy()
        _, _, inds, scores = OM.router(xr, self.wr, K, True)
        sg = M.bf16(M.matvec_f32(self.wsg[None, :], xr))[:, 0]
        sgate = M.bf16(M.sigmoid_f32(sg))
        counts = np.bincount(inds.reshape(-1), minlength=E).astype(np.int32)
        return (torch.from_numpy(inds.astype(np.int32)), torch.from_numpy(scores),
                torch.from_numpy(sgate), torch.from_numpy(counts))

    def pack(self, x, inds, scores, world):
        from vates_b200.ep import pack_reference
        ind, sc = inds.numpy(), scores.numpy()
        toks, rts, rsi, meta_row = pack_reference(ind, self.owner, world)
        rows = [t for d in range(world) for t in toks[d]]
        send_x = x[rows] if rows else x[:0]
        meta = np.zeros((len(meta_row), 3), np.int32)
        flat = [(t, j) for d in range(world) for (t, j) in rts[d]]
        for i, (t, j) in enumerate(flat):
            meta[i] = (meta_row[i], ind[t, j], np.float32(sc[t, j]).view(np.int32))
        cnt = np.array([[len(toks[d]) for d in range(world)],
                        [len(rts[d]) for d in range(world)]], np.int32)
        return send_x, torch.from_numpy(meta), torch.from_numpy(rsi.astype(np.int32)), \
            torch.from_numpy(cnt)

    def unpack(self, recv_meta, route_off, row_off, world):
        m = recv_meta.numpy()
        n = m.shape[0]
        src = np.searchsorted(np.asarray(route_off[1:]), np.arange(n), side="right")
        rows = np.asarray(row_off)[src] + m[:, 0] if n else np.zeros(0, np.int64)
        return (torch.from_numpy(rows.astype(np.int32)), torch.from_numpy(m[:, 1].copy()),
                torch.from_numpy(m[:, 2].copy().view(np.float32)))

    def experts(self, x, r_row, r_exp, r_score, name):
        xr = x.float().numpy()
        out = np.zeros((r_row.shape[0], H), np.float32)
        for i, (row, e, s) in enumerate(zip(r_row.tolist(), r_exp.tolist(), r_score.tolist())):
            if e == E:
                wg, wu, wd = OM.dequant_expert(self.shared, 0, H, I, 64, 4, to_bf16=True)
            else:
                assert self.owner[e] == self.rank, "a route reached a rank that does not own it"
                wg, wu, wd = OM.dequant_expert(self.pool, e, H, I, 64, 4, to_bf16=True)
            y = OM.expert_mlp_prefill(xr[row:row + 1], wg, wu, wd)
            out[i] = M.bf16(y * np.float32(s))[0]
        return _bf(out)

    def combine(self, inds, gcounts, y_back, rsi, y_shared, sgate):
        ind, ri = inds.numpy(), rsi.numpy()
        yb = y_back.float().numpy()
        groups = OM.expert_groups(gcounts.numpy(), LAYER_CAP, MAX_ASSIGN)
        gid = {e: g for g, (es, _) in enumerate(groups) for e in es}
        out = np.zeros((ind.shape[0], H), np.float32)
        for t in range(ind.shape[0]):
            acc = np.zeros(H, np.float32)
            for j in sorted(range(K), key=lambda j: (gid[int(ind[t, j])], j)):
                acc = M.bf16(acc + yb[ri[t, j]])
            sh = M.bf16(np.float32(sgate[t].item()) * y_shared[t].float().numpy())
            out[t] = M.bf16(acc + sh)
        return _bf(out)


def _rank(rank, world, port, owner, q):
    os.environ["MASTER_ADDR"], os.environ["MASTER_PORT"] = "127.0.0.1", str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        from vates_b200.ep import ep_prefill
        pool, shared, wr, wsg, x = _layer()
        per = T // world
        xl = _bf(x[rank * per:(rank + 1) * per])
        be = OracleEpBackend(pool, shared, wr, wsg, owner, rank)
        out = ep_prefill(be, xl)
        q.put((rank, out.float().numpy()))
    finally:
        dist.destroy_process_group()


def test_ep_prefill_two_gloo_ranks_matches_single_device():
    from vates_b200.ep import lpt_placement
    world = 2
    pool, shared, wr, wsg, x = _layer()
    owner = lpt_placement(np.arange(E)[::-1].astype(np.float64), world)
    assert set(owner.tolist()) == {0, 1}
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = 29600 + os.getpid() % 300
    procs = [ctx.Process(target=_rank, args=(r, world, port, owner, q)) for r in range(world)]
    for p in procs:
        p.start()
    res = dict(q.get(timeout=240) for _ in range(world))
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    got = np.concatenate([res[r] for r in range(world)])
    # single-device oracle
    _, _, inds, scores = OM.router(x, wr, K, True)
    routed = OM.expert_major_forward(x, inds, scores, lambda e: (pool, int(e)), H, I, 64, 4,
                                     layer_cap=LAYER_CAP, max_assignments=MAX_ASSIGN)
    ref = M.bf16(routed + OM.shared_prefill(x, shared, wsg, H, I, 64, 4))
    assert np.array_equal(got, ref)


def _rank_owners(rank, world, port, owners, q):
    _rank(rank, world, port, owners[rank], q)


def test_ep_prefill_with_replicated_hot_experts_matches_single_device():
    """Hot experts held by both ranks (each computes them for its own
    tokens), the rest owned by one rank: the output is still bit-identical
    to the single-device oracle."""
    from vates_b200.ep import placement
    world = 2
    pool, shared, wr, wsg, x = _layer()
    _, _, inds, _ = OM.router(x, wr, K, True)
    counts = np.bincount(inds.ravel(), minlength=E)
    owners = [placement(counts, world, r, share=1.0 / E)[0] for r in range(world)]
    rep = owners[0] == 0
    rep &= owners[1] == 1
    assert rep.any() and (~rep).any()
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = 29600 + (os.getpid() + 150) % 300
    procs = [ctx.Process(target=_rank_owners, args=(r, world, port, owners, q)) for r in range(world)]
    for p in procs:
        p.start()
    res = dict(q.get(timeout=240) for _ in range(world))
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    got = np.concatenate([res[r] for r in range(world)])
    routed = OM.expert_major_forward(x, inds, OM.router(x, wr, K, True)[3],
                                     lambda e: (pool, int(e)), H, I, 64, 4,
                                     layer_cap=LAYER_CAP, max_assignments=MAX_ASSIGN)
    ref = M.bf16(routed + OM.shared_prefill(x, shared, wsg, H, I, 64, 4))
    assert np.array_equal(got, ref)


def test_placement_replicates_hot_experts_only():
    from vates_b200.ep import hot_experts, placement
    counts = np.array([500, 5, 300, 4, 3, 2, 1, 0])
    hot = hot_experts(counts, 0.2)
    assert hot.tolist() == [True, False, True, False, False, False, False, False]
    o0, res0 = placement(counts, 2, 0, share=0.2)
    o1, res1 = placement(counts, 2, 1, share=0.2)
    assert o0[0] == 0 and o1[0] == 1 and o0[2] == 0 and o1[2] == 1
    cold = ~hot
    assert np.array_equal(o0[cold], o1[cold])  # one owner per cold expert
    assert (res0 | res1).all() and (res0 & res1).tolist() == hot.tolist()
    # one rank: nothing to replicate
    assert not hot_experts(counts, 0.0).any()
    assert (placement(counts, 1, 0)[0] == 0).all()


def test_lpt_placement_balances_and_is_deterministic():
    from vates_b200.ep import lpt_placement
    load = np.array([10, 9, 8, 1, 1, 1, 1, 1], np.float64)
    own = lpt_placement(load, 2)
    acc = [load[own == r].sum() for r in range(2)]
    assert abs(acc[0] - acc[1]) <= 2
    assert np.array_equal(own, lpt_placement(load, 2))


def test_pack_reference_orders_destinations_tokens_routes():
    from vates_b200.ep import pack_reference
    inds = np.array([[0, 3], [2, 1], [3, 3]])
    owner = np.array([0, 1, 1, 0])
    toks, rts, rsi, meta_row = pack_reference(inds, owner, 2)
    assert toks == [[0, 2], [1]]
    assert rts == [[(0, 0), (0, 1), (2, 0), (2, 1)], [(1, 0), (1, 1)]]
    assert rsi.tolist() == [[0, 1], [4, 5], [2, 3]]
    assert meta_row.tolist() == [0, 0, 1, 1, 0, 0]
