"""Expert-parallel prefill pieces on the GPU.

- ``vb_ep_pack`` against its numpy restatement (``pack_reference``);
- the prefill phases (route -> pack -> experts -> combine, one rank owning
  every expert) against ``vb_moe_prefill``: bit-identical;
- ``ep_prefill`` over NCCL on two GPUs against ``vb_moe_prefill`` on one:
  bit-identical (skipped unless two devices are visible).
"""
import os

import numpy as np
import pytest

from helpers import bf16_tensor, pool_to_torch, random_pool_np

pytestmark = pytest.mark.gpu

T, H, I, E, K = 320, 1024, 256, 24, 6


def _block(seed=5, owned=None):
    import torch
    from vates_b200.moe_block import MoeBlock
    from vates_b200.pool import QuantPool, make_table
    rng = np.random.default_rng(seed)
    pool_np = random_pool_np(rng, E, H, I, 4, 64)
    sh_np = random_pool_np(rng, 1, H, I, 4, 64)
    wr = bf16_tensor(rng.standard_normal((E, H)).astype(np.float32) * 0.02)
    wsg = bf16_tensor(rng.standard_normal(H).astype(np.float32) * 0.02)
    x = bf16_tensor(rng.standard_normal((T, H)).astype(np.float32))
    owned = list(range(E)) if owned is None else list(owned)
    sub = {k: v[owned] for k, v in pool_np.items()}
    pool = QuantPool.from_tensors(pool_to_torch(sub), H, I, 4, 64)
    sh = QuantPool.from_tensors(pool_to_torch(sh_np), H, I, 4, 64)
    table = make_table(E, {e: s for s, e in enumerate(owned)})
    blk = MoeBlock(wr, table, pool, sh, wsg, top_k=K)
    return blk, x


def test_ep_pack_matches_reference(cuda):
    import torch
    from vates_b200.ep import CudaEpBackend, pack_reference
    blk, x = _block()
    rng = np.random.default_rng(2)
    world = 4
    owner = rng.integers(0, world, E).astype(np.int32)
    inds = np.stack([rng.permutation(E)[:K] for _ in range(T)]).astype(np.int32)
    scores = rng.random((T, K)).astype(np.float32)
    be = CudaEpBackend(blk, torch.from_numpy(owner))
    send_x, meta, rsi, cnt = be.pack(x, torch.from_numpy(inds).cuda(),
                                     torch.from_numpy(scores).cuda(), world)
    toks, rts, rsi_ref, meta_row = pack_reference(inds, owner, world)
    cnt = cnt.cpu().numpy()
    assert cnt[0].tolist() == [len(v) for v in toks]
    assert cnt[1].tolist() == [len(v) for v in rts]
    assert np.array_equal(rsi.cpu().numpy(), rsi_ref)
    flat = [(t, j) for d in range(world) for (t, j) in rts[d]]
    m = meta.cpu().numpy()[:len(flat)]
    assert np.array_equal(m[:, 0], meta_row)
    assert np.array_equal(m[:, 1], np.array([inds[t, j] for t, j in flat]))
    assert np.array_equal(m[:, 2].view(np.float32), np.array([scores[t, j] for t, j in flat]))
    rows = [t for d in range(world) for t in toks[d]]
    assert torch.equal(send_x[:len(rows)], x[rows])


def test_prefill_phases_compose_to_the_single_call(cuda):
    import torch
    from vates_b200.ep import CudaEpBackend
    from vates_b200.prefill import moe_prefill
    blk, x = _block()
    ref = moe_prefill(blk, x)
    be = CudaEpBackend(blk, torch.zeros(E, dtype=torch.int32))
    inds, scores, sgate, counts = be.route(x)
    send_x, meta, rsi, cnt = be.pack(x, inds, scores, 1)
    n = int(cnt[1, 0].item())
    r_row, r_exp, r_score = be.unpack(meta[:n], [0, n], [0], 1)
    y = be.experts(send_x[:int(cnt[0, 0].item())], r_row, r_exp, r_score, "routed")
    s_row = torch.arange(T, dtype=torch.int32, device="cuda")
    s_exp = torch.full((T,), E, dtype=torch.int32, device="cuda")
    y_sh = be.experts(x, s_row, s_exp, torch.ones(T, device="cuda"), "shared")
    out = be.combine(inds, counts, y, rsi, y_sh, sgate)
    torch.cuda.synchronize()
    assert torch.equal(out, ref)


def _ep_rank(rank, world, port, q, owner=None, native=False):
    import torch
    import torch.distributed as dist
    os.environ["MASTER_ADDR"], os.environ["MASTER_PORT"] = "127.0.0.1", str(port)
    os.environ.setdefault("NCCL_NVLS_ENABLE", "0")
    torch.cuda.set_device(rank)
    import datetime
    dist.init_process_group("nccl", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=60),
                            device_id=torch.device("cuda", rank))
    try:
        from vates_b200.ep import CudaEpBackend, NativeEp, NcclComm, ep_prefill, lpt_placement
        if owner is None:
            owner = lpt_placement(np.ones(E), world)
        owned = [e for e in range(E) if owner[e] == rank]
        blk, x = _block(owned=owned)
        per = T // world
        xr = x[rank * per:(rank + 1) * per].contiguous()
        if native:
            comm = NcclComm()
            out = NativeEp(blk, owner, comm, max_tokens=per)(xr)
            torch.cuda.synchronize()
            comm.close()
        else:
            be = CudaEpBackend(blk, torch.from_numpy(owner))
            out = ep_prefill(be, xr)
        torch.cuda.synchronize()
        q.put((rank, out.float().cpu().numpy()))
    finally:
        dist.destroy_process_group()


def _collect(q, procs, limit_s=300):
    """Results of the rank processes; fails as soon as one of them exits
    without reporting (no waiting for the full limit)."""
    import queue
    import time
    res, t0 = {}, time.time()
    while len(res) < len(procs):
        try:
            r, out = q.get(timeout=2)
            res[r] = out
        except queue.Empty:
            dead = [p for p in procs if p.exitcode not in (None, 0)]
            if dead or time.time() - t0 > limit_s:
                for p in procs:
                    if p.is_alive():
                        p.terminate()
                pytest.fail(f"rank processes failed: {[p.exitcode for p in procs]}")
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode == 0
    return res


def test_native_ep_one_rank_matches_single_device(cuda):
    """vb_moe_prefill_ep through the C ABI on a one-rank NCCL communicator
    (every route stays on the rank: the self chunks are device copies):
    bit-identical to vb_moe_prefill, with and without replicated experts."""
    import torch
    from vates_b200.ep import NativeEp, NcclComm
    from vates_b200.prefill import moe_prefill
    blk, x = _block()
    ref = moe_prefill(blk, x)
    comm = NcclComm()
    try:
        out = NativeEp(blk, np.zeros(E, np.int32), comm, max_tokens=T)(x)
        torch.cuda.synchronize()
        assert torch.equal(out.view(torch.int16), ref.view(torch.int16))
        again = NativeEp(blk, np.zeros(E, np.int32), comm, max_tokens=2 * T)(x)
        torch.cuda.synchronize()
        assert torch.equal(again.view(torch.int16), ref.view(torch.int16))
    finally:
        comm.close()


@pytest.mark.parametrize("native", [False, True], ids=["torch_dist", "native"])
def test_ep_prefill_two_gpus_matches_one(cuda, native):
    import torch
    import torch.multiprocessing as mp
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    from vates_b200.prefill import moe_prefill
    blk, x = _block()
    ref = moe_prefill(blk, x).float().cpu().numpy()
    torch.cuda.synchronize()
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = 29700 + os.getpid() % 200
    procs = [ctx.Process(target=_ep_rank, args=(r, 2, port + int(native), q, None, native))
             for r in range(2)]
    for p in procs:
        p.start()
    res = _collect(q, procs)
    got = np.concatenate([res[0], res[1]])
    assert np.array_equal(got, ref)


@pytest.mark.parametrize("native", [False, True], ids=["torch_dist", "native"])
def test_ep_prefill_two_gpus_with_replicated_hot_experts(cuda, native):
    """Experts with many routes held by both GPUs (each computes them for
    its own tokens), the rest owned by one GPU: bit-identical to one GPU."""
    import torch
    import torch.multiprocessing as mp
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    from vates_b200.ep import placement
    from vates_b200.prefill import moe_prefill
    blk, x = _block()
    dbg = {"inds": torch.empty((T, K), dtype=torch.int32, device="cuda"),
           "scores": torch.empty((T, K), dtype=torch.bfloat16, device="cuda")}
    ref = moe_prefill(blk, x, debug=dbg).float().cpu().numpy()
    torch.cuda.synchronize()
    counts = np.bincount(dbg["inds"].cpu().numpy().ravel(), minlength=E)
    owners = [placement(counts, 2, r, share=1.0 / E)[0] for r in range(2)]
    hot = (owners[0] == 0) & (owners[1] == 1)
    assert hot.any() and (~hot).any()
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = 29700 + (os.getpid() + 100) % 200
    procs = [ctx.Process(target=_ep_rank, args=(r, 2, port + int(native), q, owners[r], native))
             for r in range(2)]
    for p in procs:
        p.start()
    res = _collect(q, procs)
    got = np.concatenate([res[0], res[1]])
    assert np.array_equal(got, ref)
