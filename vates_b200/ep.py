"""Expert-parallel (EP) expert-major prefill across the ranks of a process group.

The reference runs one device (``_expert_major_forward``, block.py:111-243);
here each rank owns the experts ``e`` with ``owner[e] == rank`` and starts
with its own slice of the tokens (``owner`` is per rank: experts replicated
on every rank map to the rank itself, see :func:`placement`). One prefill
step:

1. route the local tokens (router GEMM, top-k)                 ``vb_moe_route``
2. all-reduce the route histogram: the reference's reduce groups
   (block.py:154-172) are a property of the whole batch, so every rank adds
   its routes in the same order and the result does not depend on the
   number of ranks
3. pack token rows (once per destination rank) and route metadata ``vb_ep_pack``
4. all-to-all counts, rows and metadata (NCCL)
5. run the owned experts on the received routes                ``vb_moe_experts``
   and the shared expert on the local tokens (data parallel)
6. reverse all-to-all of the weighted route rows (NCCL)
7. reduce every token's routes in the reference's order        ``vb_moe_combine``

The collective steps are the same on every rank and in the same order. The
compute steps go through a backend object (``CudaEpBackend`` by default), so
the orchestration also runs on CPU ranks (``gloo``) with a restated backend
in the tests.
"""
from __future__ import annotations

import ctypes as C

import numpy as np
import torch
import torch.distributed as dist

from .pool import ptr, stream_handle


def lpt_placement(load: np.ndarray, world: int) -> np.ndarray:
    """Greedy longest-processing-time placement of experts over ranks:
    heaviest expert first, each to the currently least loaded rank (ties to
    the lower rank). Returns owner[e]."""
    load = np.asarray(load, np.float64)
    owner = np.zeros(load.shape[0], np.int32)
    acc = np.zeros(world, np.float64)
    for e in sorted(range(load.shape[0]), key=lambda i: (-load[i], i)):
        r = int(np.argmin(acc))
        owner[e] = r
        acc[r] += load[e]
    return owner


def hot_experts(counts: np.ndarray, share: float) -> np.ndarray:
    """Experts that carry at least ``share`` of all routes (a bool mask).

    Under skewed routing a handful of experts take most routes; sending
    their token rows to one owner and their route rows back would move most
    of the batch over NVLink and leave that owner with most of the work.
    These experts are instead held by every rank, which computes them for
    its own tokens (placement never changes a result: every route row is
    computed the same way on any rank)."""
    counts = np.asarray(counts, np.float64)
    total = counts.sum()
    if total <= 0 or share <= 0:
        return np.zeros(counts.shape[0], bool)
    return counts >= share * total


def placement(counts: np.ndarray, world: int, rank: int, share: float = 0.02):
    """This rank's ``owner[e]`` and resident-expert mask: experts of
    :func:`hot_experts` map to ``rank`` (replicated on every rank), the
    others to one rank each by :func:`lpt_placement` over their counts."""
    counts = np.asarray(counts, np.float64)
    hot = hot_experts(counts, share) if world > 1 else np.zeros(counts.shape[0], bool)
    owner = lpt_placement(np.where(hot, 0.0, counts), world)
    owner[hot] = rank
    return owner, (owner == rank)


def pack_reference(inds: np.ndarray, owner: np.ndarray, world: int):
    """What ``vb_ep_pack`` produces, restated in numpy: for every destination
    rank d (in rank order) the local tokens with a route to d (ascending) and
    the routes (t, j) to d (ascending). Returns ``(tokens_per_dest,
    routes_per_dest, route_send_idx, meta_row)`` where meta_row[i] is the row
    of route i inside its destination's chunk."""
    T, k = inds.shape
    dest = owner[inds]
    tokens_per_dest, routes_per_dest = [], []
    route_send_idx = np.full((T, k), -1, np.int64)
    meta_row = []
    base = 0
    for d in range(world):
        toks = [t for t in range(T) if (dest[t] == d).any()]
        row_of = {t: i for i, t in enumerate(toks)}
        rts = [(t, j) for t in range(T) for j in range(k) if dest[t, j] == d]
        for i, (t, j) in enumerate(rts):
            route_send_idx[t, j] = base + i
            meta_row.append(row_of[t])
        base += len(rts)
        tokens_per_dest.append(toks)
        routes_per_dest.append(rts)
    return tokens_per_dest, routes_per_dest, route_send_idx, np.asarray(meta_row, np.int64)


def _a2a(send: torch.Tensor, send_counts, recv_counts, group) -> torch.Tensor:
    """all_to_all_single with per-rank row counts (rows of the first dim)."""
    recv = send.new_empty((int(sum(recv_counts)),) + tuple(send.shape[1:]))
    dist.all_to_all_single(recv, send[: int(sum(send_counts))].contiguous(),
                           output_split_sizes=[int(c) for c in recv_counts],
                           input_split_sizes=[int(c) for c in send_counts], group=group)
    return recv


class CudaEpBackend:
    """Compute steps of the EP prefill on the local B200 (libvates_b200)."""

    def __init__(self, blk, owner: torch.Tensor, layer_cap: int = 0, max_assignments: int = 0):
        from ._lib import lib
        self.lib = lib
        self.blk = blk
        self.owner = owner.to(device=blk.router_w.device, dtype=torch.int32).contiguous()
        self.layer_cap, self.max_assignments = int(layer_cap), int(max_assignments)
        self.device = blk.router_w.device
        self._ws = {}

    def _workspace(self, name: str, nbytes: int) -> int:
        buf = self._ws.get(name)
        if buf is None or buf.numel() < nbytes + 1024:
            buf = torch.empty(nbytes + 1024, dtype=torch.uint8, device=self.device)
            self._ws[name] = buf
        return (buf.data_ptr() + 1023) // 1024 * 1024

    def route(self, x):
        from ._lib import VbMoeRouteArgs, check
        b, T, E, k = self.blk, int(x.shape[0]), self.blk.num_experts, self.blk.top_k
        inds = torch.empty((T, k), dtype=torch.int32, device=self.device)
        scores = torch.empty((T, k), dtype=torch.float32, device=self.device)
        sgate = torch.empty((T,), dtype=torch.float32, device=self.device)
        counts = torch.empty((E + 1,), dtype=torch.int32, device=self.device)
        need = self.lib.vb_moe_route_workspace_size(T, b.hidden, E)
        a = VbMoeRouteArgs()
        a.tokens, a.hidden, a.num_experts, a.top_k = T, b.hidden, E, k
        a.norm_topk = int(b.norm_topk_prob)
        a.x, a.router_w, a.router_bias = x.data_ptr(), b.router_w.data_ptr(), ptr(b.router_bias)
        a.shared_gate_w = ptr(b.shared_gate_w) if b.shared is not None else None
        a.out_inds, a.out_scores, a.out_sgate = inds.data_ptr(), scores.data_ptr(), sgate.data_ptr()
        a.out_counts = counts.data_ptr()
        a.workspace, a.workspace_bytes = self._workspace("route", need), need
        check(self.lib.vb_moe_route(C.byref(a), stream_handle(None)), "vb_moe_route")
        return inds, scores, sgate, counts[:E]

    def pack(self, x, inds, scores, world):
        from ._lib import VbEpPackArgs, check
        T, k = inds.shape
        H = int(x.shape[1])
        send_x = torch.empty((T * min(k, world), H), dtype=x.dtype, device=self.device)
        send_meta = torch.empty((T * k, 3), dtype=torch.int32, device=self.device)
        rsi = torch.empty((T, k), dtype=torch.int32, device=self.device)
        counts = torch.empty((2, world), dtype=torch.int32, device=self.device)
        a = VbEpPackArgs()
        a.tokens, a.top_k, a.hidden, a.world = T, k, H, world
        a.x, a.inds, a.scores, a.owner = x.data_ptr(), inds.data_ptr(), scores.data_ptr(), \
            self.owner.data_ptr()
        a.send_x, a.send_meta, a.route_send_idx = send_x.data_ptr(), send_meta.data_ptr(), rsi.data_ptr()
        a.dest_rows, a.dest_routes = counts[0].data_ptr(), counts[1].data_ptr()
        need = self.lib.vb_ep_pack_workspace_size(T, world)
        a.workspace, a.workspace_bytes = self._workspace("pack", need), need
        check(self.lib.vb_ep_pack(C.byref(a), stream_handle(None)), "vb_ep_pack")
        return send_x, send_meta, rsi, counts

    def unpack(self, recv_meta, route_off, row_off, world):
        from ._lib import check
        n = int(recv_meta.shape[0])
        rr = torch.empty((n,), dtype=torch.int32, device=self.device)
        re = torch.empty((n,), dtype=torch.int32, device=self.device)
        rs = torch.empty((n,), dtype=torch.float32, device=self.device)
        ro = torch.tensor(route_off, dtype=torch.int32, device=self.device)
        wo = torch.tensor(row_off, dtype=torch.int32, device=self.device)
        check(self.lib.vb_ep_unpack(ptr(recv_meta) if n else None, n, ro.data_ptr(),
                                    wo.data_ptr(), world, rr.data_ptr(), re.data_ptr(),
                                    rs.data_ptr(), stream_handle(None)), "vb_ep_unpack")
        return rr, re, rs

    def experts(self, x, r_row, r_exp, r_score, name):
        from ._lib import VbMoeExpertsArgs, check
        b, n = self.blk, int(r_row.shape[0])
        out = torch.empty((n, b.hidden), dtype=torch.bfloat16, device=self.device)
        a = VbMoeExpertsArgs()
        a.rows, a.routes, a.hidden, a.inter = int(x.shape[0]), n, b.hidden, b.inter
        a.group, a.bits, a.num_experts = b.pool.group, b.pool.bits, b.num_experts
        a.x = x.data_ptr() if x.numel() else None
        a.route_row, a.route_expert, a.route_score = ptr(r_row), ptr(r_exp), ptr(r_score)
        a.slot_table = b.slot_table.data_ptr()
        a.pool = b._pool_c
        if b._shared_c is not None:
            a.shared = b._shared_c
        a.out = out.data_ptr()
        need = self.lib.vb_moe_experts_workspace_size(n, b.hidden, b.inter, b.num_experts)
        a.workspace, a.workspace_bytes = self._workspace(name, need), need
        check(self.lib.vb_moe_experts(C.byref(a), stream_handle(None)), "vb_moe_experts")
        return out

    def combine(self, inds, gcounts, y_back, route_row, y_shared, sgate):
        from ._lib import VbMoeCombineArgs, check
        b = self.blk
        T, k = inds.shape
        out = torch.empty((T, b.hidden), dtype=torch.bfloat16, device=self.device)
        gws = torch.empty((b.num_experts,), dtype=torch.int32, device=self.device)
        a = VbMoeCombineArgs()
        a.tokens, a.hidden, a.num_experts, a.top_k = T, b.hidden, b.num_experts, k
        a.layer_cap, a.max_assignments = self.layer_cap, self.max_assignments
        a.inds, a.counts = inds.data_ptr(), gcounts.data_ptr()
        a.y_routes = y_back.data_ptr() if y_back.numel() else out.data_ptr()
        a.route_row = route_row.data_ptr()
        a.y_shared = ptr(y_shared)
        a.sgate = sgate.data_ptr()
        a.out, a.group_of_ws = out.data_ptr(), gws.data_ptr()
        check(self.lib.vb_moe_combine(C.byref(a), stream_handle(None)), "vb_moe_combine")
        return out

    def has_shared(self):
        return self.blk.shared is not None

    def num_experts(self):
        return self.blk.num_experts


class NcclComm:
    """An NCCL communicator of its own over the ranks of ``group`` (rank 0's
    ``ncclUniqueId`` is broadcast through the process group). The native EP
    prefill issues its point-to-point calls on it, apart from torch's own
    communicators."""

    class _UniqueId(C.Structure):
        _fields_ = [("internal", C.c_char * 128)]

    def __init__(self, group=None):
        self.nccl = C.CDLL("libnccl.so.2")  # the copy torch already loaded
        self.nccl.ncclGetUniqueId.argtypes = [C.POINTER(self._UniqueId)]
        self.nccl.ncclCommInitRank.argtypes = [C.POINTER(C.c_void_p), C.c_int, self._UniqueId,
                                               C.c_int]
        self.nccl.ncclCommDestroy.argtypes = [C.c_void_p]
        single = not (dist.is_available() and dist.is_initialized())
        self.world = 1 if single else dist.get_world_size(group)
        self.rank = 0 if single else dist.get_rank(group)
        uid = self._UniqueId()
        if self.rank == 0:
            rc = self.nccl.ncclGetUniqueId(C.byref(uid))
            if rc != 0:
                raise RuntimeError(f"ncclGetUniqueId failed ({rc})")
        if not single:
            # all 128 bytes (a c_char array field would stop at the first NUL)
            box = [C.string_at(C.addressof(uid), 128) if self.rank == 0 else None]
            dist.broadcast_object_list(box, src=dist.get_global_rank(group, 0) if group else 0,
                                       group=group)
            assert len(box[0]) == 128
            C.memmove(C.addressof(uid), box[0], 128)
        self.comm = C.c_void_p()
        rc = self.nccl.ncclCommInitRank(C.byref(self.comm), self.world, uid, self.rank)
        if rc != 0:
            raise RuntimeError(f"ncclCommInitRank failed ({rc})")

    def close(self):
        if self.comm:
            torch.cuda.synchronize()
            self.nccl.ncclCommDestroy(self.comm)
            self.comm = C.c_void_p()


class NativeEp:
    """Expert-parallel prefill through the C ABI (``vb_moe_prefill_ep``): the
    whole schedule of :func:`ep_prefill` in one native call per step.

    ``blk`` holds this rank's experts (its slot table is -1 for the others),
    ``owner`` the placement of :func:`placement`, ``max_tokens`` the largest
    token count of any rank."""

    def __init__(self, blk, owner, comm: NcclComm, max_tokens: int, layer_cap: int = 0,
                 max_assignments: int = 0):
        from ._lib import lib
        self.lib, self.blk, self.comm = lib, blk, comm
        self.owner = torch.as_tensor(owner).to(device=blk.router_w.device,
                                               dtype=torch.int32).contiguous()
        self.max_tokens = int(max_tokens)
        self.layer_cap, self.max_assignments = int(layer_cap), int(max_assignments)
        self._ws = None

    def __call__(self, x_local: torch.Tensor, out=None, status=None, stream=None):
        from ._lib import VbMoePrefillEpArgs, check
        from .prefill import prefill_args
        b = self.blk
        x2 = x_local.reshape(-1, b.hidden).contiguous()
        T = int(x2.shape[0])
        if out is None:
            out = torch.empty_like(x2)
        need = self.lib.vb_moe_prefill_ep_workspace_size(T, b.hidden, b.inter, b.num_experts,
                                                         b.top_k, self.comm.world,
                                                         max(self.max_tokens, T))
        if self._ws is None or self._ws.numel() < need + 1024:
            self._ws = None
            self._ws = torch.empty(need + 1024, dtype=torch.uint8, device=x2.device)
        ws = (self._ws.data_ptr() + 1023) // 1024 * 1024
        a = VbMoePrefillEpArgs()
        a.base = prefill_args(b, x2, out, ws, need, status=status, layer_cap=self.layer_cap,
                              max_assignments=self.max_assignments)
        a.owner = self.owner.data_ptr()
        a.world, a.rank = self.comm.world, self.comm.rank
        a.max_tokens_per_rank = max(self.max_tokens, T)
        check(self.lib.vb_moe_prefill_ep(C.byref(a), self.comm.comm, stream_handle(stream)),
              "vb_moe_prefill_ep")
        return out


def ep_prefill(backend, x_local: torch.Tensor, group=None, timings: dict | None = None):
    """One expert-parallel prefill step of the block on this rank's tokens.

    Every rank calls it with its own ``x_local`` (bf16 ``[T_r, H]``); the
    result is this rank's output rows. Collectives: one all_reduce and four
    all_to_all_single, in the same order on every rank.
    """
    world = dist.get_world_size(group)
    E = backend.num_experts()
    inds, scores, sgate, counts = backend.route(x_local)
    gcounts = counts.clone()
    dist.all_reduce(gcounts, group=group)
    send_x, send_meta, rsi, cnt = backend.pack(x_local, inds, scores, world)
    # rows and routes per destination -> per source
    sc = cnt.to(torch.int64).t().contiguous()    # [world, 2]
    rc = torch.empty_like(sc)
    dist.all_to_all_single(rc, sc, group=group)
    sc_h, rc_h = sc.cpu().numpy(), rc.cpu().numpy()
    send_rows, send_routes = sc_h[:, 0], sc_h[:, 1]
    recv_rows, recv_routes = rc_h[:, 0], rc_h[:, 1]
    recv_x = _a2a(send_x, send_rows, recv_rows, group)
    recv_meta = _a2a(send_meta, send_routes, recv_routes, group)
    route_off = np.concatenate([[0], np.cumsum(recv_routes)]).astype(np.int64)
    row_off = np.concatenate([[0], np.cumsum(recv_rows)[:-1]]).astype(np.int64)
    r_row, r_exp, r_score = backend.unpack(recv_meta, route_off.tolist(), row_off.tolist(), world)
    y_recv = backend.experts(recv_x, r_row, r_exp, r_score, "routed")
    y_shared = None
    if backend.has_shared():
        T = int(x_local.shape[0])
        dev = x_local.device
        s_row = torch.arange(T, dtype=torch.int32, device=dev)
        s_exp = torch.full((T,), E, dtype=torch.int32, device=dev)
        s_score = torch.ones((T,), dtype=torch.float32, device=dev)
        y_shared = backend.experts(x_local, s_row, s_exp, s_score, "shared")
    y_back = _a2a(y_recv, recv_routes, send_routes, group)
    return backend.combine(inds, gcounts, y_back, rsi, y_shared, sgate)
