"""Expert residency for pools smaller than the expert count.

Host mirror of ``ResidentExpertPool`` (mlx_streaming/core/cache/
resident_pool.py:54-640) over the native slot state of ``libvates_b200``
(``vb_res_*``, the demand state machine of native/ext/pool/demand.cpp):

- ``acquire(layer, expert_ids)`` (resident_pool.py:497-537): unique experts of
  the request, LFU note, one slot per unique miss (front free row, else the
  LFU victim that is neither pinned nor part of the request), the misses'
  bytes copied into their slots; returns ``(pool, slots)`` with one slot per
  requested id. More unique experts (plus the pins they do not use) than
  slots raises ``ValueError`` like the reference.
- ``pin(layer, expert_ids)`` (436-477): loads and pins, never evicted.
- ``acquire_gpu(layer, inds, num_experts)`` (560-580): device slot-table
  gather; hits keep the device path, misses go through ``acquire`` and the
  table is gathered again.
- ``decode(layer, block, x, ...)``: the fused decode kernel routes on the
  device and flags ``VB_STATUS_MISS`` when a routed expert is not resident;
  the host then demands the routed experts, fills the missing slots and runs
  the kernel again (its output is rewritten; inputs are not modified).

Expert bytes come from ``loader(layer, expert)`` as one blob in the
``expert_blob_v1`` layout (prep/blob_layout.py:14-32): a host array/tensor
(pinned for asynchronous copies) or a CUDA tensor. A ``DeviceBlobStore``
keeps every expert of a layer in HBM and fills a demand's misses with one
gather kernel (``vb_blob_gather``).
"""
from __future__ import annotations

import ctypes as C

import numpy as np
import torch

from ._lib import VB_ERR_CAPACITY, VB_OK, VB_STATUS_MISS, VbError, check, lib
from .pool import QuantPool, blob_layout, slot_remap, stream_handle

def _i32(n: int):
    return (C.c_int32 * max(n, 1))()


class NativeResidency:
    """The per-layer expert -> slot state (``vb_res_*``), one handle."""

    def __init__(self, layers: int, cap: int, num_experts: int, lfu: bool = True,
                 decay_interval: int = 0):
        self.layers, self.cap, self.num_experts = layers, cap, num_experts
        h = lib.vb_res_create(layers, cap, num_experts, int(lfu), decay_interval)
        if not h:
            raise VbError("vb_res_create failed: " + lib.vb_last_error().decode())
        self._h = h

    def close(self):
        if getattr(self, "_h", None):
            lib.vb_res_destroy(self._h)
            self._h = None

    def __del__(self):
        self.close()

    def demand(self, layer: int, ids):
        """-> (local list, placements [(expert, slot)], (hits, misses, loads),
        over_capacity) — the reference's demand_core_locked results."""
        ids = [int(v) for v in ids]
        n = len(ids)
        arr = (C.c_int32 * max(n, 1))(*ids)
        local, pe, ps = _i32(n), _i32(n), _i32(n)
        n_place = C.c_int32(0)
        stats = (C.c_int64 * 3)()
        rc = lib.vb_res_demand(self._h, layer, arr, n, local, pe, ps, C.byref(n_place), stats)
        if rc not in (VB_OK, VB_ERR_CAPACITY):
            check(rc, "vb_res_demand")
        place = [(pe[i], ps[i]) for i in range(n_place.value)]
        return list(local[:n]), place, tuple(stats), rc == VB_ERR_CAPACITY

    def demand_into(self, layer: int, ids: np.ndarray, local: np.ndarray, place: np.ndarray,
                    stats: np.ndarray) -> tuple[int, bool]:
        """Array form of :meth:`demand` for the per-layer hot path: ``ids``
        int32 [n]; ``local`` int32 [>= n]; ``place`` int32 [2, >= n] receives
        experts (row 0) and slots (row 1); ``stats`` int64 [3]. Returns
        (placements, over_capacity)."""
        n = int(ids.size)
        n_place = C.c_int32(0)
        rc = lib.vb_res_demand(self._h, layer, ids.ctypes.data, n, local.ctypes.data,
                               place[0].ctypes.data, place[1].ctypes.data, C.byref(n_place),
                               stats.ctypes.data)
        if rc not in (VB_OK, VB_ERR_CAPACITY):
            check(rc, "vb_res_demand")
        return n_place.value, rc == VB_ERR_CAPACITY

    def table_into(self, layer: int, out: np.ndarray) -> None:
        """The layer's table into an int32 [num_experts] array (e.g. pinned)."""
        check(lib.vb_res_table(self._h, layer, out.ctypes.data), "vb_res_table")

    def pin(self, layer: int, experts):
        """-> (slots of the unique experts, [(expert, slot)] newly placed)."""
        experts = [int(v) for v in experts]
        n = len(experts)
        arr = (C.c_int32 * max(n, 1))(*experts)
        slots, placed = _i32(n), _i32(n)
        nu = C.c_int32(0)
        rc = lib.vb_res_pin(self._h, layer, arr, n, slots, placed, C.byref(nu))
        if rc == VB_ERR_CAPACITY:
            raise ValueError(lib.vb_last_error().decode())
        check(rc, "vb_res_pin")
        uniq = list(dict.fromkeys(experts))
        return list(slots[:nu.value]), [(uniq[i], slots[i]) for i in range(nu.value) if placed[i]]

    def table(self, layer: int) -> list[int]:
        t = _i32(self.num_experts)
        check(lib.vb_res_table(self._h, layer, t), "vb_res_table")
        return list(t[:self.num_experts])

    def counts(self, layer: int) -> dict[int, int]:
        """Non-zero LFU access counts of the layer."""
        c = (C.c_uint32 * self.num_experts)()
        check(lib.vb_res_counts(self._h, layer, c), "vb_res_counts")
        return {e: int(c[e]) for e in range(self.num_experts) if c[e]}

    def resident(self, layer: int) -> list[tuple[int, int]]:
        e, s = _i32(self.cap), _i32(self.cap)
        n = C.c_int32(0)
        check(lib.vb_res_resident(self._h, layer, e, s, C.byref(n)), "vb_res_resident")
        return [(e[i], s[i]) for i in range(n.value)]


class DeviceBlobStore:
    """Every expert blob of some layers in one HBM tensor ``[layers, E, stride]``
    (or mapped pinned host memory with ``device="cpu"``, pinned); misses are
    gathered into pool slots by one kernel launch."""

    def __init__(self, blobs: torch.Tensor):
        assert blobs.dim() == 3 and blobs.dtype == torch.uint8 and blobs.is_contiguous()
        self.blobs = blobs
        self.stride = int(blobs.shape[2])

    def fill(self, layer: int, pool: QuantPool, placements, stream=None, staging=None) -> None:
        """Gather experts into pool slots: ``placements`` is a list of
        (expert, slot) or an int32 array [2, n] (experts, slots). ``staging``
        (pinned int32 [2, >= n], optional) holds the index copy; the caller
        must not rewrite it before the copy has run."""
        if isinstance(placements, np.ndarray):
            n = int(placements.shape[1])
        else:
            n = len(placements)
            placements = np.array(placements, dtype=np.int32).reshape(n, 2).T if n else None
        if n == 0:
            return
        assert pool.blob is not None and self.stride == pool.stride
        idx = staging if staging is not None else torch.empty((2, n), dtype=torch.int32,
                                                              pin_memory=True)
        h = idx.numpy()
        h[0, :n] = placements[0, :n]
        h[1, :n] = placements[1, :n] + pool.blob_slot0
        s = stream or torch.cuda.current_stream()
        with torch.cuda.stream(s):
            dev = idx[:, :n].to(pool.blob.device, non_blocking=True)
            check(lib.vb_blob_gather(self.blobs[layer].data_ptr(), self.stride, dev[0].data_ptr(),
                                     dev[1].data_ptr(), n, pool.blob.data_ptr(), s.cuda_stream),
                  "vb_blob_gather")


def fill_slots(pool: QuantPool, slots, blobs, stream=None) -> None:
    """Copy expert blobs (host or device, ``expert_blob_v1`` layout) into pool
    slots with ``vb_pool_fill``."""
    n = len(slots)
    if n == 0:
        return
    _, stride = blob_layout(pool.hidden, pool.inter, pool.bits, pool.group)
    keep, ptrs = [], (C.c_void_p * n)()
    for i, b in enumerate(blobs):
        if isinstance(b, np.ndarray):
            b = torch.from_numpy(np.ascontiguousarray(b).view(np.uint8).reshape(-1))
        b = b.contiguous()
        if b.numel() * b.element_size() != stride:
            raise VbError(f"expert blob of {b.numel() * b.element_size()} bytes, layout needs {stride}")
        keep.append(b)
        ptrs[i] = b.data_ptr()
    sl = (C.c_int32 * n)(*[int(s) for s in slots])
    pc = pool.c_struct()
    check(lib.vb_pool_fill(C.byref(pc), pool.hidden, pool.inter, pool.group, pool.bits, sl,
                           ptrs, n, stream_handle(stream)), "vb_pool_fill")
    if any(not k.is_cuda and not k.is_pinned() for k in keep):
        # Pageable sources: wait before the temporaries are released.
        (stream or torch.cuda.current_stream()).synchronize()


class ResidentExpertPool:
    """``layers`` pools of ``capacity`` slots in one HBM blob tensor
    ``[layers * capacity, stride]``, the native slot state and the device
    expert -> slot tables the kernels read."""

    def __init__(self, capacity: int, loader=None, *, layers: int, num_experts: int,
                 hidden: int, inter: int, bits: int = 4, group: int = 64,
                 eviction_policy: str = "lfu", lfu_decay_interval: int = 0,
                 blob_store: DeviceBlobStore | None = None, device="cuda"):
        # "fifo" is the native demand state with LFU counting off: every count
        # stays 0, so the victim is the earliest inserted unpinned expert.
        if eviction_policy not in ("lfu", "fifo"):
            raise ValueError(f"eviction_policy {eviction_policy!r}")
        if loader is None and blob_store is None:
            raise ValueError("a loader or a blob store is required")
        self.capacity, self.layers, self.num_experts = capacity, layers, num_experts
        self.loader, self.blob_store = loader, blob_store
        self.eviction_policy = eviction_policy
        self.state = NativeResidency(layers, capacity, num_experts,
                                     eviction_policy == "lfu", lfu_decay_interval)
        self.pool = QuantPool.empty_blob(layers * capacity, hidden, inter, bits, group, device)
        self.tables = torch.full((layers, num_experts), -1, dtype=torch.int32, device=device)
        self.hits = self.misses = self.loads = 0
        self.gpu_fastpath = self.gpu_fallback = 0
        self.over_capacity = 0
        # Pinned host staging of the per-layer hot path (decode): the status
        # word and routed ids read back, the host tables, the gather indices.
        self._h_tables = torch.full((layers, num_experts), -1, dtype=torch.int32,
                                    pin_memory=True)
        self._h_back = torch.zeros(1 + 64, dtype=torch.int32, pin_memory=True)
        self._h_idx = torch.zeros((2, capacity), dtype=torch.int32, pin_memory=True)
        self._local = np.zeros(64, np.int32)
        self._place = np.zeros((2, 64), np.int32)
        self._stats = np.zeros(3, np.int64)

    # resident_pool.py:133-135
    def cap_for(self, layer: int) -> int:
        return self.capacity

    def layer_pool(self, layer: int) -> QuantPool:
        return self.pool.view(layer * self.capacity, self.capacity)

    def _load(self, layer: int, placements, stream=None) -> None:
        """Copy the placed experts' bytes into their slots and the layer's
        table to the device, stream-ordered (``placements``: (expert, slot)
        list or int32 [2, n])."""
        if isinstance(placements, np.ndarray):
            pl = placements
        else:
            pl = np.array(placements, dtype=np.int32).reshape(-1, 2).T
        n = int(pl.shape[1])
        if n == 0:
            return
        s = stream or torch.cuda.current_stream()
        p = self.layer_pool(layer)
        if self.blob_store is not None:
            self.blob_store.fill(layer, p, pl, s, staging=self._h_idx if n <= self.capacity else None)
        else:
            fill_slots(p, pl[1].tolist(), [self.loader(layer, int(e)) for e in pl[0]], s)
        self.loads += n
        self.state.table_into(layer, self._h_tables[layer].numpy())
        with torch.cuda.stream(s):
            self.tables[layer].copy_(self._h_tables[layer], non_blocking=True)
        # The staging buffers are rewritten by the next load: wait for these
        # copies unless the caller synchronises before then (decode does).

    def acquire(self, layer: int, expert_ids, stream=None):
        ids = [int(e) for e in expert_ids]
        uniq = list(dict.fromkeys(ids))
        local, place, _, over = self.state.demand(layer, ids)
        if over:
            self.over_capacity += 1
            raise ValueError(f"request of {len(uniq)} unique experts does not fit the "
                             f"layer's {self.capacity} slots with its pins")
        self.hits += len(uniq) - len(place)
        self.misses += len(place)
        self._load(layer, place, stream)
        (stream or torch.cuda.current_stream()).synchronize()
        return self.layer_pool(layer), local

    def pin(self, layer: int, expert_ids, stream=None) -> None:
        _, placed = self.state.pin(layer, expert_ids)
        self._load(layer, placed, stream)
        (stream or torch.cuda.current_stream()).synchronize()

    def resident_count(self, layer: int) -> int:
        return len(self.state.resident(layer))

    def resident_experts(self, layer: int) -> set[int]:
        return {e for e, _ in self.state.resident(layer)}

    def acquire_gpu(self, layer: int, inds: torch.Tensor, num_experts: int | None = None,
                    stream=None):
        """-> (layer pool, local) with ``local = table[inds]`` on the device."""
        assert num_experts in (None, self.num_experts)
        ids = inds.reshape(-1).to(torch.int32)
        if stream is not None:
            stream.synchronize()
        host = ids.cpu().tolist()
        local, place, _, over = self.state.demand(layer, host)
        if over:
            self.over_capacity += 1
            raise ValueError("request does not fit the layer's slots with its pins")
        if place:
            self.gpu_fallback += 1
            self.misses += len(place)
            self.hits += len(set(host)) - len(place)
            self._load(layer, place, stream)
            (stream or torch.cuda.current_stream()).synchronize()
        else:
            self.gpu_fastpath += 1
            self.hits += len(host)
        loc = slot_remap(ids, self.tables[layer], stream=stream).reshape(inds.shape)
        return self.layer_pool(layer), loc

    def decode(self, layer: int, block, x: torch.Tensor, out: torch.Tensor, *,
               residual=None, status: torch.Tensor, debug: dict, stream=None,
               norm_eps: float = 0.0, route_first: bool = True) -> int:
        """One decode call of ``block`` (a MoeBlock over this layer's pool and
        table) with misses resolved; returns the number of kernel launches.

        With a blob store the whole flow is native (``vb_moe_decode_resident``):
        ``route_first`` runs a routing-only launch, loads the misses and then
        the block (2 launches, one host synchronisation); otherwise the block
        runs first and again only after a miss. With a host loader the same
        optimistic flow runs here. ``status`` is a device int32 word; after a
        native call it holds the last launch's status (not read here).
        ``debug`` receives the routed ids."""
        assert out.data_ptr() not in (x.data_ptr(), getattr(residual, "data_ptr", lambda: 0)())
        if self.blob_store is not None:
            x2 = x.reshape(-1, block.hidden)
            a = block.decode_args(x2, out, residual=residual, debug=debug, status=status,
                                  norm_eps=norm_eps)
            cnt = (C.c_int64 * 4)()
            st = self.blob_store.blobs[layer]
            check(lib.vb_moe_decode_resident(C.byref(a), self.state._h, layer, st.data_ptr(),
                                             self.blob_store.stride, int(route_first), cnt,
                                             stream_handle(stream)), "vb_moe_decode_resident")
            self.hits += cnt[0]
            self.misses += cnt[1]
            self.loads += cnt[1]
            return int(cnt[3])
        s = stream or torch.cuda.current_stream()
        inds = debug["inds"].reshape(-1)
        n = int(inds.numel())
        assert n <= 64
        back = self._h_back
        with torch.cuda.stream(s):
            status.zero_()
        block.decode(x, out=out, residual=residual, debug=debug, status=status, stream=s,
                     norm_eps=norm_eps)
        with torch.cuda.stream(s):
            back[:1].copy_(status, non_blocking=True)
            back[1:1 + n].copy_(inds, non_blocking=True)
        s.synchronize()
        hb = back.numpy()
        st = int(hb[0])
        ids = hb[1:1 + n]
        n_place, over = self.state.demand_into(layer, ids, self._local, self._place, self._stats)
        if over:
            self.over_capacity += 1
            raise ValueError("routed experts do not fit the layer's slots with its pins")
        uniq = len(set(ids.tolist()))
        self.hits += uniq - n_place
        self.misses += n_place
        if not (st & VB_STATUS_MISS):
            if n_place:
                raise VbError("kernel saw every expert resident but the host state placed some")
            return 1
        if st & ~VB_STATUS_MISS:
            raise VbError(f"decode status {st:#x}")
        self._load(layer, self._place[:, :n_place], s)
        with torch.cuda.stream(s):
            status.zero_()
        block.decode(x, out=out, residual=residual, debug=debug, status=status, stream=s,
                     norm_eps=norm_eps)
        with torch.cuda.stream(s):
            back[:1].copy_(status, non_blocking=True)
        s.synchronize()
        st = int(back.numpy()[0])
        if st:
            raise VbError(f"decode status {st:#x} after filling the misses")
        return 2

    def hit_rate(self) -> float:
        tot = self.hits + self.misses
        return self.hits / tot if tot else 0.0


__all__ = ["NativeResidency", "ResidentExpertPool", "DeviceBlobStore", "fill_slots"]
