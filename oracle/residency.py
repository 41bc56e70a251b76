"""Expert residency state machine, restated on the CPU (test infrastructure
only: the product is vates_b200/csrc/residency.cu, which the tests compare
with this module bit for bit).

Follows the reference's native demand path for one layer's pool of `cap`
slots (native/ext/pool/demand.cpp):
  - init (real_ensure_locked, 286-304): free rows [0, cap) in order, table
    all -1;
  - demand (demand_core_locked, 966-1027): pass 1 resolves hits and collects
    the unique misses and unique accesses in first-seen order; LFU counts of
    every unique access go up by one (note_access_locked, 625-637, with the
    optional halving decay); if the unique experts of the request plus the
    pinned experts it does not use exceed cap, nothing changes and the
    request is refused (over capacity); pass 2 gives every unique miss a slot
    (alloc_slot_locked, 542-564: the front free row, else the victim's row);
    pass 3 fills the miss positions;
  - victim (choose_victim_locked, 514-529): among resident experts in
    insertion order, skipping pinned ones and those of the current request,
    the smallest LFU count, ties to the earliest inserted;
  - pin (real_pin, 364-394): pins the unique experts first, then places the
    missing ones (evictions never take a pinned or requested expert).
The prediction/speculative share of the reference's unified pool is not part
of this path.
"""
from collections import Counter


class LayerState:
    def __init__(self, cap: int, num_experts: int):
        self.cap = cap
        self.order: list[int] = []
        self.e2r: dict[int, int] = {}
        self.free: list[int] = list(range(cap))
        self.freq: Counter = Counter()
        self.pinned: set[int] = set()
        self.access = 0
        self.table = [-1] * num_experts


class ResidencyOracle:
    def __init__(self, layers: int, cap: int, num_experts: int, lfu: bool = True,
                 decay_interval: int = 0):
        self.lfu, self.decay = lfu, decay_interval
        self.L = [LayerState(cap, num_experts) for _ in range(layers)]

    # demand.cpp:514-529
    @staticmethod
    def _victim(c: LayerState, current: set) -> int:
        victim, best = -1, 0
        for e in c.order:
            if e not in c.e2r or e in c.pinned or e in current:
                continue
            f = c.freq.get(e, 0)
            if victim < 0 or f < best:
                victim, best = e, f
        return victim

    # demand.cpp:542-564
    def _alloc(self, c: LayerState, e: int, current: set) -> int:
        if e in c.e2r:
            return c.e2r[e]
        if c.free:
            slot = c.free.pop(0)
        else:
            v = self._victim(c, current)
            if v < 0:
                return -1
            slot = c.e2r.pop(v)
            c.table[v] = -1
            c.order.remove(v)
        c.e2r[e] = slot
        c.table[e] = slot
        c.order.append(e)
        return slot

    # demand.cpp:625-637
    def _note(self, c: LayerState, uniq: list[int]):
        if not self.lfu:
            return
        for e in uniq:
            c.freq[e] += 1
        c.access += len(uniq)
        if self.decay > 0 and c.access >= self.decay:
            for e in list(c.freq):
                c.freq[e] //= 2
                if c.freq[e] == 0:
                    del c.freq[e]
            c.access = 0

    def demand(self, layer: int, ids):
        """-> (local list, placements [(expert, slot)], (hits, misses, loads),
        over_capacity)."""
        c = self.L[layer]
        n = len(ids)
        local = [-1] * n
        uniq_miss, access_order = [], []
        miss_seen, access_seen, needed = set(), set(), set()
        hits = 0
        for i, e in enumerate(int(v) for v in ids):
            if e not in access_seen:
                access_seen.add(e)
                access_order.append(e)
            needed.add(e)
            if e in c.e2r:
                local[i] = c.e2r[e]
                hits += 1
                continue
            if e not in miss_seen:
                miss_seen.add(e)
                uniq_miss.append(e)
        self._note(c, access_order)
        unavailable_pins = sum(1 for e in c.pinned if e not in needed)
        if len(needed) + unavailable_pins > c.cap:
            return [0] * n, [], (hits, n - hits, 0), True
        placements = []
        new_slot = {}
        for e in uniq_miss:
            s = self._alloc(c, e, needed)
            assert s >= 0
            new_slot[e] = s
            placements.append((e, s))
        misses = 0
        for i, e in enumerate(int(v) for v in ids):
            if local[i] < 0:
                local[i] = new_slot[e]
                misses += 1
        return local, placements, (hits, misses, len(placements)), False

    # demand.cpp:364-394
    def pin(self, layer: int, experts):
        c = self.L[layer]
        unique, requested = [], set()
        for e in (int(v) for v in experts):
            if e not in requested:
                requested.add(e)
                unique.append(e)
        if len(c.pinned | requested) > c.cap:
            raise ValueError("pin count exceeds the pool capacity")
        c.pinned |= requested
        slots, placed = [], []
        for e in unique:
            if e in c.e2r:
                slots.append(c.e2r[e])
                continue
            s = self._alloc(c, e, requested)
            if s < 0:
                raise RuntimeError("no evictable slot")
            slots.append(s)
            placed.append((e, s))
        return slots, placed
