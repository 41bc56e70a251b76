// Expert residency for the per-layer quantized pools: which expert sits in
// which slot, what to load on a miss, and the copies that fill the slots.
//
// Reference: the native demand path (native/ext/pool/demand.cpp) behind
// ResidentExpertPool (mlx_streaming/core/cache/resident_pool.py:54-580):
//  - per layer: expert -> slot map, insertion order, free rows (front
//    first), LFU counts, pinned experts, and the expert -> slot table the
//    kernels read (real_ensure_locked 286-304, real_table_set_locked 306);
//  - demand_core_locked (966-1027): hits, unique misses and unique accesses
//    in first-seen order; LFU +1 per unique access (note_access_locked
//    625-637, optional halving decay); refusal when the request's experts plus
//    the pins it does not use exceed the capacity; one slot per unique miss
//    (alloc_slot_locked 542-564: front free row, else the LFU victim,
//    choose_victim_locked 514-529, never a pinned expert or one of the
//    request); the (expert, slot) placements are returned for the caller to
//    load;
//  - real_pin (364-394).
// The host state machine runs under one mutex per manager. Loading is
// vb_pool_fill: one cudaMemcpyAsync per expert into a blob pool (contiguous
// rows), else one per tensor, from host or device memory laid out like
// prep/blob_layout.py:14-32. vb_blob_gather is the device gather of whole
// expert blobs by id (blob_mmap_gather_u4, native/ext/io/blob_load.cpp:
// 185-196).
#include <deque>
#include <mutex>
#include <unordered_map>
#include <unordered_set>
#include <vector>

#include "common.cuh"

namespace vb {
namespace {

struct ResLayer {
  int cap = 0;
  std::vector<int> order;                 // resident experts, insertion order
  std::unordered_map<int, int> e2r;       // expert -> slot
  std::deque<int> free_rows;              // free slots, front first
  std::unordered_map<int, uint32_t> freq; // LFU counts (kept across evictions)
  std::unordered_set<int> pinned;
  long access = 0;
  std::vector<int32_t> table;             // expert -> slot, -1 = not resident
};

}  // namespace
}  // namespace vb

struct VbResidency {
  int layers = 0, cap = 0, experts = 0, lfu = 1, decay = 0;
  std::vector<vb::ResLayer> L;
  std::mutex mu;
  // Staging of vb_moe_decode_resident, allocated on its first call (on the
  // device current then): pinned status + routed ids, per-layer pinned gather
  // indices and tables, device gather indices.
  int32_t *h_back = nullptr, *h_idx = nullptr, *h_table = nullptr, *d_idx = nullptr;
  ~VbResidency() {
    if (h_back) cudaFreeHost(h_back);
    if (h_idx) cudaFreeHost(h_idx);
    if (h_table) cudaFreeHost(h_table);
    if (d_idx) cudaFree(d_idx);
  }
};

namespace vb {
namespace {

int choose_victim(const ResLayer &c, const std::unordered_set<int> &current) {
  int victim = -1;
  uint32_t best = 0;
  for (int e : c.order) {
    if (!c.e2r.count(e) || c.pinned.count(e) || current.count(e)) continue;
    const auto f = c.freq.find(e);
    const uint32_t fv = f == c.freq.end() ? 0u : f->second;
    if (victim < 0 || fv < best) {
      victim = e;
      best = fv;
    }
  }
  return victim;
}

int alloc_slot(ResLayer &c, int e, const std::unordered_set<int> &current) {
  const auto it = c.e2r.find(e);
  if (it != c.e2r.end()) return it->second;
  int slot;
  if (!c.free_rows.empty()) {
    slot = c.free_rows.front();
    c.free_rows.pop_front();
  } else {
    const int v = choose_victim(c, current);
    if (v < 0) return -1;
    slot = c.e2r[v];
    c.e2r.erase(v);
    c.table[v] = -1;
    for (auto o = c.order.begin(); o != c.order.end(); ++o)
      if (*o == v) {
        c.order.erase(o);
        break;
      }
  }
  c.e2r[e] = slot;
  c.table[e] = slot;
  c.order.push_back(e);
  return slot;
}

void note_access(ResLayer &c, const std::vector<int> &uniq, bool lfu, int decay) {
  if (!lfu) return;
  for (int e : uniq) c.freq[e] += 1;
  c.access += static_cast<long>(uniq.size());
  if (decay > 0 && c.access >= decay) {
    for (auto it = c.freq.begin(); it != c.freq.end();) {
      it->second /= 2;
      if (it->second == 0) it = c.freq.erase(it);
      else ++it;
    }
    c.access = 0;
  }
}

// Segment bytes and offsets of one expert blob (gate, up, down x {w, s, b}).
void blob_segments(int H, int I, int group, int bits, size_t nb[9], size_t off[9], size_t *stride) {
  size_t o = 0;
  const int outs[3] = {I, I, H}, ins[3] = {H, H, I};
  for (int pj = 0; pj < 3; ++pj) {
    const size_t words = (size_t)ins[pj] * bits / 32, groups = (size_t)ins[pj] / group;
    const size_t sz[3] = {(size_t)outs[pj] * words * 4, (size_t)outs[pj] * groups * 2,
                          (size_t)outs[pj] * groups * 2};
    for (int k = 0; k < 3; ++k) {
      nb[3 * pj + k] = sz[k];
      off[3 * pj + k] = o;
      o += sz[k];
    }
  }
  *stride = o;
}

// out row rows[r] (or r) <- blob row experts[r]. blockIdx.y = r; each
// thread moves GATHER_UNROLL 16-byte vectors, all loads issued before the
// stores.
constexpr int GATHER_THREADS = 256, GATHER_UNROLL = 4;
__global__ void __launch_bounds__(GATHER_THREADS)
blob_gather_kernel(const uint4 *__restrict__ blob, const int32_t *__restrict__ experts,
                   const int32_t *__restrict__ rows, size_t vec_per_expert,
                   uint4 *__restrict__ out) {
  const int r = blockIdx.y;
  const uint4 *src = blob + (size_t)experts[r] * vec_per_expert;
  uint4 *dst = out + (size_t)(rows ? rows[r] : r) * vec_per_expert;
  const size_t base = (size_t)blockIdx.x * (GATHER_THREADS * GATHER_UNROLL) + threadIdx.x;
  uint4 v[GATHER_UNROLL];
#pragma unroll
  for (int u = 0; u < GATHER_UNROLL; ++u) {
    const size_t i = base + (size_t)u * GATHER_THREADS;
    if (i < vec_per_expert) v[u] = ldg_nc_v4(src + i);
  }
#pragma unroll
  for (int u = 0; u < GATHER_UNROLL; ++u) {
    const size_t i = base + (size_t)u * GATHER_THREADS;
    if (i < vec_per_expert) dst[i] = v[u];
  }
}

constexpr int RES_BACK_WORDS = 1 + 8 * 16;  // status + T*k routed ids (T <= 8, k <= 16)

int res_staging(VbResidency *r) {
  if (r->h_back) return VB_OK;
  const size_t idx = (size_t)r->layers * 2 * r->cap * sizeof(int32_t);
  const size_t tab = (size_t)r->layers * r->experts * sizeof(int32_t);
  cudaError_t e = cudaHostAlloc(&r->h_back, RES_BACK_WORDS * sizeof(int32_t), cudaHostAllocDefault);
  if (e == cudaSuccess) e = cudaHostAlloc(&r->h_idx, idx, cudaHostAllocDefault);
  if (e == cudaSuccess) e = cudaHostAlloc(&r->h_table, tab, cudaHostAllocDefault);
  if (e == cudaSuccess) e = cudaMalloc(&r->d_idx, idx);
  if (e != cudaSuccess) {
    if (r->h_back) cudaFreeHost(r->h_back);
    if (r->h_idx) cudaFreeHost(r->h_idx);
    if (r->h_table) cudaFreeHost(r->h_table);
    r->h_back = r->h_idx = r->h_table = r->d_idx = nullptr;
    return set_error(VB_ERR_CUDA, "residency staging: %s", cudaGetErrorString(e));
  }
  return VB_OK;
}

}  // namespace
}  // namespace vb

using namespace vb;

extern "C" {

VbResidency *vb_res_create(int32_t layers, int32_t cap, int32_t num_experts, int32_t lfu,
                           int32_t decay_interval) {
  if (layers <= 0 || cap <= 0 || num_experts <= 0 || decay_interval < 0) {
    set_error(VB_ERR_INVALID, "vb_res_create: layers=%d cap=%d experts=%d decay=%d", layers, cap,
              num_experts, decay_interval);
    return nullptr;
  }
  auto *r = new VbResidency;
  r->layers = layers;
  r->cap = cap;
  r->experts = num_experts;
  r->lfu = lfu ? 1 : 0;
  r->decay = decay_interval;
  r->L.resize(layers);
  for (auto &c : r->L) {
    c.cap = cap;
    for (int s = 0; s < cap; ++s) c.free_rows.push_back(s);
    c.table.assign(num_experts, -1);
  }
  return r;
}

void vb_res_destroy(VbResidency *r) { delete r; }

int vb_res_demand(VbResidency *r, int32_t layer, const int32_t *ids, int32_t n, int32_t *local,
                  int32_t *place_expert, int32_t *place_slot, int32_t *n_place, int64_t *stats) {
  VB_REQUIRE(r && layer >= 0 && layer < r->layers, "vb_res_demand: layer %d", layer);
  VB_REQUIRE(n >= 0 && (n == 0 || (ids && local)) && n_place, "vb_res_demand: null argument");
  for (int i = 0; i < n; ++i)
    VB_REQUIRE(ids[i] >= 0 && ids[i] < r->experts, "vb_res_demand: expert id %d", ids[i]);
  std::lock_guard<std::mutex> lk(r->mu);
  ResLayer &c = r->L[layer];
  std::vector<int> uniq_miss, access_order;
  std::unordered_set<int> miss_seen, access_seen, needed;
  long hits = 0;
  for (int i = 0; i < n; ++i) {
    const int e = ids[i];
    local[i] = -1;
    if (access_seen.insert(e).second) access_order.push_back(e);
    needed.insert(e);
    const auto it = c.e2r.find(e);
    if (it != c.e2r.end()) {
      local[i] = it->second;
      ++hits;
      continue;
    }
    if (miss_seen.insert(e).second) uniq_miss.push_back(e);
  }
  note_access(c, access_order, r->lfu != 0, r->decay);
  size_t unavailable_pins = 0;
  for (int e : c.pinned)
    if (!needed.count(e)) ++unavailable_pins;
  *n_place = 0;
  if (needed.size() + unavailable_pins > static_cast<size_t>(c.cap)) {
    for (int i = 0; i < n; ++i) local[i] = 0;
    if (stats) {
      stats[0] = hits;
      stats[1] = n - hits;
      stats[2] = 0;
    }
    return set_error(VB_ERR_CAPACITY,
                     "vb_res_demand: layer %d needs %zu experts (+%zu pinned) in %d slots", layer,
                     needed.size(), unavailable_pins, c.cap);
  }
  std::unordered_map<int, int> new_slot;
  for (int e : uniq_miss) {
    const int s = alloc_slot(c, e, needed);
    if (s < 0) return set_error(VB_ERR_CAPACITY, "vb_res_demand: no evictable slot");
    new_slot[e] = s;
    if (place_expert) place_expert[*n_place] = e;
    if (place_slot) place_slot[*n_place] = s;
    ++*n_place;
  }
  long misses = 0;
  for (int i = 0; i < n; ++i)
    if (local[i] < 0) {
      local[i] = new_slot[ids[i]];
      ++misses;
    }
  if (stats) {
    stats[0] = hits;
    stats[1] = misses;
    stats[2] = *n_place;
  }
  return VB_OK;
}

int vb_res_pin(VbResidency *r, int32_t layer, const int32_t *experts, int32_t n, int32_t *slots,
               int32_t *placed, int32_t *n_unique) {
  VB_REQUIRE(r && layer >= 0 && layer < r->layers, "vb_res_pin: layer %d", layer);
  VB_REQUIRE(n >= 0 && (n == 0 || (experts && slots && placed)) && n_unique,
             "vb_res_pin: null argument");
  for (int i = 0; i < n; ++i)
    VB_REQUIRE(experts[i] >= 0 && experts[i] < r->experts, "vb_res_pin: expert id %d", experts[i]);
  std::lock_guard<std::mutex> lk(r->mu);
  ResLayer &c = r->L[layer];
  std::vector<int> unique;
  std::unordered_set<int> requested;
  for (int i = 0; i < n; ++i)
    if (requested.insert(experts[i]).second) unique.push_back(experts[i]);
  std::unordered_set<int> combined = c.pinned;
  combined.insert(requested.begin(), requested.end());
  if (combined.size() > static_cast<size_t>(c.cap))
    return set_error(VB_ERR_CAPACITY, "vb_res_pin: %zu pinned experts > %d slots",
                     combined.size(), c.cap);
  c.pinned.insert(requested.begin(), requested.end());
  *n_unique = static_cast<int32_t>(unique.size());
  for (size_t u = 0; u < unique.size(); ++u) {
    const int e = unique[u];
    const auto it = c.e2r.find(e);
    if (it != c.e2r.end()) {
      slots[u] = it->second;
      placed[u] = 0;
      continue;
    }
    const int s = alloc_slot(c, e, requested);
    if (s < 0) return set_error(VB_ERR_CAPACITY, "vb_res_pin: no evictable slot");
    slots[u] = s;
    placed[u] = 1;
  }
  return VB_OK;
}

int vb_res_table(VbResidency *r, int32_t layer, int32_t *table) {
  VB_REQUIRE(r && layer >= 0 && layer < r->layers && table, "vb_res_table: layer %d", layer);
  std::lock_guard<std::mutex> lk(r->mu);
  const ResLayer &c = r->L[layer];
  std::copy(c.table.begin(), c.table.end(), table);
  return VB_OK;
}

int vb_res_counts(VbResidency *r, int32_t layer, uint32_t *counts) {
  VB_REQUIRE(r && layer >= 0 && layer < r->layers && counts, "vb_res_counts: layer %d", layer);
  std::lock_guard<std::mutex> lk(r->mu);
  const ResLayer &c = r->L[layer];
  std::fill(counts, counts + r->experts, 0u);
  for (const auto &kv : c.freq)
    if (kv.first >= 0 && kv.first < r->experts) counts[kv.first] = kv.second;
  return VB_OK;
}

int vb_res_resident(VbResidency *r, int32_t layer, int32_t *experts, int32_t *slots,
                    int32_t *n) {
  VB_REQUIRE(r && layer >= 0 && layer < r->layers && n, "vb_res_resident: layer %d", layer);
  std::lock_guard<std::mutex> lk(r->mu);
  const ResLayer &c = r->L[layer];
  int k = 0;
  for (int e : c.order) {
    const auto it = c.e2r.find(e);
    if (it == c.e2r.end()) continue;
    if (experts) experts[k] = e;
    if (slots) slots[k] = it->second;
    ++k;
  }
  *n = k;
  return VB_OK;
}

int vb_pool_fill(const VbQuantPool *pool, int32_t hidden, int32_t inter, int32_t group,
                 int32_t bits, const int32_t *slots, const void *const *blobs, int32_t n,
                 vb_stream_t stream) {
  VB_REQUIRE(pool && (n == 0 || (slots && blobs)) && n >= 0, "vb_pool_fill: null argument");
  VB_REQUIRE(hidden > 0 && inter > 0 && group > 0 && (bits == 2 || bits == 3 || bits == 4 ||
             bits == 5 || bits == 6 || bits == 8) && hidden % group == 0 && inter % group == 0 &&
             (hidden * bits) % 32 == 0 && (inter * bits) % 32 == 0,
             "vb_pool_fill: shape hidden=%d inter=%d group=%d bits=%d", hidden, inter, group, bits);
  size_t nb[9], off[9], stride;
  blob_segments(hidden, inter, group, bits, nb, off, &stride);
  // A blob pool keeps an expert's nine tensors contiguous: one copy per slot.
  bool contiguous = true;
  for (int t = 0; t < 9; ++t)
    contiguous = contiguous && pool->ptr[t] &&
                 static_cast<const uint8_t *>(pool->ptr[t]) ==
                     static_cast<const uint8_t *>(pool->ptr[0]) + off[t] &&
                 pool->slot_stride[t] == (int64_t)stride;
  cudaStream_t s = as_stream(stream);
  for (int i = 0; i < n; ++i) {
    VB_REQUIRE(slots[i] >= 0 && slots[i] < pool->cap && blobs[i], "vb_pool_fill: slot %d",
               slots[i]);
    const uint8_t *src = static_cast<const uint8_t *>(blobs[i]);
    cudaError_t e = cudaSuccess;
    if (contiguous) {
      e = cudaMemcpyAsync(const_cast<uint8_t *>(static_cast<const uint8_t *>(pool->ptr[0])) +
                              (size_t)slots[i] * stride,
                          src, stride, cudaMemcpyDefault, s);
    } else {
      for (int t = 0; t < 9 && e == cudaSuccess; ++t)
        e = cudaMemcpyAsync(const_cast<uint8_t *>(static_cast<const uint8_t *>(pool->ptr[t])) +
                                (size_t)slots[i] * pool->slot_stride[t],
                            src + off[t], nb[t], cudaMemcpyDefault, s);
    }
    if (e != cudaSuccess)
      return set_error(VB_ERR_CUDA, "vb_pool_fill: copy %d: %s", i, cudaGetErrorString(e));
  }
  return VB_OK;
}

int vb_blob_gather(const void *blob_store, int64_t blob_stride, const int32_t *experts,
                   const int32_t *out_rows, int32_t n, void *out, vb_stream_t stream) {
  VB_REQUIRE(blob_store && out && (n == 0 || experts) && n >= 0, "vb_blob_gather: null argument");
  VB_REQUIRE(blob_stride > 0 && blob_stride % 16 == 0 &&
                 ((uintptr_t)blob_store % 16) == 0 && ((uintptr_t)out % 16) == 0,
             "vb_blob_gather: stride %lld and pointers must be 16-byte multiples",
             (long long)blob_stride);
  VB_REQUIRE(n <= 65535, "vb_blob_gather: %d rows (at most 65535 per call)", n);
  if (n == 0) return VB_OK;
  const size_t vec = (size_t)blob_stride / 16;
  const size_t per_block = (size_t)GATHER_THREADS * GATHER_UNROLL;
  const dim3 grid((unsigned)((vec + per_block - 1) / per_block), (unsigned)n);
  blob_gather_kernel<<<grid, GATHER_THREADS, 0, as_stream(stream)>>>(
      static_cast<const uint4 *>(blob_store), experts, out_rows, vec, static_cast<uint4 *>(out));
  return check_launch("blob_gather_kernel");
}

int vb_moe_decode_resident(const VbMoeDecodeArgs *a, VbResidency *r, int32_t layer,
                           const void *blob_store, int64_t blob_stride, int32_t route_first,
                           int64_t *counts, vb_stream_t stream) {
  VB_REQUIRE(a && r && blob_store, "vb_moe_decode_resident: null argument");
  VB_REQUIRE(layer >= 0 && layer < r->layers, "vb_moe_decode_resident: layer %d", layer);
  VB_REQUIRE(a->out_inds && a->status && a->slot_table,
             "vb_moe_decode_resident: out_inds, status and slot_table are required");
  VB_REQUIRE(a->num_experts == r->experts && a->pool.cap == r->cap,
             "vb_moe_decode_resident: pool of %d slots / %d experts, manager has %d / %d",
             a->pool.cap, a->num_experts, r->cap, r->experts);
  VB_REQUIRE(a->flags == 0, "vb_moe_decode_resident: flags must be 0");
  const int n = a->tokens * a->top_k;
  VB_REQUIRE(n >= 1 && n + 1 <= RES_BACK_WORDS, "vb_moe_decode_resident: %d routes", n);
  size_t nb[9], off[9], stride;
  blob_segments(a->hidden, a->inter, a->group, a->bits, nb, off, &stride);
  VB_REQUIRE(blob_stride == (int64_t)stride && stride % 16 == 0,
             "vb_moe_decode_resident: blob stride %lld, layout needs %zu", (long long)blob_stride,
             stride);
  for (int t = 0; t < 9; ++t)
    VB_REQUIRE(static_cast<const uint8_t *>(a->pool.ptr[t]) ==
                       static_cast<const uint8_t *>(a->pool.ptr[0]) + off[t] &&
                   a->pool.slot_stride[t] == (int64_t)stride,
               "vb_moe_decode_resident: the pool must be one blob row per slot");
  int rc = res_staging(r);
  if (rc != VB_OK) return rc;
  cudaStream_t s = as_stream(stream);
  int32_t *back = r->h_back;
  int runs = 0;
  auto launch = [&](int32_t flags) -> int {
    cudaError_t e = cudaMemsetAsync(a->status, 0, sizeof(int32_t), s);
    if (e != cudaSuccess) return set_error(VB_ERR_CUDA, "status reset: %s", cudaGetErrorString(e));
    VbMoeDecodeArgs b = *a;
    b.flags = flags;
    ++runs;
    return vb_moe_decode(&b, stream);
  };
  // 1. route (route_first) or the whole block (optimistic), then one read-back
  rc = launch(route_first ? VB_DECODE_ROUTE_ONLY : 0);
  if (rc != VB_OK) return rc;
  cudaError_t e = cudaMemcpyAsync(back, a->status, sizeof(int32_t), cudaMemcpyDeviceToHost, s);
  if (e == cudaSuccess)
    e = cudaMemcpyAsync(back + 1, a->out_inds, n * sizeof(int32_t), cudaMemcpyDeviceToHost, s);
  if (e == cudaSuccess) e = cudaStreamSynchronize(s);
  if (e != cudaSuccess)
    return set_error(VB_ERR_CUDA, "vb_moe_decode_resident: read-back: %s", cudaGetErrorString(e));
  const int32_t st = back[0];
  if (st & ~VB_STATUS_MISS)
    return set_error(VB_ERR_CUDA, "vb_moe_decode_resident: layer %d status %#x", layer, st);
  // 2. demand: LFU note, slots for the misses
  int32_t local[8 * 16], pe[8 * 16], ps[8 * 16], n_place = 0;
  int64_t stats[3] = {0, 0, 0};
  rc = vb_res_demand(r, layer, back + 1, n, local, pe, ps, &n_place, stats);
  if (rc != VB_OK) return rc;
  if (!route_first && !(st & VB_STATUS_MISS) && n_place)
    return set_error(VB_ERR_INVALID, "vb_moe_decode_resident: device table out of step with the manager");
  // 3. load the placed experts and publish the layer's table
  if (n_place) {
    int32_t *hi = r->h_idx + (size_t)layer * 2 * r->cap, *di = r->d_idx + (size_t)layer * 2 * r->cap;
    for (int i = 0; i < n_place; ++i) {
      hi[i] = pe[i];
      hi[r->cap + i] = ps[i];
    }
    int32_t *ht = r->h_table + (size_t)layer * r->experts;
    rc = vb_res_table(r, layer, ht);
    if (rc != VB_OK) return rc;
    e = cudaMemcpyAsync(di, hi, 2 * r->cap * sizeof(int32_t), cudaMemcpyHostToDevice, s);
    if (e != cudaSuccess)
      return set_error(VB_ERR_CUDA, "vb_moe_decode_resident: index copy: %s", cudaGetErrorString(e));
    rc = vb_blob_gather(blob_store, blob_stride, di, di + r->cap, n_place,
                        const_cast<void *>(a->pool.ptr[0]), stream);
    if (rc != VB_OK) return rc;
    e = cudaMemcpyAsync(const_cast<int32_t *>(a->slot_table), ht, r->experts * sizeof(int32_t),
                        cudaMemcpyHostToDevice, s);
    if (e != cudaSuccess)
      return set_error(VB_ERR_CUDA, "vb_moe_decode_resident: table copy: %s", cudaGetErrorString(e));
  }
  // 4. the whole block once every routed expert has a slot
  if (route_first || (st & VB_STATUS_MISS)) {
    rc = launch(0);
    if (rc != VB_OK) return rc;
  }
  if (counts) {
    std::unordered_set<int> uniq(back + 1, back + 1 + n);
    counts[0] += (int64_t)uniq.size() - n_place;
    counts[1] += n_place;
    counts[2] += stats[0];
    counts[3] += runs;
  }
  return VB_OK;
}

}  // extern "C"
