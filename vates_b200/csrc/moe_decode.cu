// Decode / MTP-verify fused MoE block (T <= 8 tokens), MLX bf16 dtype chain.
//
// Reference: FileStreamingMoeBlock.__call__ (mlx_streaming/core/moe/block.py
// :245-1013) with PersistentSubGLU.forward (compute.py:145-199) and the
// shared expert (block.py:102-109, 1009-1012).
//
// One persistent kernel per block (one CTA of 16 warps per SM, all CTAs
// resident: a cooperative launch), a PDL secondary of whatever ran before it
// on the stream. Phases:
//  1. Before the PDL wait: every warp loads its part of one router row
//     (rows 0..E-1 the experts, row E the shared-expert gate) into
//     registers, and the shared expert (it needs no routing) is
//     bulk-prefetched into L2.
//  2. Every CTA stages x, applies the optional unit RMSNorm (exact double sum
//     of squares), keeps x in MMA-fragment order with its per-64-column sums
//     in shared memory, and computes its router rows: logits =
//     bf16(x.Wr^T [+bias]) and the gate sigmoid(x.w_sg), written to global
//     memory.
//  3. Grid barrier (bounded wait). Every CTA then runs the same precise
//     softmax, top-k, renormalisation and slot gather (one warp per token,
//     E/32 logits per lane in registers: maximum, exponential sum in double,
//     then k extractions of the largest (bf16 probability, expert id) key,
//     lower id winning ties), and builds the same list of "entries" in
//     shared memory: the shared expert first, then every distinct routed
//     expert in route order.
//  4. Gate/up: each CTA owns a contiguous range of items (entry, 16
//     intermediate rows); the four warps of a group split an item along the
//     hidden dimension and stream it through per-warp cp.async rings; 4-bit
//     codes become exact bf16 values 128+q for mma.m16n8k16 and the
//     per-group epilogue applies y += s*D + (b-128*s)*sum(x). The item's
//     leader adds the four partials (fixed order) and applies SwiGLU (bf16
//     per op); h goes to global memory in fragment order and the item is
//     counted on its entry (release).
//  5. Down: each CTA owns a contiguous range of items (entry, 16 output
//     rows) dealt round-robin to its warps, which stream the weights in two
//     chunks through their rings. The first warp to need an entry waits
//     (bounded, acquire) until its h is complete and stages h in shared
//     memory for the CTA. Per route the result is rounded to bf16, times the
//     route score, rounded again (MLX chain).
//  6. Combine: the warp completing a 16-row block (atomic ticket) adds the k
//     routes of every token in rank order (exact double sum of bf16 values,
//     rounded to float32 then bf16), then the gated shared expert and the
//     optional residual.
// Every wait is bounded (2 s); a wait that gives up sets VB_STATUS_TIMEOUT.
#include <algorithm>
#include <atomic>
#include <mutex>
#include <vector>

#include "common.cuh"

namespace vb {

constexpr int DEC_MAX_T = 8;
constexpr int DEC_MAX_K = 16;
constexpr int DEC_MAX_E = 1024;

struct DecEntry {
  int32_t slot;
  int32_t flags;  // bit0 = shared expert
  int32_t pad[2];
  int32_t rank[DEC_MAX_T];  // route rank of token n, -1 = not routed here
  float score[DEC_MAX_T];   // bf16 route score
};

struct DecodeLayout {
  size_t bar, sgate, ent_done, rb_count, zero_end, logits, hperm, hsum, wparts, sparts, total;
  int max_entries;
};

static DecodeLayout decode_layout(int T, int H, int I, int E, int k) {
  DecodeLayout L;
  L.max_entries = T * k + 1;
  size_t off = 0;
  L.bar = off; off += 16;  // grid barrier: 64-bit arrival count
  L.sgate = off; off += sizeof(float) * DEC_MAX_T;
  off = align_up(off, 16);
  // Tickets before the entry counters: their place depends only on H, and
  // every launch zeroes its own entry counters, so calls with different T
  // (same H) can share one workspace.
  off = align_up(off, 128);
  L.rb_count = off; off += 128 * (size_t)(H / 16);       // one 128-byte line per counter
  L.ent_done = off; off += 128 * (size_t)L.max_entries;
  L.zero_end = off;  // [0, zero_end) must be zero before the first call
  off = align_up(off, 256);
  L.logits = off; off += sizeof(float) * (size_t)T * E;
  off = align_up(off, 256);
  L.hperm = off; off += sizeof(uint32_t) * (size_t)L.max_entries * DEC_MAX_T * (I / 2);
  off = align_up(off, 256);
  L.hsum = off; off += sizeof(float) * (size_t)L.max_entries * DEC_MAX_T * (I / 16);
  off = align_up(off, 256);
  L.wparts = off; off += sizeof(uint16_t) * (size_t)T * k * H;
  off = align_up(off, 256);
  L.sparts = off; off += sizeof(uint16_t) * (size_t)T * H;
  L.total = align_up(off, 256);
  return L;
}

struct DecodeParams {
  int T, H, I, E, k, norm_topk, gshift, has_shared, route_only;
  float norm_eps;
  const uint16_t *x, *router_w, *shared_gate_w, *residual;
  const float *router_bias;
  const int32_t *table;
  VbQuantPool pool, shared;
  uint16_t *out, *out_scores;
  int32_t *out_inds, *out_local, *status;
  uint8_t *ws;
  uint64_t *trace;
  DecodeLayout L;
};

__device__ __forceinline__ uint64_t globaltimer() {
  uint64_t t;
  asm volatile("mov.u64 %0, %globaltimer;" : "=l"(t));
  return t;
}

// Optional trace: thread 0 of every CTA folds its start/end into the
// kernel's [min start, max end] pair (slots 0, 1).
struct SpanTrace {
  uint64_t *slot;
  uint64_t t0;
  __device__ __forceinline__ explicit SpanTrace(uint64_t *trace) {
    slot = (trace && threadIdx.x == 0) ? trace : nullptr;
    t0 = slot ? globaltimer() : 0;
  }
  __device__ __forceinline__ void end() {
    if (slot) {
      atomicMin(reinterpret_cast<unsigned long long *>(slot), (unsigned long long)t0);
      atomicMax(reinterpret_cast<unsigned long long *>(slot + 1),
                (unsigned long long)globaltimer());
    }
  }
};

// Optional marker: latest %globaltimer over the CTAs that pass this point.
__device__ __forceinline__ void trace_mark(uint64_t *trace, int idx) {
  if (trace && threadIdx.x == 0)
    atomicMax(reinterpret_cast<unsigned long long *>(trace + idx),
              (unsigned long long)globaltimer());
}

template <typename T>
__device__ __forceinline__ T *wsp(const DecodeParams &p, size_t off) {
  return reinterpret_cast<T *>(p.ws + off);
}

// Bytes of tensor t (gate w,s,b, up w,s,b, down w,s,b) of one 4-bit expert.
__device__ __forceinline__ uint32_t expert_tensor_bytes(const DecodeParams &p, int t) {
  const int f = t % 3;
  const uint32_t rows = t < 6 ? (uint32_t)p.I : (uint32_t)p.H;
  const uint32_t cols = t < 6 ? (uint32_t)p.H : (uint32_t)p.I;
  return f == 0 ? rows * (cols / 2) : rows * (cols >> (6 + p.gshift)) * 2u;
}

constexpr uint32_t PF_PIECE = 16u << 10;

// An expert as a sequence of 16 KB pieces (tensor by tensor): the count, and
// an L2 bulk prefetch of one piece.
__device__ __forceinline__ int expert_pieces(const DecodeParams &p) {
  int n = 0;
  for (int t = 0; t < 9; ++t) n += (expert_tensor_bytes(p, t) + PF_PIECE - 1) / PF_PIECE;
  return n;
}
__device__ __forceinline__ void prefetch_expert_piece(const DecodeParams &p, const VbQuantPool &pool,
                                                      int slot, int piece) {
  for (int t = 0; t < 9; ++t) {
    const uint32_t tb = expert_tensor_bytes(p, t);
    const int c = (tb + PF_PIECE - 1) / PF_PIECE;
    if (piece < c) {
      const uint32_t off = (uint32_t)piece * PF_PIECE;
      prefetch_l2_bulk(pool_ptr(pool, t, slot) + off, min(PF_PIECE, tb - off));
      return;
    }
    piece -= c;
  }
}

__device__ __forceinline__ uint2 lds64(const uint8_t *p) {
  return *reinterpret_cast<const uint2 *>(p);
}
__device__ __forceinline__ float bf_lo(uint32_t w) { return __uint_as_float(w << 16); }
__device__ __forceinline__ float bf_hi(uint32_t w) { return __uint_as_float(w & 0xFFFF0000u); }
// bf16 at index i (0..3) of a 2-word vector.
__device__ __forceinline__ float bf_at2(const uint2 &v, int i) {
  const uint32_t w = i < 2 ? v.x : v.y;
  return (i & 1) ? bf_hi(w) : bf_lo(w);
}

// Orderable key of a float (for unsigned max).
__device__ __forceinline__ uint32_t f2key(float f) {
  const uint32_t b = __float_as_uint(f);
  return (b & 0x80000000u) ? ~b : (b | 0x80000000u);
}
__device__ __forceinline__ float key2f(uint32_t k) {
  return __uint_as_float((k & 0x80000000u) ? (k & 0x7fffffffu) : ~k);
}

__device__ __forceinline__ void named_bar(int id, int threads) {
  asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(threads) : "memory");
}

__device__ __forceinline__ unsigned ld_acquire(const unsigned *p) {
  unsigned v;
  asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}
__device__ __forceinline__ unsigned long long ld_acquire64(const unsigned long long *p) {
  unsigned long long v;
  asm volatile("ld.acquire.gpu.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
  return v;
}
__device__ __forceinline__ unsigned atom_add_acq_rel(unsigned *p, unsigned v) {
  unsigned old;
  asm volatile("atom.acq_rel.gpu.global.add.u32 %0, [%1], %2;" : "=r"(old) : "l"(p), "r"(v) : "memory");
  return old;
}

// Sums a[0..7] over the lanes of a warp (4 + 2 + 1 + 1 + 1 shuffles): every
// round a lane keeps half of its values and receives the partner's copy of
// them. On return lanes 4t..4t+3 hold the total of value t in a[0] (a fixed
// order, the same in every lane of the group).
template <typename F>
__device__ __forceinline__ void warp_sum8(F (&a)[8], int lane) {
#pragma unroll
  for (int w = 4, o = 16; w >= 1; w >>= 1, o >>= 1) {
    const bool up = lane & o;
#pragma unroll
    for (int j = 0; j < w; ++j) {
      const F keep = up ? a[j + w] : a[j], send = up ? a[j] : a[j + w];
      a[j] = keep + __shfl_xor_sync(0xffffffffu, send, o);
    }
  }
  a[0] += __shfl_xor_sync(0xffffffffu, a[0], 2);
  a[0] += __shfl_xor_sync(0xffffffffu, a[0], 1);
}

__device__ __forceinline__ void red_release_add(unsigned *p, unsigned v) {
  asm volatile("red.release.gpu.global.add.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

constexpr uint64_t KL_WAIT_NS = 2000000000ull;  // bound of every wait

// Waits (acquire) until *p >= v; false after the bound.
__device__ __forceinline__ bool wait_ge(const unsigned *p, unsigned v) {
  const uint64_t t0 = globaltimer();
  for (;;) {
    if (ld_acquire(p) >= v) return true;
    if (globaltimer() - t0 > KL_WAIT_NS) return false;
    __nanosleep(256);
  }
}
__device__ __forceinline__ bool wait_ge64(const unsigned long long *p, unsigned long long v) {
  const uint64_t t0 = globaltimer();
  for (;;) {
    if (ld_acquire64(p) >= v) return true;
    if (globaltimer() - t0 > KL_WAIT_NS) return false;
    __nanosleep(64);
  }
}

// ----------------------------------------------------------------------------
// Tiles and the shared-memory map of the layer kernel.
// ----------------------------------------------------------------------------
constexpr int KL_THREADS = 512;
constexpr int KL_WARPS = KL_THREADS / 32;
constexpr int KL_MAX_ENT = DEC_MAX_T * DEC_MAX_K + 1;
constexpr int KL_MAX_ROUTES = DEC_MAX_T * DEC_MAX_K;
// Inter-CTA counters (entry completion, row-block tickets) sit one per
// 128-byte line (32 words apart), so that polls and atomics on different
// counters do not queue at one L2 line.
constexpr int KL_CSTRIDE = 32;
// Gate/up: an item (entry, 16 intermediate rows) is split along the hidden
// dimension over the GU_S warps of a group; their partial sums meet in
// shared memory and the item's leader applies SwiGLU.
constexpr int GU_S = 4;
constexpr int GU_NGRP = KL_WARPS / GU_S;
// Down: the entries whose h a CTA stages in shared memory (its down items
// are one contiguous range shorter than an entry's 2048 / 16 row blocks, so
// they span at most two entries).
constexpr int KL_HSLOTS = 2;

constexpr int align_c(int x, int a) { return (x + a - 1) / a * a; }

constexpr int KL_SMEM_MAX = 227 * 1024;

// 16-byte unit u of row r of a staged tile lives at unit swz<U>(r, u): the
// four rows g = 0..3 that one half-warp reads with 8-byte fragment loads
// (units 2G and 2G+1 of each row) then fall on distinct banks. U = units per
// row (rows of 32 bytes need no swizzle).
template <int U>
__device__ __forceinline__ int swz(int r, int u) {
  return U >= 8 ? u ^ ((r & 3) << 1) : (U == 4 ? u ^ (((r >> 1) & 1) << 1) : u);
}

template <int H, int I>
struct LayerTile {
  // Router: a row is split over Q warps, NVQ uint4 of the row part per lane.
  static constexpr int Q = H >= 2048 ? 4 : (H >= 1024 ? 2 : 1);
  static constexpr int RPC = KL_WARPS / Q;  // rows per CTA and round
  static constexpr int NVQ = H / (256 * Q);
  // Gate/up: chunks of CG groups of 64 columns of the item's 16 gate and 16
  // up rows; a warp streams the KP groups of its part of the hidden
  // dimension, CPW chunks per item.
  static constexpr int NG = H / 64;
  static constexpr int CG = 2;
  static constexpr int KP = NG / GU_S;
  static constexpr int CPW = KP / CG;
  static constexpr int ROWB = H / 2;         // packed bytes per row
  static constexpr int CROW = CG * 32;       // chunk bytes per row (4 units)
  static constexpr int NS64 = H / 64;        // scales per row at group 64
  static constexpr int WB = 2 * 16 * CROW;   // gate + up codes of a chunk
  static constexpr int CHUNK = WB + 4 * 16 * 4;  // + one scale word per tensor and row
  // Down: an item (entry, 16 output rows) in DCH chunks of DG groups; every
  // chunk also carries the item's whole 16-row scale/bias block.
  static constexpr int NGI = I / 64;
  static constexpr int DCH = NGI >= 2 ? 2 : 1;
  static constexpr int DG = NGI / DCH;
  static constexpr int DROWB = DG * 32;
  static constexpr int DWB = 16 * DROWB;
  static constexpr int DSB = 16 * NGI * 2;   // 16 rows of one scale tensor at group 64
  static constexpr int DSLOT = DWB + 2 * DSB;
  static constexpr int STAGE = align_c(CHUNK > DSLOT ? CHUNK : DSLOT, 128);
  // Shared memory: x fragments [NG][8][4][8] words, group sums [NG][8],
  // staged h [slot][8 tokens][NGI][4][8] words with group sums
  // [slot][NGI][8], item partials [2][warp][lane][8], entries, route flags,
  // a few words, then one ring per warp.
  static constexpr int XF = NG * DEC_MAX_T * 4 * 8 * 4;
  static constexpr int OFF_XS = XF;
  static constexpr int HF = DEC_MAX_T * NGI * 32 * 4;
  static constexpr int OFF_HF = OFF_XS + NG * DEC_MAX_T * 4;
  static constexpr int OFF_HSG = OFF_HF + KL_HSLOTS * HF;
  static constexpr int OFF_RED = align_c(OFF_HSG + KL_HSLOTS * NGI * DEC_MAX_T * 4, 128);
  static constexpr int OFF_ENT = OFF_RED + 2 * KL_WARPS * 32 * 8 * 4;
  static constexpr int OFF_OK = OFF_ENT + KL_MAX_ENT * (int)sizeof(DecEntry);
  static constexpr int OFF_MISC = OFF_OK + KL_MAX_ROUTES * 4;
  static constexpr int OFF_RING = align_c(OFF_MISC + 64, 128);
  static constexpr int RS0 = (KL_SMEM_MAX - OFF_RING) / (KL_WARPS * STAGE);
  static constexpr int RS = RS0 < 4 ? RS0 : 4;  // ring stages per warp
  static constexpr int RING = RS * STAGE;
  static constexpr int SMEM = OFF_RING + KL_WARPS * RING;
  // Router and routing temporaries, inside the rings (free until the
  // entries are built): x [8][H] bf16, slot table, first route of each
  // expert, routes (expert, slot, score, entry), reductions, candidates.
  static constexpr int TMP_TABLE = DEC_MAX_T * H * 2;
  static constexpr int TMP_FIRST = TMP_TABLE + DEC_MAX_E * 4;
  static constexpr int TMP_ROUTE = TMP_FIRST + DEC_MAX_E * 4;
  static constexpr int TMP_RED = TMP_ROUTE + 4 * KL_MAX_ROUTES * 4;
  static constexpr int TMP_PART = TMP_RED + KL_WARPS * DEC_MAX_T * 8;
  static constexpr int TMP_WMAX = TMP_PART + KL_WARPS * DEC_MAX_T * 4;
  static constexpr int TMP_WSUM = TMP_WMAX + KL_WARPS * 4;
  static constexpr int TMP_CAND = TMP_WSUM + KL_WARPS * 8;
  static constexpr int TMP_END = TMP_CAND + KL_WARPS * DEC_MAX_K * 4;
  static_assert(TMP_END <= KL_WARPS * RING, "router temporaries");
  static_assert(SMEM <= KL_SMEM_MAX, "layer kernel shared memory");
  static_assert(RS >= 2 && NVQ >= 1 && KP % CG == 0 && CPW >= 1 && DG >= 1, "layer tile");
  static_assert(KP % 2 == 0, "a chunk's scale word starts at an even group");
};

// The item's row block: gate and up codes, and the two scale tensors this
// lane loads scale words from (lanes 0-15: gate s and up s; lanes 16-31:
// gate b and up b). Only fixed fields, so the item stays in registers (a
// table of four scale pointers indexed by lane would live in local memory,
// and every chunk issue would wait for a local load first).
struct GateUpItem {
  const uint8_t *gw, *uw;
  const uint8_t *sg, *su;
};

template <int H, int I>
__device__ __forceinline__ void gateup_item(const VbQuantPool &pool, int slot, int rb, int gs,
                                            int lane, GateUpItem &it) {
  using Tl = LayerTile<H, I>;
  const size_t sb = (size_t)rb * 16 * (Tl::NS64 >> gs) * 2;
  const bool bias = lane >= 16;
  it.gw = pool_ptr(pool, 0, slot) + (size_t)rb * 16 * Tl::ROWB;
  it.uw = pool_ptr(pool, 3, slot) + (size_t)rb * 16 * Tl::ROWB;
  it.sg = pool_ptr(pool, bias ? 2 : 1, slot) + sb;
  it.su = pool_ptr(pool, bias ? 5 : 4, slot) + sb;
}

// First scale of the groups [g0, g0 + CG) of a gate/up chunk, rounded down
// to an even index: the 4-byte word holding the chunk's scales.
__device__ __forceinline__ int gu_scale_word(int g0, int gs) { return (g0 >> gs) & ~1; }

// Chunk (codes of groups [g0, g0 + CG) and their scale words) of an item
// into a ring stage: [2 matrices][16 rows][CROW] swizzled, then
// [4 tensors][16 rows] scale words.
template <int H, int I>
__device__ __forceinline__ void gateup_chunk(uint8_t *stage, const GateUpItem &it, int g0,
                                             int lane, int gs) {
  using Tl = LayerTile<H, I>;
  // 2 matrices x 16 rows x 4 units of 16 bytes: lane -> unit lane % 4 of
  // rows lane / 4 and lane / 4 + 8.
  const int r0 = lane >> 2, un = lane & 3;
  const size_t cb = (size_t)g0 * 32 + un * 16;
#pragma unroll
  for (int j = 0; j < 2; ++j) {
    const int r = r0 + 8 * j;
    uint8_t *d = stage + r * Tl::CROW + (swz<4>(r, un) << 4);
    cp_async16(d, it.gw + (size_t)r * Tl::ROWB + cb);
    cp_async16(d + 16 * Tl::CROW, it.uw + (size_t)r * Tl::ROWB + cb);
  }
  // Scale words: 4 tensors (gate s, gate b, up s, up b) x 16 rows, two per
  // lane: piece lane + 32 k is tensor (lane >> 4) + 2 k, row lane & 15.
  const int ns = Tl::NS64 >> gs, w0 = gu_scale_word(g0, gs), r = lane & 15;
  const size_t so = ((size_t)r * ns + w0) * 2;
  cp_async4(stage + Tl::WB + lane * 4, it.sg + so);
  cp_async4(stage + Tl::WB + (lane + 32) * 4, it.su + so);
}

// Chunk dc of down item (slot, 16-row block rb) into a ring stage:
// [16 rows][DROWB] codes (swizzled units), then the item's [16 rows][NSI]
// scales and biases.
template <int H, int I>
__device__ __forceinline__ void down_chunk(uint8_t *stage, const VbQuantPool &pool, int pslot,
                                           int rb, int dc, int lane, int gs) {
  using Tl = LayerTile<H, I>;
  const uint8_t *dw = pool_ptr(pool, 6, pslot) + (size_t)rb * 16 * (I / 2) + dc * Tl::DROWB;
  constexpr int CPR = Tl::DROWB / 16;  // 16-byte units per row
#pragma unroll
  for (int j = 0; j < (16 * CPR + 31) / 32; ++j) {
    const int q = lane + 32 * j, r = q / CPR, un = q % CPR;
    if (q < 16 * CPR)
      cp_async16(stage + r * Tl::DROWB + (swz<CPR>(r, un) << 4), dw + (size_t)r * (I / 2) + un * 16);
  }
  const int sb = 16 * (Tl::NGI >> gs) * 2, sch = sb / 16;
  for (int q = lane; q < 2 * sch; q += 32) {
    const int t = q / sch, cc = q % sch;
    cp_async16(stage + Tl::DWB + t * sb + cc * 16,
               pool_ptr(pool, 7 + t, pslot) + (size_t)rb * sb + cc * 16);
  }
}

// Rank-order combine of 8 rows of one 16-row block (rows 16 rb + 8 (lane & 1))
// for tokens t = ((lane >> 1) & 3) + 4 j: a warp combines four blocks at
// once (lane >> 3 picks the block). Every load of a pass is issued before
// the first add. ok: route flags [T][k] (shared memory).
__device__ __forceinline__ void down_combine_rows(const DecodeParams &p, const int32_t *ok,
                                                  int rb, int lane) {
  const int T = p.T, H = p.H, k = p.k;
  const uint16_t *wp = wsp<const uint16_t>(p, p.L.wparts);
  const int row = 16 * rb + 8 * (lane & 1);
#pragma unroll 1
  for (int t = (lane >> 1) & 3; t < T; t += 4) {
    uint4 v[DEC_MAX_K];
#pragma unroll
    for (int j = 0; j < DEC_MAX_K; ++j)
      if (j < k) v[j] = __ldcg(reinterpret_cast<const uint4 *>(wp + ((size_t)t * k + j) * H + row));
    const size_t oi = (size_t)t * H + row;
    float gate = 0.f;
    uint4 sw = make_uint4(0, 0, 0, 0), rr = sw;
    if (p.has_shared) {
      gate = __ldcg(wsp<const float>(p, p.L.sgate) + t);
      sw = __ldcg(reinterpret_cast<const uint4 *>(wsp<const uint16_t>(p, p.L.sparts) + oi));
    }
    if (p.residual) rr = __ldg(reinterpret_cast<const uint4 *>(p.residual + oi));
    double s[8];
#pragma unroll
    for (int q = 0; q < 8; ++q) s[q] = 0.0;
#pragma unroll
    for (int j = 0; j < DEC_MAX_K; ++j) {
      if (j < k && ok[t * k + j]) {
        const uint32_t w[4] = {v[j].x, v[j].y, v[j].z, v[j].w};
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          s[2 * q] += (double)bf2f(w[q] & 0xFFFFu);
          s[2 * q + 1] += (double)bf2f(w[q] >> 16);
        }
      }
    }
    const uint32_t sh[4] = {sw.x, sw.y, sw.z, sw.w};
    const uint32_t re[4] = {rr.x, rr.y, rr.z, rr.w};
    uint32_t o[4];
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      float y0 = rbf((float)s[2 * q]), y1 = rbf((float)s[2 * q + 1]);
      if (p.has_shared) {
        y0 = rbf(__fadd_rn(y0, rbf(__fmul_rn(gate, bf2f(sh[q] & 0xFFFFu)))));
        y1 = rbf(__fadd_rn(y1, rbf(__fmul_rn(gate, bf2f(sh[q] >> 16)))));
      }
      if (p.residual) {
        y0 = rbf(__fadd_rn(bf2f(re[q] & 0xFFFFu), y0));
        y1 = rbf(__fadd_rn(bf2f(re[q] >> 16), y1));
      }
      o[q] = (uint32_t)f2bf(y0) | ((uint32_t)f2bf(y1) << 16);
    }
    *reinterpret_cast<uint4 *>(p.out + oi) = make_uint4(o[0], o[1], o[2], o[3]);
  }
}


// Routing of all T tokens, run identically by every CTA of the layer kernel
// (all threads call it): precise softmax of the logits, top-k, optional
// renormalisation, slot gather, then the entry list. Token t is handled by
// warp t alone, PERW = E/32 logits per lane, warp-synchronously (no block
// barrier before the entry list): maximum, exponential sum (double, exact
// for the softmax's range, so independent of the order), then k extractions
// of the largest key. Keys are the bf16 probability bits above (0xFFFF -
// expert id), so the unsigned maximum is the largest probability with ties
// to the lower id. Results in shared memory (routes rex/rslot/rscore/rent,
// flags ok, entries ent); returns the number of entries. primary: this CTA
// also writes the optional outputs and the status bits.
template <int PERW>
__device__ __noinline__ int route_tokens(const float *logits, const int32_t *table, int T, int E,
                                         int k, int norm_topk, int has_shared, int cap,
                                         bool primary, int32_t *status, int32_t *out_inds,
                                         uint16_t *out_scores, int32_t *out_local,
                                         int *s_table, int *s_first, int *s_rex, int *s_rslot,
                                         float *s_rscore, int *s_rent, int32_t *s_ok,
                                         DecEntry *s_ent, int *s_wcnt, uint64_t *trace) {
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int t = warp;                 // token of this warp
  const bool act = t < T;
  // Slot table and logits are loaded together (one memory round trip).
  float v[PERW];
  {
    int tb[(DEC_MAX_E + KL_THREADS - 1) / KL_THREADS];
#pragma unroll
    for (int j = 0; j < (DEC_MAX_E + KL_THREADS - 1) / KL_THREADS; ++j) {
      const int i = tid + j * KL_THREADS;
      tb[j] = i < E ? __ldg(table + i) : -1;
    }
#pragma unroll
    for (int i = 0; i < PERW; ++i) {
      const int idx = lane + 32 * i;
      v[i] = (act && idx < E) ? __ldcg(logits + (size_t)t * E + idx) : -INFINITY;
    }
#pragma unroll
    for (int j = 0; j < (DEC_MAX_E + KL_THREADS - 1) / KL_THREADS; ++j) {
      const int i = tid + j * KL_THREADS;
      if (i < E) {
        s_table[i] = tb[j];
        s_first[i] = 0x7fffffff;
      }
    }
  }
  __syncthreads();  // slot table and first-route markers
  if (act) {
    uint32_t mk = 0;
#pragma unroll
    for (int i = 0; i < PERW; ++i) mk = max(mk, f2key(v[i]));
    const float m = key2f(__reduce_max_sync(0xffffffffu, mk));
    trace_mark(trace, 9);
    double sd[PERW];
#pragma unroll
    for (int i = 0; i < PERW; ++i) {
      const int idx = lane + 32 * i;
      const float ex = idx < E ? expf(__fsub_rn(v[i], m)) : 0.f;
      v[i] = ex;
      sd[i] = (double)ex;
    }
#pragma unroll
    for (int w = 1; w < PERW; w *= 2)
#pragma unroll
      for (int i = 0; i + w < PERW; i += 2 * w) sd[i] += sd[i + w];
    double st = sd[0];
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) st += __shfl_xor_sync(0xffffffffu, st, o);
    trace_mark(trace, 10);
    const float inv = __frcp_rn((float)st);
    uint32_t key[PERW], lb = 0;
#pragma unroll
    for (int i = 0; i < PERW; ++i) {
      const int idx = lane + 32 * i;
      key[i] = idx < E ? ((uint32_t)f2bf(__fmul_rn(v[i], inv)) << 16) | (0xFFFFu - idx) : 0u;
      lb = max(lb, key[i]);
    }
    // k extractions in descending key order; the selected probabilities are
    // summed in that order for the renormalisation
    double ssum = 0.0;
    uint32_t sel = 0;
    for (int r = 0; r < k; ++r) {
      const uint32_t best = __reduce_max_sync(0xffffffffu, lb);
      if (lb == best && best != 0u) {
        lb = 0;
#pragma unroll
        for (int i = 0; i < PERW; ++i) {
          if (key[i] == best) key[i] = 0u;
          lb = max(lb, key[i]);
        }
      }
      if (lane == r) sel = best;
      ssum += (double)bf2f(best >> 16);
    }
    trace_mark(trace, 11);
    const float sel_p = bf2f(sel >> 16);
    float score = sel_p;
    if (norm_topk) {
      const float denom = rbf((float)ssum);
      score = rbf(__fdiv_rn(sel_p, denom));
    }
    if (lane < k) {
      const int ex = 0xFFFF - (int)(sel & 0xFFFFu);
      int slot = -1;
      if (ex >= 0 && ex < E) {
        slot = s_table[ex];
        if (slot >= cap) {
          if (primary) flag_status(status, VB_STATUS_BOUNDS);
          slot = -1;
        } else if (slot < 0) {
          if (primary) flag_status(status, VB_STATUS_MISS);
          slot = -1;
        }
      } else if (primary) {
        flag_status(status, VB_STATUS_BOUNDS);
      }
      s_rex[t * k + lane] = ex;
      s_rslot[t * k + lane] = slot;
      s_rscore[t * k + lane] = score;
      s_ok[t * k + lane] = slot >= 0 ? 1 : 0;
      if (primary) {
        if (out_inds) out_inds[t * k + lane] = ex;
        if (out_scores) out_scores[t * k + lane] = f2bf(score);
        if (out_local) out_local[t * k + lane] = slot;
      }
    }
  }
  __syncthreads();
  trace_mark(trace, 12);

  // Entries: shared expert first, then one entry per distinct routed expert
  // in route order (t-major, rank-minor): the first route of each expert is
  // found with an atomic minimum, first routes are numbered with ballots,
  // and every route fills its (entry, token) cell.
  const int R = T * k;
  const int shared_n = has_shared ? 1 : 0;
  const int r = tid;
  const bool valid = r < R && s_rslot[r] >= 0;
  if (valid) atomicMin(&s_first[s_rex[r]], r);
  for (int i = tid; i < (R + 1) * (int)(sizeof(DecEntry) / 4); i += KL_THREADS) {
    const int f = i % (int)(sizeof(DecEntry) / 4);  // field word
    reinterpret_cast<int32_t *>(s_ent)[i] = (f >= 4 && f < 12) ? -1 : 0;
  }
  __syncthreads();
  const bool is_first = valid && s_first[s_rex[r]] == r;
  const unsigned bal = __ballot_sync(0xffffffffu, is_first);
  if (lane == 0) s_wcnt[warp] = __popc(bal);
  __syncthreads();
  if (is_first) {
    int idx = shared_n + __popc(bal & ((1u << lane) - 1u));
    for (int w = 0; w < warp; ++w) idx += s_wcnt[w];
    s_rent[r] = idx;
  }
  int n_routed = 0;
#pragma unroll
  for (int w = 0; w < KL_WARPS; ++w) n_routed += s_wcnt[w];
  __syncthreads();
  if (valid) {
    const int ei = s_rent[s_first[s_rex[r]]];
    const int tt = r / k, jj = r - tt * k;
    s_ent[ei].slot = s_rslot[r];
    s_ent[ei].rank[tt] = jj;
    s_ent[ei].score[tt] = s_rscore[r];
  }
  if (tid == 0 && has_shared) {
    s_ent[0].slot = 0;
    s_ent[0].flags = 1;
    for (int q = 0; q < T; ++q) {
      s_ent[0].rank[q] = 0;
      s_ent[0].score[q] = 1.f;
    }
  }
  __syncthreads();
  return shared_n + n_routed;
}

// ----------------------------------------------------------------------------
// The layer kernel. Trace slots (optional): 0/1 span; latest CTA past the
// PDL wait (2), done with its router rows (3), past the grid barrier (4),
// done with routing (5); latest warp done with gate/up (6), with its down
// items (7), with its combines (8); latest CTA past the routing steps: the
// maximum (9), the exponential sum (10), the per-warp candidates (11), the
// top-k (12).
// ----------------------------------------------------------------------------
template <int H, int I>
__global__ void __launch_bounds__(KL_THREADS, 1) moe_layer_kernel(DecodeParams p) {
  using Tl = LayerTile<H, I>;
  constexpr int Q = Tl::Q, RPC = Tl::RPC, NVQ = Tl::NVQ, NG = Tl::NG, CG = Tl::CG,
                KP = Tl::KP, CPW = Tl::CPW, RS = Tl::RS, NGI = Tl::NGI, DCH = Tl::DCH,
                DG = Tl::DG;
  constexpr int RB = I / 16;    // gate/up items per entry
  constexpr int RBN = H / 16;   // down items per entry
  extern __shared__ __align__(128) uint8_t smem[];
  uint32_t *xf = reinterpret_cast<uint32_t *>(smem);  // [NG][8][4][8] words
  float *xsm = reinterpret_cast<float *>(smem + Tl::OFF_XS);  // [NG][8]
  uint32_t *hf = reinterpret_cast<uint32_t *>(smem + Tl::OFF_HF);  // [slot][8][NGI][4][8]
  float *hsg = reinterpret_cast<float *>(smem + Tl::OFF_HSG);      // [slot][NGI][8]
  DecEntry *s_ent = reinterpret_cast<DecEntry *>(smem + Tl::OFF_ENT);
  int32_t *s_ok = reinterpret_cast<int32_t *>(smem + Tl::OFF_OK);
  int *s_misc = reinterpret_cast<int *>(smem + Tl::OFF_MISC);  // [0] entries, [1] abort, [4..] h slot flags
  uint8_t *rings = smem + Tl::OFF_RING;
  uint16_t *xb = reinterpret_cast<uint16_t *>(rings);  // [T][H] bf16 (router phase)
  double *s_dred = reinterpret_cast<double *>(rings + Tl::TMP_RED);
  float *s_part = reinterpret_cast<float *>(rings + Tl::TMP_PART);
  __shared__ int s_wcnt[KL_WARPS];
  __shared__ unsigned long long s_tm[3];

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int g = lane >> 2, c = lane & 3;
  const int T = p.T, E = p.E, gs = p.gshift;
  const int G = gridDim.x;
  SpanTrace span(p.trace);

  // ---------------- 1. before the PDL wait ----------------
  const int nrows = E + p.has_shared;
  const int rloc = warp / Q, part = warp % Q;
  uint4 wv[NVQ];
  auto load_row = [&](int row) {
    const uint16_t *src = row < E ? p.router_w + (size_t)row * H : p.shared_gate_w;
    const uint4 *w4 = reinterpret_cast<const uint4 *>(src + part * (H / Q));
#pragma unroll
    for (int u = 0; u < NVQ; ++u) wv[u] = ldg_nc_v4(w4 + u * 32 + lane);
  };
  if (blockIdx.x * RPC + rloc < nrows) load_row(blockIdx.x * RPC + rloc);
  if (blockIdx.x == 0 && tid * 32 < E) prefetch_l2(p.table + tid * 32);
  if (p.has_shared && lane == 0) {
    const int piece = blockIdx.x * KL_WARPS + warp;
    if (piece < expert_pieces(p)) prefetch_expert_piece(p, p.shared, 0, piece);
  }
  if (tid < 3) s_tm[tid] = 0ull;
  if (tid < KL_HSLOTS) s_misc[4 + tid] = 0;
  pdl_wait();
  pdl_launch_dependents();
  trace_mark(p.trace, 2);

  // ---------------- 2. x, RMSNorm, fragments, router rows ----------------
  {
    const uint4 *src = reinterpret_cast<const uint4 *>(p.x);
    uint4 *dst = reinterpret_cast<uint4 *>(xb);
    constexpr int PT = (DEC_MAX_T * H / 8 + KL_THREADS - 1) / KL_THREADS;
    const int nvec = T * (H / 8);
    uint4 v[PT];
#pragma unroll
    for (int u = 0; u < PT; ++u) {
      const int i = u * KL_THREADS + tid;
      if (i < nvec) v[u] = __ldcg(src + i);
    }
#pragma unroll
    for (int u = 0; u < PT; ++u) {
      const int i = u * KL_THREADS + tid;
      if (i < nvec) dst[i] = v[u];
    }
  }
  if (blockIdx.x == 0)  // entry counters of this launch (all counting follows the grid barrier)
    for (int i = tid; i < p.L.max_entries; i += KL_THREADS)
      wsp<unsigned>(p, p.L.ent_done)[i * KL_CSTRIDE] = 0u;
  for (int i = tid; i < NG * DEC_MAX_T; i += KL_THREADS)
    if ((i & 7) >= T) xsm[i] = 0.f;  // group sums beyond T
  __syncthreads();
  // Unit-weight RMSNorm of the block input (decoder post-attention norm):
  // y = bf16(x * (1/sqrt(mean(x^2) + eps))), float32 math with an exact
  // (double) sum of squares: squares of bf16 values have 16 significant
  // bits, so their double sum does not depend on the order. Every warp
  // derives the factors itself (lane t for token t).
  const bool norm = p.norm_eps > 0.f;
  float inv_lane = 1.f;
  if (norm) {
    constexpr int VPT = H / 8;  // uint4 per token
    double ss[DEC_MAX_T];
#pragma unroll
    for (int t = 0; t < DEC_MAX_T; ++t) ss[t] = 0.0;
    for (int v = tid; v < VPT; v += KL_THREADS) {
#pragma unroll
      for (int t = 0; t < DEC_MAX_T; ++t) {
        if (t < T) {
          const uint4 q = reinterpret_cast<const uint4 *>(xb + (size_t)t * H)[v];
          const uint32_t w[4] = {q.x, q.y, q.z, q.w};
#pragma unroll
          for (int j = 0; j < 4; ++j) {
            const double a = bf2f(w[j] & 0xFFFF), b = bf2f(w[j] >> 16);
            ss[t] = fma(a, a, ss[t]);
            ss[t] = fma(b, b, ss[t]);
          }
        }
      }
    }
    warp_sum8(ss, lane);
    if ((lane & 3) == 0) s_dred[warp * DEC_MAX_T + (lane >> 2)] = ss[0];
    __syncthreads();
    if (lane < T) {
      double tot = 0.0;
#pragma unroll
      for (int w = 0; w < KL_WARPS; ++w) tot += s_dred[w * DEC_MAX_T + lane];
      const float ms = __fdiv_rn((float)tot, (float)H);
      inv_lane = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(ms, p.norm_eps)));
    }
  }
  {
    // One pass over x (8 columns per thread and step): normalise in place,
    // write the MMA fragment words and the per-64-column sums. Fragment
    // word (G, n, c, w) = x[n][base], x[n][base + 4] with base = 64G + 16c
    // + 8(w/4) + 2((w/2)&1) + (w&1): the 8 columns 8v..8v+7 (v = 8G + 2c +
    // j) give words 4j..4j+3 of (G, n, c). The 8 threads of a 64-column
    // group add their sums with three shuffles.
    constexpr int VPT = H / 8;
    for (int i = tid; i < T * VPT; i += KL_THREADS) {  // warp-uniform bound (VPT % 32 == 0)
      const int n = i / VPT, v = i % VPT;
      const float inv = __shfl_sync(0xffffffffu, inv_lane, n);
      const uint4 q = reinterpret_cast<const uint4 *>(xb)[i];
      const uint32_t w[4] = {q.x, q.y, q.z, q.w};
      float f[8];
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        f[2 * j] = bf2f(w[j] & 0xFFFF);
        f[2 * j + 1] = bf2f(w[j] >> 16);
      }
      if (norm) {
#pragma unroll
        for (int j = 0; j < 8; ++j) f[j] = rbf(__fmul_rn(f[j], inv));
        reinterpret_cast<uint4 *>(xb)[i] = make_uint4(pack_bf2(f[0], f[1]), pack_bf2(f[2], f[3]),
                                                      pack_bf2(f[4], f[5]), pack_bf2(f[6], f[7]));
      }
      const int Gi = v >> 3, cc = (v >> 1) & 3, j = v & 1;
      reinterpret_cast<uint4 *>(xf + ((Gi * DEC_MAX_T + n) * 4 + cc) * 8 + 4 * j)[0] =
          make_uint4(pack_bf2(f[0], f[4]), pack_bf2(f[1], f[5]), pack_bf2(f[2], f[6]),
                     pack_bf2(f[3], f[7]));
      float gsum = ((f[0] + f[1]) + (f[2] + f[3])) + ((f[4] + f[5]) + (f[6] + f[7]));
      gsum += __shfl_xor_sync(0xffffffffu, gsum, 4);
      gsum += __shfl_xor_sync(0xffffffffu, gsum, 2);
      gsum += __shfl_xor_sync(0xffffffffu, gsum, 1);
      if ((v & 7) == 0) xsm[Gi * DEC_MAX_T + n] = gsum;
    }
  }
  __syncthreads();
  // Router rows: this CTA's rows (blockIdx.x + G * round) * RPC + rloc.
  for (int round = 0;; ++round) {
    const int rb0 = (blockIdx.x + G * round) * RPC;
    if (rb0 >= nrows) break;
    const int row = rb0 + rloc;
    if (round > 0 && row < nrows) load_row(row);
    if (row < nrows) {
      float acc[DEC_MAX_T];
#pragma unroll
      for (int t = 0; t < DEC_MAX_T; ++t) acc[t] = 0.f;
#pragma unroll
      for (int u = 0; u < NVQ; ++u) {
        const int v = part * (H / Q / 8) + u * 32 + lane;
        const uint32_t wr[4] = {wv[u].x, wv[u].y, wv[u].z, wv[u].w};
#pragma unroll
        for (int t = 0; t < DEC_MAX_T; ++t) {
          if (t < T) {
            const uint4 xv = reinterpret_cast<const uint4 *>(xb + (size_t)t * H)[v];
            const uint32_t xr[4] = {xv.x, xv.y, xv.z, xv.w};
            float a = acc[t];
#pragma unroll
            for (int q = 0; q < 4; ++q) {
              a = fmaf(bf2f(wr[q] & 0xFFFF), bf2f(xr[q] & 0xFFFF), a);
              a = fmaf(bf2f(wr[q] >> 16), bf2f(xr[q] >> 16), a);
            }
            acc[t] = a;
          }
        }
      }
      warp_sum8(acc, lane);
      if ((lane & 3) == 0) s_part[(rloc * Q + part) * DEC_MAX_T + (lane >> 2)] = acc[0];
    }
    __syncthreads();
    if (tid < RPC * DEC_MAX_T) {
      const int rl = tid / DEC_MAX_T, t = tid % DEC_MAX_T;
      const int r = rb0 + rl;
      if (r < nrows && t < T) {
        float a = 0.f;
#pragma unroll
        for (int q = 0; q < Q; ++q) a += s_part[(rl * Q + q) * DEC_MAX_T + t];
        if (r < E) {
          if (p.router_bias) a = a + p.router_bias[r];
          wsp<float>(p, p.L.logits)[(size_t)t * E + r] = rbf(a);
        } else {
          wsp<float>(p, p.L.sgate)[t] = rbf(mlx_sigmoid(rbf(a)));
        }
      }
    }
    __syncthreads();
  }
  trace_mark(p.trace, 3);

  // ---------------- 3. grid barrier, routing ----------------
  if (tid == 0) {
    // Arrivals only ever grow (by G per launch, the grid size being fixed per
    // device): this launch's CTAs see old in [n G, (n + 1) G) and wait for
    // (n + 1) G.
    unsigned long long *bar = wsp<unsigned long long>(p, p.L.bar);
    __threadfence();
    const unsigned long long old = atomicAdd(bar, 1ull);
    const bool ok = wait_ge64(bar, (old / G + 1) * G);
    __threadfence();
    if (!ok) flag_status(p.status, VB_STATUS_TIMEOUT);
    s_misc[1] = ok ? 0 : 1;
  }
  __syncthreads();
  if (s_misc[1]) {
    span.end();
    return;
  }
  trace_mark(p.trace, 4);
  {
    int *s_table = reinterpret_cast<int *>(rings + Tl::TMP_TABLE);
    int *s_first = reinterpret_cast<int *>(rings + Tl::TMP_FIRST);
    int *s_rex = reinterpret_cast<int *>(rings + Tl::TMP_ROUTE);
    int *s_rslot = s_rex + KL_MAX_ROUTES;
    float *s_rscore = reinterpret_cast<float *>(s_rslot + KL_MAX_ROUTES);
    int *s_rent = reinterpret_cast<int *>(s_rscore + KL_MAX_ROUTES);
    const float *lg = wsp<const float>(p, p.L.logits);
    const bool primary = blockIdx.x == 0;
    const int need = (E + 31) / 32;  // logits per lane (one warp per token)
    int n;
#define VB_ROUTE(PERW)                                                                         \
  route_tokens<PERW>(lg, p.table, T, E, p.k, p.norm_topk, p.has_shared, p.pool.cap, primary,  \
                     p.status, p.out_inds, p.out_scores, p.out_local, s_table, s_first, s_rex, \
                     s_rslot, s_rscore, s_rent, s_ok, s_ent, s_wcnt, p.trace)
    if (need <= 4) n = VB_ROUTE(4);
    else if (need <= 8) n = VB_ROUTE(8);
    else if (need <= 16) n = VB_ROUTE(16);
    else n = VB_ROUTE(32);
#undef VB_ROUTE
    if (tid == 0) s_misc[0] = n;
  }
  __syncthreads();  // the rings are free from here on
  trace_mark(p.trace, 5);
  if (p.route_only) {  // routing outputs written; no counter touched yet
    span.end();
    return;
  }
  const int n_ent = s_misc[0];

  // ---------------- 4. gate/up + SwiGLU ----------------
  uint8_t *ring = rings + warp * Tl::RING;
  float *red = reinterpret_cast<float *>(smem + Tl::OFF_RED);  // [2][warp][lane][8]
  unsigned *ent_done = wsp<unsigned>(p, p.L.ent_done);
  // Each warp runs one sequence of jobs through its ring: its gate/up
  // chunks, then its down chunks, so the down weights stream in as soon as
  // gate/up stages free up.
  // Gate/up: this CTA's items are the contiguous range [a0, a1) of
  // (entry, row block) pairs; group grp takes items a0 + grp + GU_NGRP r,
  // and warp wi of the group the groups [wi KP, (wi + 1) KP) of each.
  const int grp = warp / GU_S, wi = warp % GU_S;
  const int n_items = n_ent * RB;
  const int a0 = (int)(((long long)n_items * blockIdx.x) / G);
  const int a1 = (int)(((long long)n_items * (blockIdx.x + 1)) / G);
  const int my_items = a1 - a0 > grp ? (a1 - a0 - grp + GU_NGRP - 1) / GU_NGRP : 0;
  const int nq_gu = my_items * CPW;
  // Down: this CTA's items are the contiguous range [d0, d1) of (entry,
  // 16-row block) pairs, dealt round-robin over the warps.
  const int n_items_d = n_ent * RBN;
  const int d0 = (int)(((long long)n_items_d * blockIdx.x) / G);
  const int d1 = (int)(((long long)n_items_d * (blockIdx.x + 1)) / G);
  const int nj = d1 - d0 > warp ? (d1 - d0 - warp + KL_WARPS - 1) / KL_WARPS : 0;
  const int e_lo = d0 / RBN;
  int j_end = nj;
  GateUpItem cur;
  int issue_q = 0;
  const int nq = nq_gu + nj * DCH;
  auto issue_next = [&]() {
    uint8_t *stage = ring + (issue_q % RS) * Tl::STAGE;
    if (issue_q < nq_gu) {
      const int r = issue_q / CPW, ch = issue_q % CPW;
      const int i = a0 + grp + GU_NGRP * r;
      if (ch == 0) {
        const int e = i / RB;
        if (p.has_shared && e == 0) gateup_item<H, I>(p.shared, 0, i % RB, gs, lane, cur);
        else gateup_item<H, I>(p.pool, s_ent[e].slot, i % RB, gs, lane, cur);
      }
      gateup_chunk<H, I>(stage, cur, wi * KP + ch * CG, lane, gs);
    } else if (issue_q < nq) {
      const int jj = (issue_q - nq_gu) / DCH, dc = (issue_q - nq_gu) % DCH;
      const int i = d0 + warp + KL_WARPS * jj;
      const int e = i / RBN, rb = i % RBN;
      const bool sh = p.has_shared && e == 0;
      down_chunk<H, I>(stage, sh ? p.shared : p.pool, sh ? 0 : s_ent[e].slot, rb, dc, lane, gs);
    }
    cp_async_commit();
    ++issue_q;
  };
#pragma unroll 1
  for (int kq = 0; kq < RS - 1; ++kq) issue_next();
  {
    // Fragment offsets inside a staged chunk (rows g and g+8 share a swizzle).
    int fo[CG];
#pragma unroll
    for (int gl = 0; gl < CG; ++gl) fo[gl] = g * Tl::CROW + (swz<4>(g, 2 * gl + (c >> 1)) << 4) + (c & 1) * 8;
    float accg[4], accu[4];
#pragma unroll 1
    for (int q = 0; q < nq_gu; ++q) {
      const int r = q / CPW, ch = q % CPW;
      const int li = grp + GU_NGRP * r;  // item index inside this CTA's range
      cp_async_wait<RS - 2>();
      __syncwarp();
      issue_next();  // into the stage consumed one chunk ago
      if (ch == 0) {
#pragma unroll
        for (int j = 0; j < 4; ++j) accg[j] = accu[j] = 0.f;
      }
      const uint8_t *st = ring + (q % RS) * Tl::STAGE;
      const int g0 = wi * KP + ch * CG;
      const int w0 = gu_scale_word(g0, gs);
      // Scale words of rows g and g+8: gate s, gate b, up s, up b.
      uint32_t sv[8];
#pragma unroll
      for (int a = 0; a < 8; ++a)
        sv[a] = *reinterpret_cast<const uint32_t *>(st + Tl::WB + ((a >> 1) * 16 + ((a & 1) ? g + 8 : g)) * 4);
#pragma unroll
      for (int gl = 0; gl < CG; ++gl) {
        const int Gi = g0 + gl;
        uint4 x0 = make_uint4(0, 0, 0, 0), x1 = x0;
        if (g < T) {
          const uint4 *xp = reinterpret_cast<const uint4 *>(xf + ((Gi * DEC_MAX_T + g) * 4 + c) * 8);
          x0 = xp[0];
          x1 = xp[1];
        }
        const float2 xs = *reinterpret_cast<const float2 *>(xsm + Gi * DEC_MAX_T + 2 * c);
        const uint2 ag0 = lds64(st + fo[gl]);
        const uint2 ag1 = lds64(st + 8 * Tl::CROW + fo[gl]);
        const uint2 au0 = lds64(st + 16 * Tl::CROW + fo[gl]);
        const uint2 au1 = lds64(st + 24 * Tl::CROW + fo[gl]);
        uint32_t pg0[2][4], pg1[2][4], pu0[2][4], pu1[2][4];
        nib_pairs4(ag0.x, pg0[0]);
        nib_pairs4(ag0.y, pg0[1]);
        nib_pairs4(ag1.x, pg1[0]);
        nib_pairs4(ag1.y, pg1[1]);
        nib_pairs4(au0.x, pu0[0]);
        nib_pairs4(au0.y, pu0[1]);
        nib_pairs4(au1.x, pu1[0]);
        nib_pairs4(au1.y, pu1[1]);
        const uint32_t xw[8] = {x0.x, x0.y, x0.z, x0.w, x1.x, x1.y, x1.z, x1.w};
        float dg[4] = {0.f, 0.f, 0.f, 0.f}, du[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
        for (int m = 0; m < 4; ++m) {
          const int i0 = 2 * (m & 1), h = m >> 1;
          mma_bf16(dg, pg0[h][i0], pg1[h][i0], pg0[h][i0 + 1], pg1[h][i0 + 1], xw[2 * m],
                   xw[2 * m + 1]);
          mma_bf16(du, pu0[h][i0], pu1[h][i0], pu0[h][i0 + 1], pu1[h][i0 + 1], xw[2 * m],
                   xw[2 * m + 1]);
        }
        // The group's scale is half (Gi >> gs) - w0 of the chunk's word.
        const bool hi = ((Gi >> gs) - w0) != 0;
        auto sc = [&](uint32_t w) { return hi ? bf_hi(w) : bf_lo(w); };
        const float sg0 = sc(sv[0]), sg1 = sc(sv[1]), bg0 = sc(sv[2]), bg1 = sc(sv[3]);
        const float su0 = sc(sv[4]), su1 = sc(sv[5]), bu0 = sc(sv[6]), bu1 = sc(sv[7]);
        const float bpg0 = fmaf(-128.f, sg0, bg0), bpg1 = fmaf(-128.f, sg1, bg1);
        const float bpu0 = fmaf(-128.f, su0, bu0), bpu1 = fmaf(-128.f, su1, bu1);
        accg[0] = fmaf(bpg0, xs.x, fmaf(sg0, dg[0], accg[0]));
        accg[1] = fmaf(bpg0, xs.y, fmaf(sg0, dg[1], accg[1]));
        accg[2] = fmaf(bpg1, xs.x, fmaf(sg1, dg[2], accg[2]));
        accg[3] = fmaf(bpg1, xs.y, fmaf(sg1, dg[3], accg[3]));
        accu[0] = fmaf(bpu0, xs.x, fmaf(su0, du[0], accu[0]));
        accu[1] = fmaf(bpu0, xs.y, fmaf(su0, du[1], accu[1]));
        accu[2] = fmaf(bpu1, xs.x, fmaf(su1, du[2], accu[2]));
        accu[3] = fmaf(bpu1, xs.y, fmaf(su1, du[3], accu[3]));
      }
      if (ch == CPW - 1) {
        // Group hand-off: every warp's partials to the item's leader, which
        // adds them in warp order and applies SwiGLU.
        const int b = r & 1;
        float *mine = red + ((b * KL_WARPS + warp) * 32 + lane) * 8;
        *reinterpret_cast<float4 *>(mine) = make_float4(accg[0], accg[1], accg[2], accg[3]);
        *reinterpret_cast<float4 *>(mine + 4) = make_float4(accu[0], accu[1], accu[2], accu[3]);
        named_bar(1 + grp, GU_S * 32);
        if (wi == r % GU_S) {
          float sg[4] = {0.f, 0.f, 0.f, 0.f}, su[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
          for (int w = 0; w < GU_S; ++w) {
            const float *o = red + ((b * KL_WARPS + grp * GU_S + w) * 32 + lane) * 8;
            const float4 og = *reinterpret_cast<const float4 *>(o);
            const float4 ou = *reinterpret_cast<const float4 *>(o + 4);
            sg[0] += og.x; sg[1] += og.y; sg[2] += og.z; sg[3] += og.w;
            su[0] += ou.x; su[1] += ou.y; su[2] += ou.z; su[3] += ou.w;
          }
          // SwiGLU (bf16 per op) of rows g, g+8 x tokens 2c, 2c+1; h of the
          // 16 rows in fragment order (via shuffles) and its per-token sums.
          const int item = a0 + li;
          const int e = item / RB, rb = item % RB;
          float hv[4];
#pragma unroll
          for (int j = 0; j < 4; ++j) {
            const int n = 2 * c + (j & 1);
            hv[j] = n < T ? swiglu_bf16(rbf(sg[j]), rbf(su[j])) : 0.f;
          }
          // Lane (g, c) holds h[row g | g+8][token 2c | 2c+1]. Fragment word
          // w of token n = pack(h[olo][n], h[olo + 4][n]) with olo = 8j + i0
          // + pp (m = w / 2, pp = w & 1, j = m / 2, i0 = 2 (m & 1)); the
          // owner of h[row][n] is lane 4 (row & 7) + n / 2, value index
          // (row >= 8 ? 2 : 0) + (n & 1).
          uint32_t *hperm = wsp<uint32_t>(p, p.L.hperm);
#pragma unroll
          for (int h2 = 0; h2 < 2; ++h2) {
            const int idx = lane + 32 * h2;  // (token n, word w)
            const int n = idx >> 3, w = idx & 7;
            const int m = w >> 1, pp = w & 1, j = m >> 1, i0 = 2 * (m & 1);
            const int olo = 8 * j + i0 + pp, ohi = olo + 4;
            const int src_lo = 4 * (olo & 7) + (n >> 1), src_hi = 4 * (ohi & 7) + (n >> 1);
            const int vlo = (olo >= 8 ? 2 : 0) + (n & 1), vhi = (ohi >= 8 ? 2 : 0) + (n & 1);
            float lo = 0.f, hi2 = 0.f;
#pragma unroll
            for (int q2 = 0; q2 < 4; ++q2) {
              const float a = __shfl_sync(0xffffffffu, hv[q2], src_lo);
              const float bq = __shfl_sync(0xffffffffu, hv[q2], src_hi);
              if (q2 == vlo) lo = a;
              if (q2 == vhi) hi2 = bq;
            }
            if (n < T)
              hperm[((((size_t)e * DEC_MAX_T + n) * NGI + (rb >> 2)) * 4 + (rb & 3)) * 8 + w] =
                  pack_bf2(lo, hi2);
          }
          // per-token sums of the 16 rows: lanes (g, c) add their rows, then
          // the 8 lanes of a token column pair add over g
          float s0 = hv[0] + hv[2], s1 = hv[1] + hv[3];
#pragma unroll
          for (int o = 4; o < 32; o <<= 1) {
            s0 += __shfl_xor_sync(0xffffffffu, s0, o);
            s1 += __shfl_xor_sync(0xffffffffu, s1, o);
          }
          if (g == 0) {
            float *hs = wsp<float>(p, p.L.hsum);
            if (2 * c < T) hs[((size_t)e * DEC_MAX_T + 2 * c) * RB + rb] = s0;
            if (2 * c + 1 < T) hs[((size_t)e * DEC_MAX_T + 2 * c + 1) * RB + rb] = s1;
          }
          __syncwarp();
          if (lane == 0) red_release_add(ent_done + e * KL_CSTRIDE, 1u);  // h rows of this item are out
        }
      }
    }
  }
  if (p.trace && lane == 0) atomicMax(&s_tm[0], (unsigned long long)globaltimer());

  // ---------------- 5. down projection ----------------
  uint16_t *wparts = wsp<uint16_t>(p, p.L.wparts);
  uint16_t *sparts = wsp<uint16_t>(p, p.L.sparts);
  {
    const int nsi = NGI >> gs, sbh = 16 * nsi;  // scales per row; bf16 per scale tensor
    int cur_e = -1, slot = 0;
    int rank0 = -1, rank1 = -1;
    float score0 = 0.f, score1 = 0.f;
    bool is_sh = false;
    volatile int *hflag = s_misc + 4;
#pragma unroll 1
    for (int jj = 0; jj < nj; ++jj) {
      const int i = d0 + warp + KL_WARPS * jj;
      const int e = i / RBN, rb = i % RBN;
      if (e != cur_e) {
        // The entry's h (complete once its RB gate/up items are counted) is
        // staged once per CTA: the first warp to need it claims the slot,
        // waits for the entry and copies h and its group sums; the others
        // wait for the slot's flag (0 empty, 1 loading, 2 ready, 3 failed).
        slot = e - e_lo;
        int claim = 1;
        if (lane == 0) claim = atomicCAS(const_cast<int *>(hflag + slot), 0, 1);
        claim = __shfl_sync(0xffffffffu, claim, 0);
        bool ok = true;
        if (claim == 0) {
          ok = wait_ge(ent_done + e * KL_CSTRIDE, (unsigned)RB);
          ok = __all_sync(0xffffffffu, ok);
          if (ok) {
            const uint4 *src = reinterpret_cast<const uint4 *>(wsp<const uint32_t>(p, p.L.hperm) +
                                                               (size_t)e * DEC_MAX_T * (I / 2));
            uint4 *dst = reinterpret_cast<uint4 *>(hf + slot * (Tl::HF / 4));
            for (int u = lane; u < T * NGI * 8; u += 32) dst[u] = __ldcg(src + u);
            const float *hsum = wsp<const float>(p, p.L.hsum) + (size_t)e * DEC_MAX_T * RB;
            for (int u = lane; u < T * NGI; u += 32) {
              const int n = u / NGI, Gi = u % NGI;
              const float4 v = __ldcg(reinterpret_cast<const float4 *>(hsum + (size_t)n * RB + 4 * Gi));
              hsg[(slot * NGI + Gi) * DEC_MAX_T + n] = ((v.x + v.y) + v.z) + v.w;
            }
            for (int u = lane; u < NGI * DEC_MAX_T; u += 32)
              if ((u & 7) >= T) hsg[slot * NGI * DEC_MAX_T + u] = 0.f;
          }
          __syncwarp();
          if (lane == 0) {
            __threadfence_block();
            hflag[slot] = ok ? 2 : 3;
          }
        } else {
          // every lane observes the flag itself, then reads the slot
          int f = 0;
          const uint64_t t0 = globaltimer();
          for (;;) {
            f = hflag[slot];
            if (f >= 2) break;
            if (globaltimer() - t0 > KL_WAIT_NS) break;
            __nanosleep(128);
          }
          __threadfence_block();
          ok = __all_sync(0xffffffffu, f == 2);
        }
        if (!ok) {
          if (lane == 0) flag_status(p.status, VB_STATUS_TIMEOUT);
          j_end = jj;
          break;
        }
        cur_e = e;
        is_sh = s_ent[e].flags & 1;
        rank0 = 2 * c < T ? s_ent[e].rank[2 * c] : -1;
        rank1 = 2 * c + 1 < T ? s_ent[e].rank[2 * c + 1] : -1;
        score0 = 2 * c < T ? s_ent[e].score[2 * c] : 0.f;
        score1 = 2 * c + 1 < T ? s_ent[e].score[2 * c + 1] : 0.f;
      }
      const uint32_t *hs_f = hf + slot * (Tl::HF / 4);
      const float *hs_g = hsg + slot * NGI * DEC_MAX_T;
      float acc[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll 1
      for (int dc = 0; dc < DCH; ++dc) {
        cp_async_wait<RS - 2>();
        __syncwarp();
        issue_next();
        const int qd = nq_gu + jj * DCH + dc;
        const uint8_t *st = ring + (qd % RS) * Tl::STAGE;
        const uint16_t *ss = reinterpret_cast<const uint16_t *>(st + Tl::DWB);
#pragma unroll
        for (int gl = 0; gl < DG; ++gl) {
          const int Gi = dc * DG + gl;
          constexpr int CPR = Tl::DROWB / 16;
          const int fo = g * Tl::DROWB + (swz<CPR>(g, 2 * gl + (c >> 1)) << 4) + (c & 1) * 8;
          const uint2 a0 = lds64(st + fo);
          const uint2 a1 = lds64(st + 8 * Tl::DROWB + fo);
          uint4 hb0 = make_uint4(0, 0, 0, 0), hb1 = hb0;
          if (g < T) {
            const uint4 *hp = reinterpret_cast<const uint4 *>(hs_f + ((g * NGI + Gi) * 4 + c) * 8);
            hb0 = hp[0];
            hb1 = hp[1];
          }
          const float2 hsv = *reinterpret_cast<const float2 *>(hs_g + Gi * DEC_MAX_T + 2 * c);
          uint32_t p0[2][4], p1[2][4];
          nib_pairs4(a0.x, p0[0]);
          nib_pairs4(a0.y, p0[1]);
          nib_pairs4(a1.x, p1[0]);
          nib_pairs4(a1.y, p1[1]);
          const uint32_t hw[8] = {hb0.x, hb0.y, hb0.z, hb0.w, hb1.x, hb1.y, hb1.z, hb1.w};
          float dd[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
          for (int m = 0; m < 4; ++m) {
            const int i0m = 2 * (m & 1), h = m >> 1;
            mma_bf16(dd, p0[h][i0m], p1[h][i0m], p0[h][i0m + 1], p1[h][i0m + 1], hw[2 * m],
                     hw[2 * m + 1]);
          }
          const int si = Gi >> gs;
          const float s0 = bf2f(ss[g * nsi + si]), s1 = bf2f(ss[(g + 8) * nsi + si]);
          const float b0 = bf2f(ss[sbh + g * nsi + si]);
          const float b1 = bf2f(ss[sbh + (g + 8) * nsi + si]);
          const float bp0 = fmaf(-128.f, s0, b0), bp1 = fmaf(-128.f, s1, b1);
          acc[0] = fmaf(bp0, hsv.x, fmaf(s0, dd[0], acc[0]));
          acc[1] = fmaf(bp0, hsv.y, fmaf(s0, dd[1], acc[1]));
          acc[2] = fmaf(bp1, hsv.x, fmaf(s1, dd[2], acc[2]));
          acc[3] = fmaf(bp1, hsv.y, fmaf(s1, dd[3], acc[3]));
        }
      }
      const int r0 = 16 * rb + g, r1 = r0 + 8;
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        const int n = 2 * c + (q & 1);
        if (n >= T) continue;
        const int row = (q >> 1) ? r1 : r0;
        const float yb = rbf(acc[q]);
        if (is_sh) {
          sparts[(size_t)n * H + row] = f2bf(yb);
        } else {
          const int rk = (q & 1) ? rank1 : rank0;
          const float sc = (q & 1) ? score1 : score0;
          if (rk >= 0) wparts[((size_t)n * p.k + rk) * H + row] = f2bf(__fmul_rn(yb, sc));
        }
      }
    }
    cp_async_wait<0>();
  }
  if (p.trace && lane == 0) atomicMax(&s_tm[1], (unsigned long long)globaltimer());

  // ---------------- 6. tickets and combine ----------------
  // One acquire-release ticket per item (lanes in parallel; the warp barrier
  // orders every lane's stores before them); the warp that completes a
  // 16-row block combines it.
  __syncwarp();
  unsigned *cnt = wsp<unsigned>(p, p.L.rb_count);
#pragma unroll 1
  for (int base = 0; base < j_end; base += 32) {
    const int jj = base + lane;
    int rb = 0;
    bool win = false;
    if (jj < j_end) {
      rb = (d0 + warp + KL_WARPS * jj) % RBN;
      win = atom_add_acq_rel(cnt + rb * KL_CSTRIDE, 1u) == (unsigned)n_ent - 1;
    }
    unsigned m = __ballot_sync(0xffffffffu, win);
    __syncwarp();
    while (m) {
      // up to four completed blocks at a time, one per group of 8 lanes
      int mine = -1;
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        const int src = m ? __ffs(m) - 1 : 0;
        const int rbq = __shfl_sync(0xffffffffu, rb, src);
        if (m && (lane >> 3) == q) mine = rbq;
        m &= m - 1;
      }
      if (mine >= 0) {
        down_combine_rows(p, s_ok, mine, lane);
        if ((lane & 7) == 0) cnt[mine * KL_CSTRIDE] = 0u;  // ready for the next launch
      }
      __syncwarp();
    }
  }
  if (p.trace) {
    if (lane == 0) atomicMax(&s_tm[2], (unsigned long long)globaltimer());
    __syncthreads();
    if (tid < 3) atomicMax(reinterpret_cast<unsigned long long *>(p.trace + 6 + tid), s_tm[tid]);
  }
  span.end();
}

// One-time per-kernel attributes: the dynamic shared memory it needs and the
// largest shared-memory carveout.
static cudaError_t decode_kernel_attrs(const void *fn, size_t smem) {
  static std::mutex mu;
  static std::vector<std::pair<const void *, size_t>> done;
  std::lock_guard<std::mutex> lock(mu);
  for (auto &d : done)
    if (d.first == fn && d.second >= smem) return cudaSuccess;
  cudaError_t e = cudaFuncSetAttribute(fn, cudaFuncAttributePreferredSharedMemoryCarveout,
                                       (int)cudaSharedmemCarveoutMaxShared);
  if (e == cudaSuccess && smem > 48 * 1024)
    e = cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  if (e == cudaSuccess) done.emplace_back(fn, smem);
  return e;
}

static int sm_count() {
  static int n = 0;
  if (!n) {
    int dev = 0;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
    if (n <= 0) n = 148;
  }
  return n;
}

}  // namespace vb

using namespace vb;

// Scratch of vb_moe_decode_noalloc: one fixed array per device, shared by
// every call of that entry point on the device. Its device address is looked
// up once per device (with that device current) and cached here.
static __device__ __align__(256) uint8_t g_decode_noalloc_scratch[VB_MOE_DECODE_NOALLOC_SCRATCH_BYTES];

namespace {
constexpr int kNoallocMaxDevices = 64;
std::mutex g_noalloc_mu;
void *g_noalloc_ptr[kNoallocMaxDevices];

int noalloc_scratch(void **out) {
  int dev = -1;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess)
    return set_error(VB_ERR_CUDA, "vb_moe_decode_noalloc: cudaGetDevice: %s", cudaGetErrorString(e));
  VB_REQUIRE(dev >= 0 && dev < kNoallocMaxDevices, "vb_moe_decode_noalloc: device %d", dev);
  std::lock_guard<std::mutex> lock(g_noalloc_mu);
  if (!g_noalloc_ptr[dev]) {
    void *ptr = nullptr;
    e = cudaGetSymbolAddress(&ptr, g_decode_noalloc_scratch);
    if (e != cudaSuccess || !ptr)
      return set_error(VB_ERR_CUDA, "vb_moe_decode_noalloc: cudaGetSymbolAddress: %s",
                       cudaGetErrorString(e));
    g_noalloc_ptr[dev] = ptr;
  }
  *out = g_noalloc_ptr[dev];
  return VB_OK;
}

using LayerFn = void (*)(DecodeParams);

// Launch of the layer kernel: cooperative (the runtime places every CTA at
// once, which the grid barrier needs) and, unless timing events surround it,
// a programmatic dependent launch. If the runtime refuses the pair on the
// first (uncaptured) launch, later launches use PDL alone: one CTA per SM
// still fits, so the CTAs are resident whenever the kernel runs alone.
std::atomic<int> g_coop_state{-1};  // -1 untried, 0 refused, 1 accepted

cudaError_t launch_layer(LayerFn fn, int grid, size_t smem, cudaStream_t s, bool pdl,
                         const DecodeParams &p) {
  for (;;) {
    const int state = g_coop_state.load();
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(grid);
    cfg.blockDim = dim3(KL_THREADS);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = s;
    cudaLaunchAttribute attr[2];
    int na = 0;
    if (pdl) {
      attr[na].id = cudaLaunchAttributeProgrammaticStreamSerialization;
      attr[na].val.programmaticStreamSerializationAllowed = 1;
      ++na;
    }
    if (state != 0) {
      attr[na].id = cudaLaunchAttributeCooperative;
      attr[na].val.cooperative = 1;
      ++na;
    }
    cfg.attrs = attr;
    cfg.numAttrs = na;
    const cudaError_t e = cudaLaunchKernelEx(&cfg, fn, p);
    if (state != -1) return e;
    if (e == cudaSuccess) {
      g_coop_state = 1;
      return e;
    }
    cudaStreamCaptureStatus cs = cudaStreamCaptureStatusNone;
    if (cudaStreamIsCapturing(s, &cs) != cudaSuccess || cs != cudaStreamCaptureStatusNone)
      return e;
    (void)cudaGetLastError();  // the refusal is not sticky
    g_coop_state = 0;
  }
}

// The layer kernel and its shared memory for (H, I).
bool layer_kernel(int H, int I, LayerFn *fn, size_t *smem) {
#define VB_HI(HH, II)                                 \
  if (H == HH && I == II) {                           \
    *fn = moe_layer_kernel<HH, II>;                   \
    *smem = LayerTile<HH, II>::SMEM;                  \
    return true;                                      \
  }
  VB_HI(512, 128) VB_HI(512, 256) VB_HI(512, 512)
  VB_HI(1024, 128) VB_HI(1024, 256) VB_HI(1024, 512)
  VB_HI(2048, 128) VB_HI(2048, 256) VB_HI(2048, 512)
  VB_HI(4096, 128) VB_HI(4096, 256) VB_HI(4096, 512)
#undef VB_HI
  return false;
}
}  // namespace

extern "C" {

size_t vb_moe_decode_workspace_size(int32_t tokens, int32_t hidden,
                                    int32_t inter, int32_t num_experts,
                                    int32_t top_k) {
  if (tokens <= 0 || hidden <= 0 || inter <= 0 || num_experts <= 0 || top_k <= 0)
    return 0;
  return decode_layout(tokens, hidden, inter, num_experts, top_k).total;
}

}  // extern "C"

namespace {
// vb_moe_decode after its argument checks; with clear_bytes > 0 the first
// clear_bytes of the workspace are zeroed on the stream right before the
// launch, once every check has passed (a rejected call touches neither the
// device nor the stream).
int moe_decode_impl(const VbMoeDecodeArgs *a, vb_stream_t stream, size_t clear_bytes) {
  VB_REQUIRE(a, "vb_moe_decode: null args");
  const int T = a->tokens, H = a->hidden, I = a->inter, E = a->num_experts,
            k = a->top_k;
  VB_REQUIRE(T >= 1 && T <= DEC_MAX_T, "vb_moe_decode: tokens=%d not in [1,8]", T);
  VB_REQUIRE(a->bits == 4, "vb_moe_decode: bits=%d (only 4-bit)", a->bits);
  VB_REQUIRE(a->group == 64 || a->group == 128, "vb_moe_decode: group=%d", a->group);
  VB_REQUIRE(H == 512 || H == 1024 || H == 2048 || H == 4096, "vb_moe_decode: hidden=%d", H);
  VB_REQUIRE(I == 128 || I == 256 || I == 512, "vb_moe_decode: inter=%d", I);
  VB_REQUIRE(H / a->group >= 8 && I >= a->group, "vb_moe_decode: group too large");
  VB_REQUIRE(E >= k && E <= DEC_MAX_E, "vb_moe_decode: num_experts=%d", E);
  VB_REQUIRE(k >= 1 && k <= DEC_MAX_K, "vb_moe_decode: top_k=%d", k);
  VB_REQUIRE(T * k + 1 <= sm_count(),
             "vb_moe_decode: tokens*top_k+1=%d entries exceed the %d SMs", T * k + 1, sm_count());
  VB_REQUIRE(a->x && a->router_w && a->slot_table && a->out, "vb_moe_decode: null tensor");
  VB_REQUIRE(a->pool.ptr[0] && a->pool.cap > 0, "vb_moe_decode: empty pool");
  const bool has_shared = a->shared.ptr[0] != nullptr;
  VB_REQUIRE(!has_shared || a->shared_gate_w, "vb_moe_decode: shared expert without gate");
  DecodeLayout L = decode_layout(T, H, I, E, k);
  VB_REQUIRE(a->workspace && a->workspace_bytes >= L.total,
             "vb_moe_decode: workspace %zu < %zu", a->workspace_bytes, L.total);
  VB_REQUIRE(((uintptr_t)a->workspace % 256) == 0, "vb_moe_decode: workspace must be 256-byte aligned");
  VB_REQUIRE(((uintptr_t)a->x % 16) == 0 && ((uintptr_t)a->out % 16) == 0 &&
                 ((uintptr_t)a->residual % 16) == 0,
             "vb_moe_decode: x, out and residual must be 16-byte aligned");
  for (int i = 0; i < 9; ++i)
    VB_REQUIRE(((uintptr_t)a->pool.ptr[i] % 16) == 0 && (a->pool.slot_stride[i] % 16) == 0 &&
                   (!has_shared || (((uintptr_t)a->shared.ptr[i] % 16) == 0)),
               "vb_moe_decode: pool tensors and slot strides must be 16-byte aligned");

  DecodeParams p;
  p.T = T; p.H = H; p.I = I; p.E = E; p.k = k; p.norm_topk = a->norm_topk;
  p.norm_eps = a->norm_eps;
  p.gshift = a->group == 128 ? 1 : 0;
  p.has_shared = has_shared ? 1 : 0;
  p.route_only = (a->flags & VB_DECODE_ROUTE_ONLY) ? 1 : 0;
  VB_REQUIRE((a->flags & ~VB_DECODE_ROUTE_ONLY) == 0, "vb_moe_decode: unknown flags %#x", a->flags);
  p.x = a->x; p.router_w = a->router_w; p.shared_gate_w = a->shared_gate_w;
  p.residual = a->residual; p.router_bias = a->router_bias; p.table = a->slot_table;
  p.pool = a->pool; p.shared = a->shared;
  p.out = a->out; p.out_scores = a->out_scores; p.out_inds = a->out_inds;
  p.out_local = a->out_local; p.status = a->status;
  p.ws = static_cast<uint8_t *>(a->workspace);
  p.trace = a->trace;
  p.L = L;

  LayerFn fn = nullptr;
  size_t smem = 0;
  VB_REQUIRE(layer_kernel(H, I, &fn, &smem), "vb_moe_decode: no kernel for hidden=%d inter=%d", H, I);
  cudaError_t err = decode_kernel_attrs((const void *)fn, smem);
  if (err != cudaSuccess) return set_error(VB_ERR_CUDA, "decode kernel attributes: %s", cudaGetErrorString(err));
  // The grid barrier needs every CTA resident: one CTA per SM.
  int per_sm = 0;
  err = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, fn, KL_THREADS, smem);
  if (err != cudaSuccess || per_sm < 1)
    return set_error(VB_ERR_CUDA, "moe_layer_kernel does not fit an SM (%s)",
                     err != cudaSuccess ? cudaGetErrorString(err) : "occupancy 0");

  cudaStream_t s = as_stream(stream);
  if (clear_bytes > 0) {
    err = cudaMemsetAsync(a->workspace, 0, clear_bytes, s);
    if (err != cudaSuccess)
      return set_error(VB_ERR_CUDA, "vb_moe_decode_noalloc: clearing scratch: %s",
                       cudaGetErrorString(err));
  }
  cudaEvent_t *ev = a->timing_events ? (cudaEvent_t *)a->timing_events : nullptr;
  const bool pdl = ev == nullptr;  // event records would break the PDL chain
  if (ev) cudaEventRecord(ev[0], s);
  err = launch_layer(fn, sm_count(), smem, s, pdl, p);
  if (err != cudaSuccess) return set_error(VB_ERR_CUDA, "moe_layer_kernel: %s", cudaGetErrorString(err));
  if (ev) cudaEventRecord(ev[1], s);
  return VB_OK;
}
}  // namespace

extern "C" {

int vb_moe_decode(const VbMoeDecodeArgs *a, vb_stream_t stream) {
  return moe_decode_impl(a, stream, 0);
}

int vb_moe_decode_noalloc(const VbMoeDecodeArgs *a, vb_stream_t stream) {
  VB_REQUIRE(a, "vb_moe_decode_noalloc: null args");
  const size_t need = vb_moe_decode_workspace_size(a->tokens, a->hidden, a->inter,
                                                   a->num_experts, a->top_k);
  VB_REQUIRE(need > 0, "vb_moe_decode_noalloc: invalid shape");
  if (need > VB_MOE_DECODE_NOALLOC_SCRATCH_BYTES)
    return set_error(VB_ERR_WORKSPACE,
                     "vb_moe_decode_noalloc: this shape needs %zu bytes of scratch, more than "
                     "the fixed %zu-byte array; use vb_moe_decode with a workspace",
                     need, (size_t)VB_MOE_DECODE_NOALLOC_SCRATCH_BYTES);
  void *scratch = nullptr;
  const int rc = noalloc_scratch(&scratch);
  if (rc != VB_OK) return rc;
  // The array keeps the previous call's contents: the words the kernel
  // expects at zero (grid barrier, shared gates, entry counters, row-block
  // tickets) are zeroed in stream order before this call's kernel, after
  // every argument check has passed.
  const DecodeLayout L = decode_layout(a->tokens, a->hidden, a->inter, a->num_experts, a->top_k);
  VbMoeDecodeArgs b = *a;
  b.workspace = scratch;
  b.workspace_bytes = VB_MOE_DECODE_NOALLOC_SCRATCH_BYTES;
  return moe_decode_impl(&b, stream, L.zero_end);
}

}  // extern "C"
