// Decode / MTP-verify fused MoE block (T <= 8 tokens), MLX bf16 dtype chain.
//
// Reference: FileStreamingMoeBlock.__call__ (mlx_streaming/core/moe/block.py
// :245-1013) with PersistentSubGLU.forward (compute.py:145-199) and the
// shared expert (block.py:102-109, 1009-1012).
//
// Three kernels per block, chained with programmatic dependent launch (PDL):
//  K1 router: optional unit RMSNorm of x, logits = bf16(x.Wr^T [+bias]) and
//     the shared-expert gate sigmoid(x.w_sg) as one more row; every row is
//     split over 2-4 warps and loaded before the PDL wait. All CTAs share
//     writing x in MMA-fragment order (xperm) and per-64-column sums (xsum).
//     The last CTA (atomic ticket) runs the precise softmax, top-k (one warp
//     reduction per pick on (bf16 probability, expert id) keys, lower id wins
//     ties), renormalisation and slot gather, and writes the list of
//     "entries": the shared expert first, then every distinct routed expert.
//  K2 gate/up: persistent CTAs; the two warps of a pair split an item (entry,
//     16 intermediate rows) over the hidden dimension and stream it through
//     per-warp cp.async rings; 4-bit codes become exact bf16 values 128+q for
//     mma.m16n8k16 and the per-group epilogue applies y += s*D + (b-128*s)*
//     sum(x). SwiGLU (bf16 per op); h in fragment order (hperm). Item blocks
//     and the matching down-projection rows are bulk-prefetched into L2.
//  K3 down + combine: one CTA per (entry, 128 output rows), weights requested
//     before the PDL wait; per route the result is rounded to bf16, times the
//     route score, rounded again (MLX chain). The last CTA of each 128-row
//     block (atomic ticket) adds the k routes of every token in rank order
//     (exact double sum of bf16 values, rounded to float32 then bf16), then
//     the gated shared expert and the optional residual.
#include <algorithm>
#include <mutex>
#include <vector>

#include "common.cuh"

namespace vb {

constexpr int DEC_MAX_T = 8;
constexpr int DEC_MAX_K = 16;
constexpr int DEC_MAX_E = 1024;
constexpr int DEC_SMEM_BUDGET = 200 * 1024;

struct DecEntry {
  int32_t slot;
  int32_t flags;  // bit0 = shared expert
  int32_t pad[2];
  int32_t rank[DEC_MAX_T];  // route rank of token n, -1 = not routed here
  float score[DEC_MAX_T];   // bf16 route score
};

struct DecodeLayout {
  size_t counter, n_entries, sgate, rb_count, zero_end, logits, entries, route_ok, xperm, xsum,
      hperm, hsum, wparts, sparts, total;
  int max_entries;
};

static DecodeLayout decode_layout(int T, int H, int I, int E, int k) {
  DecodeLayout L;
  L.max_entries = T * k + 1;
  size_t off = 0;
  L.counter = off; off += 4;
  L.n_entries = off; off += 4;
  off = align_up(off, 16);
  L.sgate = off; off += sizeof(float) * DEC_MAX_T;
  off = align_up(off, 16);
  L.rb_count = off; off += sizeof(unsigned) * (H / 16);
  L.zero_end = off;  // [0, zero_end) must be zero before a call (tickets)
  off = align_up(off, 256);
  L.logits = off; off += sizeof(float) * (size_t)T * E;
  off = align_up(off, 256);
  L.entries = off; off += sizeof(DecEntry) * (size_t)L.max_entries;
  off = align_up(off, 256);
  L.route_ok = off; off += sizeof(int32_t) * (size_t)T * k;
  off = align_up(off, 256);
  L.xperm = off; off += sizeof(uint32_t) * (size_t)T * (H / 2);
  off = align_up(off, 256);
  L.xsum = off; off += sizeof(float) * (size_t)T * (H / 64);
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
  int T, H, I, E, k, norm_topk, gshift, has_shared;
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

// Optional span trace: thread 0 of every CTA folds its start/end into the
// kernel's [min start, max end] pair.
struct SpanTrace {
  uint64_t *slot;
  uint64_t t0;
  __device__ __forceinline__ SpanTrace(uint64_t *trace, int kernel) {
    slot = (trace && threadIdx.x == 0) ? trace + 2 * kernel : nullptr;
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

// L2 bulk prefetch of tensors [t0, t1) of one expert, pieces [first, ...) of
// the expert's piece sequence with stride `step` (pieces are 16 KB).
__device__ __forceinline__ int expert_pieces(const DecodeParams &p, int t0, int t1) {
  int n = 0;
  for (int t = t0; t < t1; ++t) n += (expert_tensor_bytes(p, t) + PF_PIECE - 1) / PF_PIECE;
  return n;
}
__device__ __forceinline__ void prefetch_expert_piece(const DecodeParams &p, const VbQuantPool &pool,
                                                      int slot, int t0, int piece) {
  for (int t = t0; t < 9; ++t) {
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

// ----------------------------------------------------------------------------
// K1: router GEMV + last-CTA softmax/top-k/entries. H is a template constant
// so that every index is a shift. Rows 0..E-1 are the experts' router rows,
// row E (when there is a shared expert) the shared-expert gate row; each row
// is split over Q warps (RPC = 8/Q rows per CTA) whose partial dots are added
// in part order. Rows are loaded before the PDL wait.
// ----------------------------------------------------------------------------
constexpr int K1_THREADS = 256;
constexpr int K1_WARPS = K1_THREADS / 32;

template <int H>
struct RouterTile {
  static constexpr int Q = H >= 1024 ? 4 : 2;  // warps per row
  static constexpr int RPC = K1_WARPS / Q;      // rows per CTA
  static constexpr int NVQ = H / (256 * Q);     // uint4 of a row part per lane
  static_assert(NVQ >= 1, "router tile");
};

// Orderable key of a float (for unsigned max).
__device__ __forceinline__ uint32_t f2key(float f) {
  const uint32_t b = __float_as_uint(f);
  return (b & 0x80000000u) ? ~b : (b | 0x80000000u);
}
__device__ __forceinline__ float key2f(uint32_t k) {
  return __uint_as_float((k & 0x80000000u) ? (k & 0x7fffffffu) : ~k);
}

template <int H, int PER>  // PER = ceil(E / 32) logits per lane
__global__ void __launch_bounds__(K1_THREADS, 2) moe_router_kernel(DecodeParams p) {
  using Tl = RouterTile<H>;
  constexpr int Q = Tl::Q, RPC = Tl::RPC, NVQ = Tl::NVQ;
  constexpr int NG = H / 64;
  extern __shared__ __align__(16) uint8_t smem_raw[];
  uint16_t *xs = reinterpret_cast<uint16_t *>(smem_raw);  // [T][H] bf16
  __shared__ double s_ss[K1_WARPS][DEC_MAX_T];
  __shared__ float s_inv[DEC_MAX_T];
  __shared__ float s_part[RPC][Q][DEC_MAX_T];
  const int T = p.T, E = p.E;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  SpanTrace span(p.trace, 0);

  // This warp's row part; row E is the shared-expert gate.
  const int rloc = warp / Q, part = warp % Q;
  const int row = blockIdx.x * RPC + rloc;
  const int nrows = E + (p.has_shared ? 1 : 0);
  uint4 wv[NVQ];
  if (row < nrows) {
    const uint16_t *src = row < E ? p.router_w + (size_t)row * H : p.shared_gate_w;
    const uint4 *w4 = reinterpret_cast<const uint4 *>(src + part * (H / Q));
#pragma unroll
    for (int u = 0; u < NVQ; ++u) wv[u] = ldg_nc_v4(w4 + u * 32 + lane);
  }
  if (blockIdx.x == 0 && tid * 32 < E) prefetch_l2(p.table + tid * 32);  // slot table lines
  pdl_wait();
  pdl_launch_dependents();
  trace_mark(p.trace, 8);

  {
    // Stage x: independent 16-byte loads issued before the stores.
    const uint4 *src = reinterpret_cast<const uint4 *>(p.x);
    uint4 *dst = reinterpret_cast<uint4 *>(xs);
    constexpr int PT = (DEC_MAX_T * H / 8 + K1_THREADS - 1) / K1_THREADS;
    const int nvec = T * (H / 8);
    uint4 v[PT];
#pragma unroll
    for (int u = 0; u < PT; ++u) {
      const int i = u * K1_THREADS + tid;
      if (i < nvec) v[u] = __ldcg(src + i);
    }
#pragma unroll
    for (int u = 0; u < PT; ++u) {
      const int i = u * K1_THREADS + tid;
      if (i < nvec) dst[i] = v[u];
    }
  }
  __syncthreads();
  trace_mark(p.trace, 11);
  if (p.norm_eps > 0.f) {
    // Unit-weight RMSNorm of the block input (decoder post-attention norm):
    // y = bf16(x * (1/sqrt(mean(x^2) + eps))), float32 math with an exact
    // (double) sum of squares: squares of bf16 values have 16 significant
    // bits, so their double sum does not depend on the order. Every CTA
    // computes it identically.
    constexpr int VPT = H / 8;  // uint4 per token
    double ss[DEC_MAX_T];
#pragma unroll
    for (int t = 0; t < DEC_MAX_T; ++t) ss[t] = 0.0;
#pragma unroll
    for (int t = 0; t < DEC_MAX_T; ++t) {
      if (t < T) {
        for (int v = tid; v < VPT; v += K1_THREADS) {
          const uint4 q = reinterpret_cast<const uint4 *>(xs + (size_t)t * H)[v];
          const uint32_t w[4] = {q.x, q.y, q.z, q.w};
#pragma unroll
          for (int j = 0; j < 4; ++j) {
            const double a = bf2f(w[j] & 0xFFFF), b = bf2f(w[j] >> 16);
            ss[t] = fma(a, a, ss[t]);
            ss[t] = fma(b, b, ss[t]);
          }
        }
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) ss[t] += __shfl_xor_sync(0xffffffffu, ss[t], o);
        if (lane == 0) s_ss[warp][t] = ss[t];
      }
    }
    __syncthreads();
    if (tid < T) {
      double tot = 0.0;
#pragma unroll
      for (int w = 0; w < K1_WARPS; ++w) tot += s_ss[w][tid];
      const float ms = __fdiv_rn((float)tot, (float)H);
      s_inv[tid] = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(ms, p.norm_eps)));
    }
    __syncthreads();
    for (int i = tid; i < T * (H / 8); i += K1_THREADS) {
      const int t = i / (H / 8);
      uint4 v = reinterpret_cast<const uint4 *>(xs)[i];
      uint32_t w[4] = {v.x, v.y, v.z, v.w};
      const float inv = s_inv[t];
#pragma unroll
      for (int q = 0; q < 4; ++q)
        w[q] = pack_bf2(__fmul_rn(bf2f(w[q] & 0xFFFF), inv), __fmul_rn(bf2f(w[q] >> 16), inv));
      reinterpret_cast<uint4 *>(xs)[i] = make_uint4(w[0], w[1], w[2], w[3]);
    }
    __syncthreads();
  }
  trace_mark(p.trace, 12);

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
          const uint4 xv = reinterpret_cast<const uint4 *>(xs + (size_t)t * H)[v];
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
#pragma unroll
    for (int t = 0; t < DEC_MAX_T; ++t) {
      if (t < T) {
        float a = acc[t];
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) a += __shfl_xor_sync(0xffffffffu, a, o);
        if (lane == 0) s_part[rloc][part][t] = a;
      }
    }
  }
  __syncthreads();
  if (tid < RPC * DEC_MAX_T) {
    const int rl = tid / DEC_MAX_T, t = tid % DEC_MAX_T;
    const int r = blockIdx.x * RPC + rl;
    if (r < nrows && t < T) {
      float a = 0.f;
#pragma unroll
      for (int q = 0; q < Q; ++q) a += s_part[rl][q][t];
      if (r < E) {
        if (p.router_bias) a = a + p.router_bias[r];
        wsp<float>(p, p.L.logits)[(size_t)t * E + r] = rbf(a);
      } else {
        wsp<float>(p, p.L.sgate)[t] = rbf(mlx_sigmoid(rbf(a)));
      }
    }
  }
  trace_mark(p.trace, 13);

  {
    // x in MMA fragment order (xperm) and per-64-column sums (xsum), spread
    // over all CTAs (each holds the whole normalised x in shared memory).
    uint32_t *xperm = wsp<uint32_t>(p, p.L.xperm);
    const int gtid = blockIdx.x * blockDim.x + tid, gstride = gridDim.x * blockDim.x;
    for (int i = gtid; i < T * (H / 2); i += gstride) {
      const int n = i / (H / 2);
      const int r = i % (H / 2);
      const int G = r >> 5, c = (r >> 3) & 3, w = r & 7;
      const int m = w >> 1, pp = w & 1, j = m >> 1, i0 = 2 * (m & 1);
      const int base = 64 * G + 16 * c + 8 * j + i0 + pp;
      const uint32_t lo = xs[(size_t)n * H + base], hi = xs[(size_t)n * H + base + 4];
      xperm[i] = lo | (hi << 16);
    }
    float *xsum = wsp<float>(p, p.L.xsum);
    const int gwarp = blockIdx.x * K1_WARPS + warp;
    const int nwarps = gridDim.x * K1_WARPS;
    for (int it = gwarp; it < T * NG; it += nwarps) {
      const int n = it / NG, G = it % NG;
      const uint32_t v = reinterpret_cast<const uint32_t *>(xs + (size_t)n * H + 64 * G)[lane];
      float s = bf2f(v & 0xFFFF) + bf2f(v >> 16);
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
      if (lane == 0) xsum[it] = s;
    }
  }

  // Last-CTA ticket.
  __shared__ unsigned s_ticket;
  trace_mark(p.trace, 9);
  __threadfence();
  __syncthreads();
  if (tid == 0) s_ticket = atomicAdd(wsp<unsigned>(p, p.L.counter), 1u);
  __syncthreads();
  if (s_ticket != gridDim.x - 1) {
    span.end();
    return;
  }
  __threadfence();
  trace_mark(p.trace, 10);

  // ---- softmax + top-k per token (one warp per token) ----
  __shared__ int s_ex[DEC_MAX_T * DEC_MAX_K];
  __shared__ int s_slot[DEC_MAX_T * DEC_MAX_K];
  __shared__ float s_score[DEC_MAX_T * DEC_MAX_K];
  __shared__ int s_first[DEC_MAX_E];  // first route of each expert
  __shared__ int s_ent[DEC_MAX_T * DEC_MAX_K];
  __shared__ int s_wcnt[K1_WARPS];
  __shared__ __align__(16) DecEntry s_entries[DEC_MAX_T * DEC_MAX_K + 1];
  __shared__ int s_table[DEC_MAX_E];
  const int k = p.k;
  const float *logits = wsp<float>(p, p.L.logits);
  // Slot table and logits are loaded together (one memory round trip).
  float v[PER];
  {
    const int t = warp;
    int tb[(DEC_MAX_E + K1_THREADS - 1) / K1_THREADS];
#pragma unroll
    for (int j = 0; j < (DEC_MAX_E + K1_THREADS - 1) / K1_THREADS; ++j) {
      const int i = tid + j * K1_THREADS;
      tb[j] = i < E ? __ldg(p.table + i) : -1;
    }
#pragma unroll
    for (int i = 0; i < PER; ++i) {
      const int idx = lane + 32 * i;
      v[i] = (t < T && idx < E) ? __ldcg(logits + (size_t)t * E + idx) : -INFINITY;
    }
#pragma unroll
    for (int j = 0; j < (DEC_MAX_E + K1_THREADS - 1) / K1_THREADS; ++j) {
      const int i = tid + j * K1_THREADS;
      if (i < E) {
        s_table[i] = tb[j];
        s_first[i] = 0x7fffffff;
      }
    }
  }
  __syncthreads();
  for (int t = warp; t < T; t += K1_WARPS) {
    uint32_t mk = 0;
#pragma unroll
    for (int i = 0; i < PER; ++i) mk = max(mk, f2key(v[i]));
    const float m = key2f(__reduce_max_sync(0xffffffffu, mk));
    double sd[PER];
#pragma unroll
    for (int i = 0; i < PER; ++i) {
      const int idx = lane + 32 * i;
      const float ex = idx < E ? expf(__fsub_rn(v[i], m)) : 0.f;
      v[i] = ex;
      sd[i] = (double)ex;
    }
    // Pairwise sum (float sums of a few hundred exponentials are exact in
    // double, so the order does not matter).
#pragma unroll
    for (int w = 1; w < PER; w *= 2)
#pragma unroll
      for (int i = 0; i + w < PER; i += 2 * w) sd[i] += sd[i + w];
    double s = sd[0];
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
    const float inv = __frcp_rn((float)s);
    // Keys: bf16 probability bits above (0xFFFF - expert id), so the unsigned
    // maximum is the largest probability with ties to the lower id.
    uint32_t key[PER];
    uint32_t lb = 0;
#pragma unroll
    for (int i = 0; i < PER; ++i) {
      const int idx = lane + 32 * i;
      key[i] = idx < E ? ((uint32_t)f2bf(__fmul_rn(v[i], inv)) << 16) | (0xFFFFu - idx) : 0u;
      lb = max(lb, key[i]);
    }
    double ssum = 0.0;
    uint32_t sel = 0;
    for (int r = 0; r < k; ++r) {
      const uint32_t best = __reduce_max_sync(0xffffffffu, lb);
      if (lb == best) {  // the one lane holding it drops it and rescans
        lb = 0;
#pragma unroll
        for (int i = 0; i < PER; ++i) {
          if (key[i] == best) key[i] = 0u;
          lb = max(lb, key[i]);
        }
      }
      if (lane == r) sel = best;
      ssum += (double)bf2f(best >> 16);
    }
    const float sel_p = bf2f(sel >> 16);
    float score = sel_p;
    if (p.norm_topk) {
      const float denom = rbf((float)ssum);
      score = rbf(__fdiv_rn(sel_p, denom));
    }
    if (lane < k) {
      const int ex = 0xFFFF - (int)(sel & 0xFFFFu);
      int slot = -1;
      if (ex >= 0 && ex < E) {
        slot = s_table[ex];
        if (slot >= p.pool.cap) {
          flag_status(p.status, VB_STATUS_BOUNDS);
          slot = -1;
        } else if (slot < 0) {
          flag_status(p.status, VB_STATUS_MISS);
          slot = -1;
        }
      } else {
        flag_status(p.status, VB_STATUS_BOUNDS);
      }
      s_ex[t * k + lane] = ex;
      s_slot[t * k + lane] = slot;
      s_score[t * k + lane] = score;
      wsp<int32_t>(p, p.L.route_ok)[t * k + lane] = slot >= 0 ? 1 : 0;
      if (p.out_inds) p.out_inds[t * k + lane] = ex;
      if (p.out_scores) p.out_scores[t * k + lane] = f2bf(score);
      if (p.out_local) p.out_local[t * k + lane] = slot;
    }
  }
  __syncthreads();
  trace_mark(p.trace, 14);

  // ---- entries: shared expert first, then one entry per distinct routed
  // expert in route order (t-major, rank-minor): the first route of each
  // expert is found with an atomic minimum, first routes are numbered with
  // ballots, and every route fills its (entry, token) cell.
  const int R = T * k;
  const int shared_n = p.has_shared ? 1 : 0;
  const int r = tid;
  const bool valid = r < R && s_slot[r] >= 0;
  if (valid) atomicMin(&s_first[s_ex[r]], r);
  // Entry table defaults: slot -1 / rank -1.
  for (int i = tid; i < (R + 1) * (int)(sizeof(DecEntry) / 4); i += K1_THREADS) {
    const int f = i % (int)(sizeof(DecEntry) / 4);  // field word
    reinterpret_cast<int32_t *>(s_entries)[i] = (f >= 4 && f < 12) ? -1 : 0;
  }
  __syncthreads();
  const bool is_first = valid && s_first[s_ex[r]] == r;
  const unsigned bal = __ballot_sync(0xffffffffu, is_first);
  if (lane == 0) s_wcnt[warp] = __popc(bal);
  __syncthreads();
  if (is_first) {
    int idx = shared_n + __popc(bal & ((1u << lane) - 1u));
    for (int w = 0; w < warp; ++w) idx += s_wcnt[w];
    s_ent[r] = idx;
  }
  int n_routed = 0;
#pragma unroll
  for (int w = 0; w < K1_WARPS; ++w) n_routed += s_wcnt[w];
  __syncthreads();
  if (valid) {
    const int ei = s_ent[s_first[s_ex[r]]];
    const int tt = r / k, jj = r - tt * k;
    s_entries[ei].slot = s_slot[r];
    s_entries[ei].rank[tt] = jj;
    s_entries[ei].score[tt] = s_score[r];
  }
  if (tid == 0 && p.has_shared) {
    s_entries[0].slot = 0;
    s_entries[0].flags = 1;
    for (int q = 0; q < T; ++q) { s_entries[0].rank[q] = 0; s_entries[0].score[q] = 1.f; }
  }
  __syncthreads();
  const int n = shared_n + n_routed;
  trace_mark(p.trace, 15);
  const int words = n * (int)(sizeof(DecEntry) / 4);
  int32_t *dst = wsp<int32_t>(p, p.L.entries);
  for (int i = tid; i < words; i += K1_THREADS)
    dst[i] = reinterpret_cast<const int32_t *>(s_entries)[i];
  if (tid == 0) {
    *wsp<int32_t>(p, p.L.n_entries) = n;
    *wsp<unsigned>(p, p.L.counter) = 0u;  // ready for the next launch
  }
  span.end();
}

// ----------------------------------------------------------------------------
// K2: gate/up + SwiGLU. Persistent CTAs of W warps; an item (entry, 16
// intermediate rows) is split over the hidden dimension between the two
// warps of a pair, and each warp streams its half through its own cp.async
// ring of chunks (16 rows x 4 groups of 64 columns of gate and up plus their
// scales and biases; rows padded so that the MMA fragment reads hit distinct
// banks), RS-1 chunks ahead of the math. Item i runs on CTA i % grid, so
// every SM gets the same share. The odd warp hands its partial sums to the
// even one through shared memory (one named barrier per pair and item), which
// adds them in half order and applies SwiGLU (bf16 per op); h goes out in MMA
// fragment order for the down projection. Weights are the A operand of
// mma.m16n8k16 (4-bit codes as exact bf16 128+q, one LOP3 per pair), tokens
// the 8 B columns; per 64-column group y += s*D + (b - 128*s)*sum(x). x in
// fragment order and its group sums sit in shared memory for all warps. The
// shared expert's first chunks are requested before the PDL wait.
// ----------------------------------------------------------------------------
constexpr int K2_SMEM_MAX = 225 * 1024;

template <int H, int GS>  // GS: log2(group / 64)
struct GateUpTile {
  static constexpr int NG = H / 64;           // 64-column groups per row
  static constexpr int CG = 4;                // groups per chunk
  static constexpr int NCH = NG / CG;         // chunks per row block
  static constexpr int CPH = NCH / 2;         // chunks per half
  static constexpr int ROWB = H / 2;          // packed bytes per row
  static constexpr int CROW = CG * 32;        // chunk bytes per row (128)
  static constexpr int PITCH = CROW + 32;     // padded chunk row pitch
  static constexpr int NS = H >> (6 + GS);    // scales per row
  static constexpr int SCB = (CG >> GS) * 2;  // scale bytes per row per chunk
  static constexpr int WB = 2 * 16 * PITCH;   // gate + up codes of a chunk
  static constexpr int CHUNK = WB + 4 * 16 * SCB;
  static constexpr int RS = 3;                // ring stages per warp
  static constexpr int XB = NG * DEC_MAX_T * 4 * 8 * 4 + NG * DEC_MAX_T * 4;  // x frags, sums
  // Per warp pair: two rings, the odd warp's partials (2 slots x 32 lanes x
  // 8 floats) and the h tile (16 rows x 8 tokens).
  static constexpr int PER_PAIR = 2 * RS * CHUNK + 2048 + 512;
  static constexpr int P_FIT = (K2_SMEM_MAX - XB) / PER_PAIR;
  static constexpr int WARPS = 2 * (P_FIT < 6 ? P_FIT : 6);
  static constexpr int THREADS = 32 * WARPS;
  static constexpr int SMEM = XB + (WARPS / 2) * PER_PAIR;
  static_assert(CPH >= 1 && WARPS >= 2 && (WARPS & 1) == 0, "gate/up tile");
};

// Load 2*count bytes of bf16 scales (count in {1,2,4,8}) into a uint4.
__device__ __forceinline__ uint4 ld_scales(const uint16_t *ptr, int count) {
  uint4 r = make_uint4(0, 0, 0, 0);
  if (count >= 8) {
    r = __ldg(reinterpret_cast<const uint4 *>(ptr));
  } else if (count == 4) {
    const uint2 v = __ldg(reinterpret_cast<const uint2 *>(ptr));
    r.x = v.x;
    r.y = v.y;
  } else if (count == 2) {
    r.x = __ldg(reinterpret_cast<const unsigned *>(ptr));
  } else {
    r.x = __ldg(ptr);
  }
  return r;
}
__device__ __forceinline__ float bf_at(const uint4 &v, int i) {
  const uint32_t w = i < 2 ? v.x : (i < 4 ? v.y : (i < 6 ? v.z : v.w));
  return bf2f((i & 1) ? (w >> 16) : (w & 0xFFFF));
}
__device__ __forceinline__ float bf_lo(uint32_t w) { return __uint_as_float(w << 16); }
__device__ __forceinline__ float bf_hi(uint32_t w) { return __uint_as_float(w & 0xFFFF0000u); }
// bf16 at index i (0..3) of a 2-word vector.
__device__ __forceinline__ float bf_at2(const uint2 &v, int i) {
  const uint32_t w = i < 2 ? v.x : v.y;
  return (i & 1) ? bf_hi(w) : bf_lo(w);
}

struct GateUpItem {
  const uint8_t *gw, *uw;  // row block start of the gate and up codes
  const uint8_t *sc[4];    // row block start of gate s, gate b, up s, up b
};

template <int H, int GS>
__device__ __forceinline__ void gateup_item(const VbQuantPool &pool, int slot, int rb,
                                            GateUpItem &it) {
  using Tl = GateUpTile<H, GS>;
  it.gw = pool_ptr(pool, 0, slot) + (size_t)rb * 16 * Tl::ROWB;
  it.uw = pool_ptr(pool, 3, slot) + (size_t)rb * 16 * Tl::ROWB;
  it.sc[0] = pool_ptr(pool, 1, slot) + (size_t)rb * 16 * Tl::NS * 2;
  it.sc[1] = pool_ptr(pool, 2, slot) + (size_t)rb * 16 * Tl::NS * 2;
  it.sc[2] = pool_ptr(pool, 4, slot) + (size_t)rb * 16 * Tl::NS * 2;
  it.sc[3] = pool_ptr(pool, 5, slot) + (size_t)rb * 16 * Tl::NS * 2;
}

// Chunk ch (codes and scales) of an item into a ring stage.
template <int H, int GS>
__device__ __forceinline__ void gateup_chunk(uint8_t *stage, const GateUpItem &it, int ch,
                                             int lane) {
  using Tl = GateUpTile<H, GS>;
  // 2 matrices x 16 rows x 8 pieces of 16 bytes; lane -> piece lane%8 of
  // rows lane/8 + 4j.
  const int r0 = lane >> 3, p16 = (lane & 7) * 16;
  const uint8_t *g = it.gw + r0 * Tl::ROWB + ch * Tl::CROW + p16;
  const uint8_t *u = it.uw + r0 * Tl::ROWB + ch * Tl::CROW + p16;
  uint8_t *dg = stage + r0 * Tl::PITCH + p16;
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    cp_async16(dg + 4 * j * Tl::PITCH, g + 4 * j * Tl::ROWB);
    cp_async16(dg + 16 * Tl::PITCH + 4 * j * Tl::PITCH, u + 4 * j * Tl::ROWB);
  }
  // Scales: 4 tensors x 16 rows x SCB bytes -> [tensor][row][SCB].
#pragma unroll
  for (int k = 0; k < 2; ++k) {
    const int piece = lane + 32 * k, a = piece >> 4, r = piece & 15;
    const uint8_t *src = it.sc[a] + r * Tl::NS * 2 + ch * Tl::SCB;
    uint8_t *dst = stage + Tl::WB + piece * Tl::SCB;
    if (Tl::SCB == 8) cp_async8(dst, src);
    else cp_async4(dst, src);
  }
}

__device__ __forceinline__ void named_bar(int id, int threads) {
  asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(threads) : "memory");
}

template <int H, int GS>
__global__ void __launch_bounds__(GateUpTile<H, GS>::THREADS, 1) moe_gateup_kernel(DecodeParams p) {
  using Tl = GateUpTile<H, GS>;
  constexpr int NG = Tl::NG, CG = Tl::CG, CPH = Tl::CPH, RS = Tl::RS, W = Tl::WARPS;
  constexpr int PAIRS = W / 2;
  extern __shared__ __align__(16) uint8_t smem[];
  uint32_t *xf = reinterpret_cast<uint32_t *>(smem);                         // [NG][8][4][8] words
  float *xsm = reinterpret_cast<float *>(smem + NG * DEC_MAX_T * 4 * 8 * 4);  // [NG][8]
  __shared__ int s_slot[DEC_MAX_T * DEC_MAX_K + 1];
  __shared__ int s_n;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int g = lane >> 2, c = lane & 3;
  const int T = p.T;
  SpanTrace span(p.trace, 1);
  const int pair = warp >> 1, half = warp & 1;
  uint8_t *pbase = smem + Tl::XB + pair * Tl::PER_PAIR;
  uint8_t *ring = pbase + half * RS * Tl::CHUNK;
  float *red = reinterpret_cast<float *>(pbase + 2 * RS * Tl::CHUNK);  // [2][32][8]
  float *hbuf = red + 2 * 32 * 8;                                        // [16][8]
  const int rb_shift = 31 - __clz(p.I / 16);  // row blocks per entry = I/16
  const int RB = 1 << rb_shift;
  const int grid = gridDim.x;
  // This pair's items: blockIdx.x + grid * (pair + PAIRS * r), r = 0, 1, ...
  const int first = blockIdx.x + grid * pair, step = grid * PAIRS;

  GateUpItem cur;
  int issue_q = 0;
  auto issue_next = [&](int n_items) {
    const int r = issue_q / CPH, ch = half * CPH + issue_q % CPH;
    const int i = first + r * step;
    if (i < n_items) {
      if (issue_q % CPH == 0) {
        const int e = i >> rb_shift;
        if (p.has_shared && e == 0) gateup_item<H, GS>(p.shared, 0, i & (RB - 1), cur);
        else gateup_item<H, GS>(p.pool, s_slot[e], i & (RB - 1), cur);
      }
      gateup_chunk<H, GS>(ring + (issue_q % RS) * Tl::CHUNK, cur, ch, lane);
    }
    cp_async_commit();
    ++issue_q;
  };

  // The shared expert (entry 0) needs no routing: its chunks go first.
  const bool pre = p.has_shared && first < RB;
  if (pre) {
#pragma unroll 1
    for (int k = 0; k < RS - 1; ++k) issue_next(first + 1);
  }
  pdl_wait();
  pdl_launch_dependents();
  const int max_e = p.L.max_entries;
  if (tid == 0) s_n = *wsp<const int32_t>(p, p.L.n_entries);
  for (int i = tid; i < max_e; i += blockDim.x) s_slot[i] = wsp<const DecEntry>(p, p.L.entries)[i].slot;
  {
    // x fragments [token][group][c][8 words] -> [group][token][c][8 words],
    // group sums [token][group] -> [group][8] (zero beyond T).
    const uint4 *src = reinterpret_cast<const uint4 *>(wsp<const uint32_t>(p, p.L.xperm));
    uint4 *dst = reinterpret_cast<uint4 *>(xf);
    for (int u = tid; u < T * NG * 8; u += blockDim.x) {
      const int n = u / (NG * 8), rest = u % (NG * 8), G = rest >> 3, k = rest & 7;
      dst[(G * DEC_MAX_T + n) * 8 + k] = __ldcg(src + u);
    }
    const float *xs = wsp<const float>(p, p.L.xsum);
    for (int i = tid; i < NG * DEC_MAX_T; i += blockDim.x) {
      const int G = i >> 3, n = i & 7;
      xsm[i] = n < T ? __ldcg(xs + n * NG + G) : 0.f;
    }
  }
  __syncthreads();
  trace_mark(p.trace, 6);
  const int n_items = s_n << rb_shift;
  if (!pre) {
#pragma unroll 1
    for (int k = 0; k < RS - 1; ++k) issue_next(n_items);
  }
  if (!half && lane < 9) {
    // Whole row blocks of this pair's items into L2 in one go (contiguous
    // 16-row blocks of gate and up codes and of their four scale tensors):
    // DRAM then streams each block at once and the chunk copies hit L2.
    // Lanes 6..8 do the same for the slice of the entry's down projection
    // (rows [rb, rb + 1) * H / RB) that the next kernel reads.
    for (int i = first; i < n_items; i += step) {
      const int e = i >> rb_shift, rb = i & (RB - 1);
      const VbQuantPool &pool = (p.has_shared && e == 0) ? p.shared : p.pool;
      const int slot = (p.has_shared && e == 0) ? 0 : s_slot[e];
      if (lane < 6) {
        GateUpItem it;
        gateup_item<H, GS>(pool, slot, rb, it);
        if (lane < 2) prefetch_l2_bulk(lane ? it.uw : it.gw, 16 * Tl::ROWB);
        else prefetch_l2_bulk(it.sc[lane - 2], 16 * Tl::NS * 2);
      } else {
        const int rows = H / RB, ngi = p.I >> (6 + GS);
        const uint32_t rbytes = lane == 6 ? (uint32_t)p.I / 2 : (uint32_t)ngi * 2;
        prefetch_l2_bulk(pool_ptr(pool, lane, slot) + (size_t)rb * rows * rbytes, rows * rbytes);
      }
    }
  }

  const int NI = p.I / 64;
  float accg[4], accu[4];
#pragma unroll 1
  for (int q = 0;; ++q) {
    const int r = q / CPH, cq = q % CPH, ch = half * CPH + cq;
    const int item = first + r * step;
    if (item >= n_items) break;
    cp_async_wait<RS - 2>();
    __syncwarp();
    issue_next(n_items);  // into the stage consumed one chunk ago
    if (cq == 0) {
#pragma unroll
      for (int j = 0; j < 4; ++j) accg[j] = accu[j] = 0.f;
    }
    const uint8_t *st = ring + (q % RS) * Tl::CHUNK;
    // Scales of this chunk's groups for rows g and g+8: gate s, gate b,
    // up s, up b.
    uint2 sv[8];
#pragma unroll
    for (int a = 0; a < 8; ++a) {
      const uint8_t *sp = st + Tl::WB + ((a >> 1) * 16 + ((a & 1) ? g + 8 : g)) * Tl::SCB;
      if (Tl::SCB == 8) sv[a] = *reinterpret_cast<const uint2 *>(sp);
      else sv[a] = make_uint2(*reinterpret_cast<const uint32_t *>(sp), 0u);
    }
#pragma unroll
    for (int gl = 0; gl < CG; ++gl) {
      const int G = ch * CG + gl;
      uint4 x0 = make_uint4(0, 0, 0, 0), x1 = x0;
      if (g < T) {
        const uint4 *xp = reinterpret_cast<const uint4 *>(xf + ((G * DEC_MAX_T + g) * 4 + c) * 8);
        x0 = xp[0];
        x1 = xp[1];
      }
      const float2 xs = *reinterpret_cast<const float2 *>(xsm + G * DEC_MAX_T + 2 * c);
      const uint2 ag0 = lds64(st + g * Tl::PITCH + gl * 32 + 8 * c);
      const uint2 ag1 = lds64(st + (g + 8) * Tl::PITCH + gl * 32 + 8 * c);
      const uint2 au0 = lds64(st + (16 + g) * Tl::PITCH + gl * 32 + 8 * c);
      const uint2 au1 = lds64(st + (24 + g) * Tl::PITCH + gl * 32 + 8 * c);
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
      const int si = gl >> GS;
      const float sg0 = bf_at2(sv[0], si), sg1 = bf_at2(sv[1], si);
      const float bg0 = bf_at2(sv[2], si), bg1 = bf_at2(sv[3], si);
      const float su0 = bf_at2(sv[4], si), su1 = bf_at2(sv[5], si);
      const float bu0 = bf_at2(sv[6], si), bu1 = bf_at2(sv[7], si);
      const float bpg0 = fmaf(-128.f, sg0, bg0), bpg1 = fmaf(-128.f, sg1, bg1);
      const float bpu0 = fmaf(-128.f, su0, bu0), bpu1 = fmaf(-128.f, su1, bu1);
      accg[0] += fmaf(sg0, dg[0], bpg0 * xs.x);
      accg[1] += fmaf(sg0, dg[1], bpg0 * xs.y);
      accg[2] += fmaf(sg1, dg[2], bpg1 * xs.x);
      accg[3] += fmaf(sg1, dg[3], bpg1 * xs.y);
      accu[0] += fmaf(su0, du[0], bpu0 * xs.x);
      accu[1] += fmaf(su0, du[1], bpu0 * xs.y);
      accu[2] += fmaf(su1, du[2], bpu1 * xs.x);
      accu[3] += fmaf(su1, du[3], bpu1 * xs.y);
    }
    if (cq == CPH - 1) {
      // Pair hand-off: the odd warp's partials to the even warp.
      float *slot = red + ((r & 1) * 32 + lane) * 8;
      if (half) {
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          slot[j] = accg[j];
          slot[4 + j] = accu[j];
        }
      }
      named_bar(1 + pair, 64);
      if (!half) {
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          accg[j] += slot[j];
          accu[j] += slot[4 + j];
        }
        // SwiGLU (bf16 per op) of rows g, g+8 x tokens 2c, 2c+1, then h of
        // the 16 rows in fragment order and its per-token sums.
        const int e = item >> rb_shift, rb = item & (RB - 1);
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          const int row = (j >> 1) ? g + 8 : g, n = 2 * c + (j & 1);
          hbuf[row * 8 + n] = n < T ? swiglu_bf16(rbf(accg[j]), rbf(accu[j])) : 0.f;
        }
        __syncwarp();
        uint32_t *hperm = wsp<uint32_t>(p, p.L.hperm);
#pragma unroll
        for (int h2 = 0; h2 < 2; ++h2) {
          const int idx = lane + 32 * h2;  // (token n, word w)
          const int n = idx >> 3, w = idx & 7;
          const int m = w >> 1, pp = w & 1, j = m >> 1, i0 = 2 * (m & 1);
          const int olo = 8 * j + i0 + pp, ohi = olo + 4;
          if (n < T)
            hperm[((((size_t)e * DEC_MAX_T + n) * NI + (rb >> 2)) * 4 + (rb & 3)) * 8 + w] =
                pack_bf2(hbuf[olo * 8 + n], hbuf[ohi * 8 + n]);
        }
        if (lane < T) {
          float sh = 0.f;
#pragma unroll
          for (int o = 0; o < 16; ++o) sh += hbuf[o * 8 + lane];
          wsp<float>(p, p.L.hsum)[((size_t)e * DEC_MAX_T + lane) * (p.I / 16) + rb] = sh;
        }
        __syncwarp();
        if (r == 0) trace_mark(p.trace, 7);
      }
    }
  }
  cp_async_wait<0>();
  span.end();
}

// ----------------------------------------------------------------------------
// K3: down projection + fused combine. Persistent CTAs of 8 warps; the items
// (entry, 16 output rows) are split into contiguous entry-major ranges, one
// per warp (warps of consecutive global index sit on different SMs), so a
// warp keeps one entry's h fragments in registers across its row blocks.
// Each item's 16 weight rows and scales are copied by the warp with
// cp.async into a per-warp ring (the first ones before the PDL wait: the
// entry list is final by then); h and its group sums are read after it.
// Per route the result is rounded to bf16, times the route score, rounded
// again (MLX chain). The last warp to finish a 16-row block (atomic ticket
// per block) adds the routes of every token in rank order (exact double sum
// of bf16 values, rounded to float32 then bf16), then the gated shared
// expert and the optional residual.
// ----------------------------------------------------------------------------
constexpr int K3_THREADS = 256;
constexpr int K3_WARPS = K3_THREADS / 32;

template <int I, int GS>
struct DownTile {
  static constexpr int NGI = I / 64;
  static constexpr int ROWB = I / 2;        // packed bytes per row
  static constexpr int PITCH = ROWB + 32;   // padded smem pitch (conflict-free fragments)
  static constexpr int NSI = I >> (6 + GS); // scales per row
  static constexpr int WB = 16 * PITCH;
  static constexpr int SB = 16 * NSI * 2;   // 16 rows of one scale tensor
  static constexpr int SLOT = WB + 2 * SB;
  static constexpr int RS = 5;
  static constexpr int SMEM = K3_WARPS * RS * SLOT;
};

template <int I, int GS>
__device__ __forceinline__ void down_issue(uint8_t *slot, const VbQuantPool &pool, int pslot,
                                           int rb, int lane) {
  using Tl = DownTile<I, GS>;
  const uint8_t *dw = pool_ptr(pool, 6, pslot) + (size_t)rb * 16 * Tl::ROWB;
  constexpr int CPR = Tl::ROWB / 16;  // chunks per row
#pragma unroll
  for (int j = 0; j < 16 * CPR / 32; ++j) {
    const int q = lane + 32 * j, r = q / CPR, c16 = (q % CPR) * 16;
    cp_async16(slot + r * Tl::PITCH + c16, dw + r * Tl::ROWB + c16);
  }
  constexpr int SCH = Tl::SB / 16;  // chunks per scale tensor
  for (int q = lane; q < 2 * SCH; q += 32) {
    const int t = q / SCH, c = q % SCH;
    cp_async16(slot + Tl::WB + t * Tl::SB + c * 16,
               pool_ptr(pool, 7 + t, pslot) + (size_t)rb * Tl::SB + c * 16);
  }
}

// Rank-order combine of one 16-row block for all tokens (one warp; lane =
// token t = lane / 8 (+4 per pass), row pair 2 * (lane % 8)). Every load of a
// pass is issued before the first add.
__device__ __forceinline__ void down_combine_block(const DecodeParams &p, int rb, int lane) {
  const int T = p.T, H = p.H, k = p.k;
  const uint32_t *wp = wsp<const uint32_t>(p, p.L.wparts);
  const int32_t *okr = wsp<const int32_t>(p, p.L.route_ok);
  const int rp = 16 * rb + 2 * (lane & 7);
#pragma unroll 1
  for (int t = lane >> 3; t < T; t += 4) {
    uint32_t v[DEC_MAX_K];
    int ok[DEC_MAX_K];
#pragma unroll
    for (int j = 0; j < DEC_MAX_K; ++j) {
      if (j < k) {
        ok[j] = __ldcg(okr + t * k + j);
        v[j] = __ldcg(wp + (((size_t)t * k + j) * H + rp) / 2);
      }
    }
    float gate = 0.f;
    uint32_t sw = 0, rr = 0;
    const size_t oi = (size_t)t * H + rp;
    if (p.has_shared) {
      gate = __ldcg(wsp<const float>(p, p.L.sgate) + t);
      sw = __ldcg(wsp<const uint32_t>(p, p.L.sparts) + oi / 2);
    }
    if (p.residual) rr = __ldg(reinterpret_cast<const uint32_t *>(p.residual) + oi / 2);
    double s0 = 0.0, s1 = 0.0;
#pragma unroll
    for (int j = 0; j < DEC_MAX_K; ++j) {
      if (j < k && ok[j]) {
        s0 += (double)bf2f(v[j] & 0xFFFFu);
        s1 += (double)bf2f(v[j] >> 16);
      }
    }
    float y0 = rbf((float)s0), y1 = rbf((float)s1);
    if (p.has_shared) {
      y0 = rbf(__fadd_rn(y0, rbf(__fmul_rn(gate, bf2f(sw & 0xFFFFu)))));
      y1 = rbf(__fadd_rn(y1, rbf(__fmul_rn(gate, bf2f(sw >> 16)))));
    }
    if (p.residual) {
      y0 = rbf(__fadd_rn(bf2f(rr & 0xFFFFu), y0));
      y1 = rbf(__fadd_rn(bf2f(rr >> 16), y1));
    }
    reinterpret_cast<uint32_t *>(p.out)[oi / 2] = (uint32_t)f2bf(y0) | ((uint32_t)f2bf(y1) << 16);
  }
}

template <int I, int GS>
__global__ void __launch_bounds__(K3_THREADS, 1) moe_down_kernel(DecodeParams p) {
  using Tl = DownTile<I, GS>;
  constexpr int NGI = Tl::NGI, RS = Tl::RS;
  extern __shared__ __align__(16) uint8_t smem[];
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int g = lane >> 2, c = lane & 3;
  const int T = p.T, H = p.H;
  SpanTrace span(p.trace, 2);
  uint8_t *ring = smem + warp * RS * Tl::SLOT;
  const int RBN = H / 16;
  const int n_entries = __ldcg(wsp<const int32_t>(p, p.L.n_entries));
  const DecEntry *ents = wsp<const DecEntry>(p, p.L.entries);
  // This warp's contiguous item range (entry-major).
  const int nw = gridDim.x * K3_WARPS;
  const int wg = blockIdx.x + gridDim.x * warp;
  const int n_items = n_entries * RBN;
  const int i0 = (int)(((long long)n_items * wg) / nw);
  const int i1 = (int)(((long long)n_items * (wg + 1)) / nw);

  // The entry list is final before this kernel starts (the router ran two
  // launches back): weights are copied before the PDL wait.
  int issue_i = i0;
  auto issue_next = [&]() {
    if (issue_i < i1) {
      const int e = issue_i / RBN, rb = issue_i % RBN;
      const int2 sf = __ldcg(reinterpret_cast<const int2 *>(&ents[e]));  // slot, flags
      const bool sh = sf.y & 1;
      down_issue<I, GS>(ring + ((issue_i - i0) % RS) * Tl::SLOT, sh ? p.shared : p.pool,
                        sh ? 0 : sf.x, rb, lane);
    }
    cp_async_commit();
    ++issue_i;
  };
#pragma unroll 1
  for (int k = 0; k < RS - 1; ++k) issue_next();
  pdl_wait();
  pdl_launch_dependents();

  uint16_t *wparts = wsp<uint16_t>(p, p.L.wparts);
  uint16_t *sparts = wsp<uint16_t>(p, p.L.sparts);
  int cur_e = -1;
  uint32_t hb[NGI][8];
  float hs0[NGI], hs1[NGI];
  int rank0 = -1, rank1 = -1;
  float score0 = 0.f, score1 = 0.f;
  bool is_sh = false;
#pragma unroll 1
  for (int i = i0; i < i1; ++i) {
    const int e = i / RBN, rb = i % RBN;
    if (e != cur_e) {
      // h fragments and group sums of the entry (tokens g and 2c, 2c+1),
      // requested while the weight copy is still in flight.
      cur_e = e;
      const uint32_t *hp = wsp<const uint32_t>(p, p.L.hperm) + (size_t)e * DEC_MAX_T * (I / 2);
      const float *hsum = wsp<const float>(p, p.L.hsum) + (size_t)e * DEC_MAX_T * (I / 16);
#pragma unroll
      for (int G = 0; G < NGI; ++G) {
        uint4 a = make_uint4(0, 0, 0, 0), b = a;
        if (g < T) {
          const uint4 *src = reinterpret_cast<const uint4 *>(hp + ((size_t)g * NGI + G) * 32 + c * 8);
          a = __ldcg(src);
          b = __ldcg(src + 1);
        }
        hb[G][0] = a.x; hb[G][1] = a.y; hb[G][2] = a.z; hb[G][3] = a.w;
        hb[G][4] = b.x; hb[G][5] = b.y; hb[G][6] = b.z; hb[G][7] = b.w;
        float v0 = 0.f, v1 = 0.f;
        if (2 * c < T) {
          const float4 v = __ldcg(reinterpret_cast<const float4 *>(hsum + (size_t)(2 * c) * (I / 16) + 4 * G));
          v0 = ((v.x + v.y) + v.z) + v.w;
        }
        if (2 * c + 1 < T) {
          const float4 v = __ldcg(reinterpret_cast<const float4 *>(hsum + (size_t)(2 * c + 1) * (I / 16) + 4 * G));
          v1 = ((v.x + v.y) + v.z) + v.w;
        }
        hs0[G] = v0;
        hs1[G] = v1;
      }
      is_sh = __ldcg(&ents[e].flags) & 1;
      rank0 = 2 * c < T ? __ldcg(&ents[e].rank[2 * c]) : -1;
      rank1 = 2 * c + 1 < T ? __ldcg(&ents[e].rank[2 * c + 1]) : -1;
      score0 = 2 * c < T ? __ldcg(&ents[e].score[2 * c]) : 0.f;
      score1 = 2 * c + 1 < T ? __ldcg(&ents[e].score[2 * c + 1]) : 0.f;
    }
    cp_async_wait<RS - 2>();
    __syncwarp();
    issue_next();
    const uint8_t *st = ring + ((i - i0) % RS) * Tl::SLOT;
    float acc[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
    for (int G = 0; G < NGI; ++G) {
      const uint2 a0 = lds64(st + g * Tl::PITCH + G * 32 + 8 * c);
      const uint2 a1 = lds64(st + (g + 8) * Tl::PITCH + G * 32 + 8 * c);
      uint32_t p0[2][4], p1[2][4];
      nib_pairs4(a0.x, p0[0]);
      nib_pairs4(a0.y, p0[1]);
      nib_pairs4(a1.x, p1[0]);
      nib_pairs4(a1.y, p1[1]);
      float dd[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
      for (int m = 0; m < 4; ++m) {
        const int i0m = 2 * (m & 1), h = m >> 1;
        mma_bf16(dd, p0[h][i0m], p1[h][i0m], p0[h][i0m + 1], p1[h][i0m + 1], hb[G][2 * m],
                 hb[G][2 * m + 1]);
      }
      const int si = G >> GS;
      const uint16_t *ss = reinterpret_cast<const uint16_t *>(st + Tl::WB);
      const float s0 = bf2f(ss[g * Tl::NSI + si]), s1 = bf2f(ss[(g + 8) * Tl::NSI + si]);
      const float b0 = bf2f(ss[Tl::SB / 2 + g * Tl::NSI + si]);
      const float b1 = bf2f(ss[Tl::SB / 2 + (g + 8) * Tl::NSI + si]);
      const float bp0 = fmaf(-128.f, s0, b0), bp1 = fmaf(-128.f, s1, b1);
      acc[0] += fmaf(s0, dd[0], bp0 * hs0[G]);
      acc[1] += fmaf(s0, dd[1], bp0 * hs1[G]);
      acc[2] += fmaf(s1, dd[2], bp1 * hs0[G]);
      acc[3] += fmaf(s1, dd[3], bp1 * hs1[G]);
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
  // ---- tickets: one fence for all of this warp's items, one atomic per item
  // (lanes in parallel); the warp that completes a 16-row block combines it.
  __threadfence();
  __syncwarp();
  unsigned *cnt = wsp<unsigned>(p, p.L.rb_count);
#pragma unroll 1
  for (int base = i0; base < i1; base += 32) {
    const int i = base + lane;
    int rb = 0;
    bool win = false;
    if (i < i1) {
      rb = i % RBN;
      win = atomicAdd(cnt + rb, 1u) == (unsigned)n_entries - 1;
    }
    unsigned m = __ballot_sync(0xffffffffu, win);
    if (m) __threadfence();
    while (m) {
      const int src = __ffs(m) - 1;
      m &= m - 1;
      const int rbw = __shfl_sync(0xffffffffu, rb, src);
      down_combine_block(p, rbw, lane);
      if (lane == 0) cnt[rbw] = 0u;  // ready for the next launch
    }
  }
  span.end();
}

// One-time per-kernel attributes: the dynamic shared memory it needs and the
// largest shared-memory carveout, so that consecutive decode kernels never
// make an SM switch its L1/shared split.
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
}  // namespace

extern "C" {

size_t vb_moe_decode_workspace_size(int32_t tokens, int32_t hidden,
                                    int32_t inter, int32_t num_experts,
                                    int32_t top_k) {
  if (tokens <= 0 || hidden <= 0 || inter <= 0 || num_experts <= 0 || top_k <= 0)
    return 0;
  return decode_layout(tokens, hidden, inter, num_experts, top_k).total;
}

int vb_moe_decode(const VbMoeDecodeArgs *a, vb_stream_t stream) {
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
  VB_REQUIRE(a->x && a->router_w && a->slot_table && a->out, "vb_moe_decode: null tensor");
  VB_REQUIRE(a->pool.ptr[0] && a->pool.cap > 0, "vb_moe_decode: empty pool");
  const bool has_shared = a->shared.ptr[0] != nullptr;
  VB_REQUIRE(!has_shared || a->shared_gate_w, "vb_moe_decode: shared expert without gate");
  DecodeLayout L = decode_layout(T, H, I, E, k);
  VB_REQUIRE(a->workspace && a->workspace_bytes >= L.total,
             "vb_moe_decode: workspace %zu < %zu", a->workspace_bytes, L.total);
  VB_REQUIRE(((uintptr_t)a->workspace % 256) == 0, "vb_moe_decode: workspace must be 256-byte aligned");
  for (int i = 0; i < 9; ++i)
    VB_REQUIRE(((uintptr_t)a->pool.ptr[i] % 16) == 0 && (a->pool.slot_stride[i] % 16) == 0 &&
                   (!has_shared || (((uintptr_t)a->shared.ptr[i] % 16) == 0)),
               "vb_moe_decode: pool tensors and slot strides must be 16-byte aligned");

  DecodeParams p;
  p.T = T; p.H = H; p.I = I; p.E = E; p.k = k; p.norm_topk = a->norm_topk;
  p.norm_eps = a->norm_eps;
  p.gshift = a->group == 128 ? 1 : 0;
  p.has_shared = has_shared ? 1 : 0;
  p.x = a->x; p.router_w = a->router_w; p.shared_gate_w = a->shared_gate_w;
  p.residual = a->residual; p.router_bias = a->router_bias; p.table = a->slot_table;
  p.pool = a->pool; p.shared = a->shared;
  p.out = a->out; p.out_scores = a->out_scores; p.out_inds = a->out_inds;
  p.out_local = a->out_local; p.status = a->status;
  p.ws = static_cast<uint8_t *>(a->workspace);
  p.trace = a->trace;
  p.L = L;

  void (*k1)(DecodeParams) = nullptr;
  void (*k2)(DecodeParams) = nullptr;
  const int per = E <= 256 ? 8 : (E <= 512 ? 16 : 32);
#define VB_K1(HH) (per == 8 ? moe_router_kernel<HH, 8> : per == 16 ? moe_router_kernel<HH, 16> \
                                                      : moe_router_kernel<HH, 32>)
  size_t k2_smem = 0;
  int k2_threads = 0;
#define VB_K2(HH)                                                             \
  do {                                                                        \
    k1 = VB_K1(HH);                                                           \
    if (p.gshift) {                                                           \
      k2 = moe_gateup_kernel<HH, 1>;                                          \
      k2_smem = GateUpTile<HH, 1>::SMEM;                                      \
      k2_threads = GateUpTile<HH, 1>::THREADS;                                \
    } else {                                                                  \
      k2 = moe_gateup_kernel<HH, 0>;                                          \
      k2_smem = GateUpTile<HH, 0>::SMEM;                                      \
      k2_threads = GateUpTile<HH, 0>::THREADS;                                \
    }                                                                         \
  } while (0)
  switch (H) {
    case 512: VB_K2(512); break;
    case 1024: VB_K2(1024); break;
    case 2048: VB_K2(2048); break;
    default: VB_K2(4096); break;
  }
#undef VB_K2
#undef VB_K1
  void (*k3)(DecodeParams) = nullptr;
  size_t k3_smem = 0;
#define VB_K3(II)                                                 \
  do {                                                            \
    if (p.gshift) {                                               \
      k3 = moe_down_kernel<II, 1>;                                \
      k3_smem = DownTile<II, 1>::SMEM;                            \
    } else {                                                      \
      k3 = moe_down_kernel<II, 0>;                                \
      k3_smem = DownTile<II, 0>::SMEM;                            \
    }                                                             \
  } while (0)
  switch (I) {
    case 128: VB_K3(128); break;
    case 256: VB_K3(256); break;
    default: VB_K3(512); break;
  }
#undef VB_K3

  cudaStream_t s = as_stream(stream);
  cudaEvent_t *ev = a->timing_events ? (cudaEvent_t *)a->timing_events : nullptr;
  const bool pdl = ev == nullptr;  // event records would break the PDL chain
  // K1 is a PDL secondary of whatever ran before it on the stream (the
  // previous block's down kernel): it only reads weights before the wait.
  if (ev) cudaEventRecord(ev[0], s);
  const size_t smem1 = (size_t)T * H * 2;
  cudaError_t err = decode_kernel_attrs((const void *)k1, smem1);
  if (err == cudaSuccess) err = decode_kernel_attrs((const void *)k2, k2_smem);
  if (err == cudaSuccess) err = decode_kernel_attrs((const void *)k3, k3_smem);
  if (err != cudaSuccess) return set_error(VB_ERR_CUDA, "decode kernel attributes: %s", cudaGetErrorString(err));
  const int rpc = K1_WARPS / (H >= 1024 ? 4 : 2);
  const int grid1 = (E + (has_shared ? 1 : 0) + rpc - 1) / rpc;
  err = vb_launch(k1, dim3(grid1), dim3(K1_THREADS), smem1, s, pdl, p);
  if (err != cudaSuccess) return set_error(VB_ERR_CUDA, "moe_router_kernel: %s", cudaGetErrorString(err));
  if (ev) cudaEventRecord(ev[1], s);

  {
    const int grid2 = std::min(sm_count(), L.max_entries * (I / 16));
    err = vb_launch(k2, dim3(grid2), dim3(k2_threads), k2_smem, s, pdl, p);
  }
  if (err != cudaSuccess) return set_error(VB_ERR_CUDA, "moe_gateup_kernel: %s", cudaGetErrorString(err));
  if (ev) cudaEventRecord(ev[2], s);

  err = vb_launch(k3, dim3(std::min(sm_count(), L.max_entries * (H / 16))), dim3(K3_THREADS),
                  k3_smem, s, pdl, p);
  if (err != cudaSuccess) return set_error(VB_ERR_CUDA, "moe_down_kernel: %s", cudaGetErrorString(err));
  if (ev) cudaEventRecord(ev[3], s);
  return VB_OK;
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
  // The array keeps the previous call's contents: zero the words the kernels
  // expect at zero (route ticket, entry count, shared gates, row-block
  // tickets) before this call's kernels, in stream order.
  const DecodeLayout L = decode_layout(a->tokens, a->hidden, a->inter, a->num_experts, a->top_k);
  const size_t clear = L.zero_end;
  const cudaError_t e = cudaMemsetAsync(scratch, 0, clear, as_stream(stream));
  if (e != cudaSuccess)
    return set_error(VB_ERR_CUDA, "vb_moe_decode_noalloc: clearing scratch: %s", cudaGetErrorString(e));
  VbMoeDecodeArgs b = *a;
  b.workspace = scratch;
  b.workspace_bytes = VB_MOE_DECODE_NOALLOC_SCRATCH_BYTES;
  return vb_moe_decode(&b, stream);
}

}  // extern "C"
