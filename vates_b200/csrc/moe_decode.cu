// Decode / MTP-verify fused MoE block (T <= 8 tokens), MLX bf16 dtype chain.
//
// Reference: FileStreamingMoeBlock.__call__ (mlx_streaming/core/moe/block.py
// :245-1013) with PersistentSubGLU.forward (compute.py:145-199) and the
// shared expert (block.py:102-109, 1009-1012).
//
// Four kernels per block, chained with programmatic dependent launch (PDL):
//  K1 router: optional unit RMSNorm of x, logits = bf16(x.Wr^T [+bias]) with
//     one warp per expert row (row loaded before the PDL wait). The last CTA
//     (atomic ticket) runs the precise softmax, top-k (lower id wins ties),
//     renormalisation and slot gather, and writes the list of "entries":
//     the shared expert first, then every distinct routed slot. All CTAs
//     share writing x in MMA-fragment order (xperm), per-64-column sums
//     (xsum) and the shared-expert gate sigmoid(x.w_sg).
//  K2 gate/up: persistent CTAs walk items (entry, 16 intermediate rows). All
//     512 threads stream an item's packed rows and scales into a multi-stage
//     cp.async ring (per-thread copy offsets are fixed at kernel start; H is a
//     template constant). Weights are the A operand of mma.m16n8k16 (16 rows
//     x 16 columns), tokens the 8 B columns: 4-bit codes become the exact
//     bf16 values 128+q with one LOP3 per pair, so per 64-column group the
//     epilogue applies y += s*D + (b - 128*s)*sum(x). 16 warps split the
//     hidden dimension and their partials are added in warp order; SwiGLU
//     (bf16 per op) follows and h is stored in fragment order (hperm).
//     The shared expert's weights are requested before the PDL wait.
//  K3 down: persistent CTAs walk items (entry, 128 output rows), weights
//     requested before the PDL wait; per route the result is rounded to
//     bf16, multiplied by the route score and rounded again (MLX chain).
//  K4 combine: per token and column, the k routes are added in rank order
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
constexpr int DEC_ROUTER_WARPS = 4;
constexpr int DEC_SMEM_BUDGET = 200 * 1024;

struct DecEntry {
  int32_t slot;
  int32_t flags;  // bit0 = shared expert
  int32_t pad[2];
  int32_t rank[DEC_MAX_T];  // route rank of token n, -1 = not routed here
  float score[DEC_MAX_T];   // bf16 route score
};

struct DecodeLayout {
  size_t counter, n_entries, sgate, rb_count, logits, entries, route_ok, xperm, xsum, hperm,
      hsum, wparts, sparts, total;
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
  L.rb_count = off; off += sizeof(unsigned) * (H / 128);
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

__device__ __forceinline__ const uint8_t *pool_ptr(const VbQuantPool &pool, int t, int slot) {
  return (const uint8_t *)pool.ptr[t] + (size_t)slot * pool.slot_stride[t];
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
// so that every index is a shift.
// ----------------------------------------------------------------------------
template <int H, int PER>  // PER = ceil(E / 32) logits per lane
__global__ void __launch_bounds__(DEC_ROUTER_WARPS * 32)
moe_router_kernel(DecodeParams p) {
  constexpr int NVL = H / 256;  // uint4 of a row per lane
  constexpr int NG = H / 64;
  extern __shared__ __align__(16) uint8_t smem_raw[];
  uint16_t *xs = reinterpret_cast<uint16_t *>(smem_raw);  // [T][H] bf16
  const int T = p.T, E = p.E;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  SpanTrace span(p.trace, 0);

  // Router row of this warp and (CTAs t < T, warp 0) the shared-expert gate
  // row: both independent of the previous kernel.
  const int e = blockIdx.x * DEC_ROUTER_WARPS + warp;
  uint4 wv[NVL];
  if (e < E) {
    const uint4 *wrow = reinterpret_cast<const uint4 *>(p.router_w + (size_t)e * H);
#pragma unroll
    for (int u = 0; u < NVL; ++u) wv[u] = ldg_nc_v4(wrow + u * 32 + lane);
  }
  const bool gate_cta = p.has_shared && (int)blockIdx.x < T && warp == 0;
  uint4 gv[NVL];
  if (gate_cta) {
    const uint4 *grow = reinterpret_cast<const uint4 *>(p.shared_gate_w);
#pragma unroll
    for (int u = 0; u < NVL; ++u) gv[u] = ldg_nc_v4(grow + u * 32 + lane);
  }
  if (p.has_shared && tid == 0) {
    // The shared expert is fixed per layer: stream it into L2 right away.
    const int np = expert_pieces(p, 0, 9);
    for (int i = blockIdx.x; i < np; i += gridDim.x) prefetch_expert_piece(p, p.shared, 0, 0, i);
  }
  pdl_wait();
  pdl_launch_dependents();
  trace_mark(p.trace, 8);

  {
    // Stage x: independent 16-byte loads issued before the stores.
    const uint4 *src = reinterpret_cast<const uint4 *>(p.x);
    uint4 *dst = reinterpret_cast<uint4 *>(xs);
    const int nvec = T * (H / 8);
    constexpr int STEP = DEC_ROUTER_WARPS * 32;
    for (int base = 0; base < nvec; base += 8 * STEP) {
      uint4 v[8];
#pragma unroll
      for (int u = 0; u < 8; ++u) {
        const int i = base + u * STEP + tid;
        if (i < nvec) v[u] = __ldcg(src + i);
      }
#pragma unroll
      for (int u = 0; u < 8; ++u) {
        const int i = base + u * STEP + tid;
        if (i < nvec) dst[i] = v[u];
      }
    }
  }
  __syncthreads();
  trace_mark(p.trace, 11);
  if (p.norm_eps > 0.f) {
    // Unit-weight RMSNorm of the block input (decoder post-attention norm):
    // y = bf16(x * (1/sqrt(mean(x^2) + eps))), float32 math with an exact
    // (double) sum of squares. Every CTA computes it identically.
    __shared__ float s_inv[DEC_MAX_T];
    for (int t = warp; t < T; t += DEC_ROUTER_WARPS) {
      double ss = 0.0;
#pragma unroll
      for (int u = 0; u < NVL; ++u) {
        const uint4 v = reinterpret_cast<const uint4 *>(xs + (size_t)t * H)[u * 32 + lane];
        const uint32_t w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          const double a = bf2f(w[q] & 0xFFFF), b = bf2f(w[q] >> 16);
          ss = fma(a, a, ss);
          ss = fma(b, b, ss);
        }
      }
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
      if (lane == 0) {
        const float ms = __fdiv_rn((float)ss, (float)H);
        s_inv[t] = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(ms, p.norm_eps)));
      }
    }
    __syncthreads();
    for (int i = tid; i < T * (H / 8); i += blockDim.x) {
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
  if (e < E) {
    float acc[DEC_MAX_T];
#pragma unroll
    for (int t = 0; t < DEC_MAX_T; ++t) acc[t] = 0.f;
#pragma unroll
    for (int u = 0; u < NVL; ++u) {
      const int v = u * 32 + lane;
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
        if (lane == 0) {
          if (p.router_bias) a = a + p.router_bias[e];
          wsp<float>(p, p.L.logits)[(size_t)t * E + e] = rbf(a);
        }
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
    const int gwarp = blockIdx.x * DEC_ROUTER_WARPS + warp;
    const int nwarps = gridDim.x * DEC_ROUTER_WARPS;
    for (int it = gwarp; it < T * NG; it += nwarps) {
      const int n = it / NG, G = it % NG;
      const uint32_t v = reinterpret_cast<const uint32_t *>(xs + (size_t)n * H + 64 * G)[lane];
      float s = bf2f(v & 0xFFFF) + bf2f(v >> 16);
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
      if (lane == 0) xsum[it] = s;
    }
    for (int t = blockIdx.x; gate_cta && t < T; t += gridDim.x) {
      float a = 0.f;
#pragma unroll
      for (int u = 0; u < NVL; ++u) {
        const uint32_t gr[4] = {gv[u].x, gv[u].y, gv[u].z, gv[u].w};
        const uint4 xv = reinterpret_cast<const uint4 *>(xs + (size_t)t * H)[u * 32 + lane];
        const uint32_t xr[4] = {xv.x, xv.y, xv.z, xv.w};
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          a = fmaf(bf2f(gr[q] & 0xFFFF), bf2f(xr[q] & 0xFFFF), a);
          a = fmaf(bf2f(gr[q] >> 16), bf2f(xr[q] >> 16), a);
        }
      }
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) a += __shfl_xor_sync(0xffffffffu, a, o);
      if (lane == 0) wsp<float>(p, p.L.sgate)[t] = rbf(mlx_sigmoid(rbf(a)));
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
  __shared__ int s_slot[DEC_MAX_T * DEC_MAX_K];
  __shared__ float s_score[DEC_MAX_T * DEC_MAX_K];
  __shared__ int s_first[DEC_MAX_T * DEC_MAX_K];  // 1 = first route of its slot
  __shared__ int s_ent[DEC_MAX_T * DEC_MAX_K];
  __shared__ __align__(16) DecEntry s_entries[DEC_MAX_T * DEC_MAX_K + 1];
  const int k = p.k;
  const float *logits = wsp<float>(p, p.L.logits);
  for (int t = warp; t < T; t += DEC_ROUTER_WARPS) {
    float v[PER];
    float m = -INFINITY;
#pragma unroll
    for (int i = 0; i < PER; ++i) {
      const int idx = lane + 32 * i;
      v[i] = idx < E ? __ldcg(logits + (size_t)t * E + idx) : -INFINITY;
      m = fmaxf(m, v[i]);
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
    double s = 0.0;
#pragma unroll
    for (int i = 0; i < PER; ++i) {
      const int idx = lane + 32 * i;
      const float ex = idx < E ? expf(__fsub_rn(v[i], m)) : 0.f;
      v[i] = ex;
      s += (double)ex;
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
    const float inv = __frcp_rn((float)s);
    // Probabilities (bf16) and this lane's running maximum; ties resolve to
    // the lower expert id.
    float lb = -INFINITY;
    int li = 0x7fffffff;
#pragma unroll
    for (int i = 0; i < PER; ++i) {
      const int idx = lane + 32 * i;
      v[i] = idx < E ? rbf(__fmul_rn(v[i], inv)) : -INFINITY;
      if (v[i] > lb) { lb = v[i]; li = idx; }
    }
    double ssum = 0.0;
    float sel_p = 0.f;
    int sel_e = 0;
    for (int r = 0; r < k; ++r) {
      float bv = lb;
      int bi = li;
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) {
        const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
        const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
        if (ov > bv || (ov == bv && oi < bi)) { bv = ov; bi = oi; }
      }
      if ((bi & 31) == lane) {  // winner: drop the value, rescan this lane
        lb = -INFINITY;
        li = 0x7fffffff;
#pragma unroll
        for (int i = 0; i < PER; ++i) {
          const int idx = lane + 32 * i;
          if (idx == bi) v[i] = -INFINITY;
          if (v[i] > lb) { lb = v[i]; li = idx; }
        }
      }
      if (lane == r) { sel_p = bv; sel_e = bi; }
      ssum += (double)bv;
    }
    float score = sel_p;
    if (p.norm_topk) {
      const float denom = rbf((float)ssum);
      score = rbf(__fdiv_rn(sel_p, denom));
    }
    if (lane < k) {
      const int ex = sel_e;
      int slot = -1;
      if (ex >= 0 && ex < E) {
        slot = __ldg(p.table + ex);
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
      s_slot[t * k + lane] = slot;
      s_score[t * k + lane] = score;
      wsp<int32_t>(p, p.L.route_ok)[t * k + lane] = slot >= 0 ? 1 : 0;
      if (p.out_inds) p.out_inds[t * k + lane] = ex;
      if (p.out_scores) p.out_scores[t * k + lane] = f2bf(score);
      if (p.out_local) p.out_local[t * k + lane] = slot;
    }
  }
  trace_mark(p.trace, 14);
  // Entry table in shared memory: slot -1 / rank -1 defaults.
  for (int i = tid; i < (DEC_MAX_T * DEC_MAX_K + 1) * (int)(sizeof(DecEntry) / 4);
       i += blockDim.x) {
    const int f = i % (int)(sizeof(DecEntry) / 4);  // field word
    reinterpret_cast<int32_t *>(s_entries)[i] = (f >= 4 && f < 12) ? -1 : 0;
  }
  __syncthreads();

  // ---- entries: shared expert first, then the distinct routed slots in
  // route order (t-major, rank-minor). One thread per route: it finds the
  // first route with its slot, first routes are numbered by counting the
  // earlier first routes, and every route fills its (entry, token) cell.
  const int R = T * k;
  const int shared_n = p.has_shared ? 1 : 0;
  const int r = tid;
  const int slot = r < R ? s_slot[r] : -1;
  int first = r;
#pragma unroll 8
  for (int q = 0; q < R; ++q) {
    const int sq = s_slot[q];
    first = (q < first && sq == slot) ? q : first;
  }
  const bool is_first = slot >= 0 && first == r;
  if (r < R) s_first[r] = is_first ? 1 : 0;
  const int n_routed = __syncthreads_count(is_first);
  if (is_first) {
    int idx = shared_n;
#pragma unroll 8
    for (int q = 0; q < r; ++q) idx += s_first[q];
    s_ent[r] = idx;
  }
  __syncthreads();
  if (r < R && slot >= 0) {
    const int ei = s_ent[first];
    const int tt = r / k, jj = r - tt * k;
    s_entries[ei].slot = slot;
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
  for (int i = tid; i < words; i += blockDim.x)
    dst[i] = reinterpret_cast<const int32_t *>(s_entries)[i];
  if (tid == 0) {
    *wsp<int32_t>(p, p.L.n_entries) = n;
    *wsp<unsigned>(p, p.L.counter) = 0u;  // ready for the next launch
  }
  span.end();
}

// ----------------------------------------------------------------------------
// K2: gate/up + SwiGLU, persistent. One CTA per SM walks the items (entry,
// 16 intermediate rows) b, b + grid, ... An item's 16 gate rows, 16 up rows
// and their scales/biases (each contiguous in the pool) are copied by all
// threads with 16-byte cp.async into an S-stage shared-memory ring, S-1
// items ahead of the math. Rows are padded by 32 bytes so that the MMA
// fragment reads (row g, 8 bytes at column 8c) fall in distinct banks. The
// shared expert's item is requested before the PDL wait. The 8 warps split
// the hidden dimension (GPW groups of 64 columns each); their partials are
// added in warp order, then SwiGLU (bf16 per op) and h in fragment order.
// ----------------------------------------------------------------------------
constexpr int K2_SMEM_MAX = 200 * 1024;

template <int H, int GS>  // GS: log2(group / 64)
struct GateUpTile {
  static constexpr int NG = H / 64;
  static constexpr int WARPS = NG < 16 ? NG : 16;
  static constexpr int THREADS = 32 * WARPS;
  static constexpr int GPW = NG / WARPS;
  static constexpr int NS = H >> (6 + GS);          // scales per row
  static constexpr int SC = GPW >> GS ? GPW >> GS : 1;  // scales per warp row slice
  static constexpr int ROWB = H / 2;                // packed bytes per row
  static constexpr int PITCH = ROWB + 32;           // padded smem row pitch
  static constexpr int WBYTES = 16 * PITCH;         // 16 rows of one matrix
  static constexpr int SBYTES = 16 * NS * 2;        // 16 rows of one scale tensor
  static constexpr int SCH = SBYTES / 16;           // its 16-byte chunks
  static constexpr int STAGE = 2 * WBYTES + 4 * SBYTES;
  static constexpr int S = (K2_SMEM_MAX / STAGE) < 6 ? (K2_SMEM_MAX / STAGE) : 6;
  static constexpr int CPR = ROWB / 16;             // 16-byte chunks per row
  static constexpr int RSTEP = THREADS / CPR;       // rows per copy pass
  static constexpr int PASSES = 16 / RSTEP;
  static constexpr int SMEM = S * STAGE;
  static_assert(S >= 2 && RSTEP >= 1 && PASSES * RSTEP == 16, "gate/up tile");
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

// bf16 scales (count in {1,2,4,8}) from shared memory into a uint4.
__device__ __forceinline__ uint4 lds_scales(const uint8_t *ptr, int count) {
  uint4 r = make_uint4(0, 0, 0, 0);
  if (count >= 8) {
    r = *reinterpret_cast<const uint4 *>(ptr);
  } else if (count == 4) {
    const uint2 v = *reinterpret_cast<const uint2 *>(ptr);
    r.x = v.x;
    r.y = v.y;
  } else if (count == 2) {
    r.x = *reinterpret_cast<const unsigned *>(ptr);
  } else {
    r.x = *reinterpret_cast<const uint16_t *>(ptr);
  }
  return r;
}
__device__ __forceinline__ float bf_at(const uint4 &v, int i) {
  const uint32_t w = i < 2 ? v.x : (i < 4 ? v.y : (i < 6 ? v.z : v.w));
  return bf2f((i & 1) ? (w >> 16) : (w & 0xFFFF));
}

// Copy item (expert tensors `base`, row block rb) into one ring stage.
// base: gate w, gate s, gate b, up w, up s, up b of the expert's slot.
template <int H, int GS>
__device__ __forceinline__ void gateup_issue(uint8_t *stage, const uint8_t *const (&base)[6],
                                             int rb, int tid) {
  using Tl = GateUpTile<H, GS>;
  const int r0 = tid / Tl::CPR, c16 = (tid % Tl::CPR) * 16;
  const uint8_t *gw = base[0] + (size_t)(16 * rb) * Tl::ROWB;
  const uint8_t *uw = base[3] + (size_t)(16 * rb) * Tl::ROWB;
#pragma unroll
  for (int j = 0; j < Tl::PASSES; ++j) {
    const int r = r0 + j * Tl::RSTEP;
    cp_async16(stage + r * Tl::PITCH + c16, gw + r * Tl::ROWB + c16);
    cp_async16(stage + Tl::WBYTES + r * Tl::PITCH + c16, uw + r * Tl::ROWB + c16);
  }
  // Scale tensors (16 rows x NS bf16 each), compact in shared memory.
#pragma unroll
  for (int q0 = 0; q0 < 4 * Tl::SCH; q0 += Tl::THREADS) {
    const int q = q0 + tid;
    if (q < 4 * Tl::SCH) {
      const int a = q / Tl::SCH, c = q % Tl::SCH;
      const uint8_t *t = a == 0 ? base[1] : a == 1 ? base[2] : a == 2 ? base[4] : base[5];
      cp_async16(stage + 2 * Tl::WBYTES + a * Tl::SBYTES + c * 16,
                 t + (size_t)rb * Tl::SBYTES + c * 16);
    }
  }
}

template <int H, int GS>
__global__ void __launch_bounds__(GateUpTile<H, GS>::THREADS, 1) moe_gateup_kernel(DecodeParams p) {
  using Tl = GateUpTile<H, GS>;
  constexpr int NG = Tl::NG;
  constexpr int GPW = Tl::GPW;
  constexpr int S = Tl::S;
  constexpr int WARPS = Tl::WARPS;
  extern __shared__ __align__(16) uint8_t ring[];
  __shared__ float red[WARPS][256];
  __shared__ float hval[128];
  __shared__ int s_slot[DEC_MAX_T * DEC_MAX_K + 1];
  __shared__ int s_n;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int g = lane >> 2, c = lane & 3;
  const int T = p.T;
  SpanTrace span(p.trace, 1);
  const int G0 = warp * GPW;
  const int rb_shift = 31 - __clz(p.I / 16);  // items per entry = I/16
  const int RB = 1 << rb_shift;
  const int b = blockIdx.x, grid = gridDim.x;

  auto bases = [&](const VbQuantPool &pool, int slot, const uint8_t *(&base)[6]) {
#pragma unroll
    for (int t = 0; t < 6; ++t) base[t] = pool_ptr(pool, t, slot);
  };
  // The shared expert (entry 0) needs no routing: its item goes first.
  const bool pre = p.has_shared && b < RB;
  if (pre) {
    const uint8_t *base[6];
    bases(p.shared, 0, base);
    gateup_issue<H, GS>(ring, base, b, tid);
  }
  cp_async_commit();
  pdl_wait();
  pdl_launch_dependents();
  const int max_e = p.L.max_entries;
  if (tid == 0) s_n = *wsp<const int32_t>(p, p.L.n_entries);
  if (tid < max_e) s_slot[tid] = wsp<const DecEntry>(p, p.L.entries)[tid].slot;
  __syncthreads();
  trace_mark(p.trace, 6);
  const int n_items = s_n << rb_shift;
  auto issue = [&](int k) {
    const int i = b + k * grid;
    if (i < n_items) {
      const int e = i >> rb_shift;
      const uint8_t *base[6];
      if (p.has_shared && e == 0) bases(p.shared, 0, base);
      else bases(p.pool, s_slot[e], base);
      gateup_issue<H, GS>(ring + (k % S) * Tl::STAGE, base, i & (RB - 1), tid);
    }
  };
  if (!pre) issue(0);
  cp_async_commit();
#pragma unroll 1
  for (int k = 1; k < S - 1; ++k) {
    issue(k);
    cp_async_commit();
  }

  // x fragments and column sums of this warp's groups (written by the router).
  uint4 xb[GPW][2];
  float xs0[GPW], xs1[GPW];
  {
    const uint32_t *xperm = wsp<const uint32_t>(p, p.L.xperm);
    const float *xsum = wsp<const float>(p, p.L.xsum);
#pragma unroll
    for (int i = 0; i < GPW; ++i) {
      const int G = G0 + i;
      if (g < T) {
        const uint4 *src = reinterpret_cast<const uint4 *>(xperm + (((size_t)g * NG + G) * 4 + c) * 8);
        xb[i][0] = __ldcg(src);
        xb[i][1] = __ldcg(src + 1);
      } else {
        xb[i][0] = xb[i][1] = make_uint4(0, 0, 0, 0);
      }
      xs0[i] = 2 * c < T ? __ldcg(xsum + (2 * c) * NG + G) : 0.f;
      xs1[i] = 2 * c + 1 < T ? __ldcg(xsum + (2 * c + 1) * NG + G) : 0.f;
    }
  }

  const int NI = p.I / 64;
#pragma unroll 1
  for (int k = 0; b + k * grid < n_items; ++k) {
    cp_async_wait<S - 2>();
    __syncthreads();
    issue(k + S - 1);
    cp_async_commit();
    const int item = b + k * grid;
    const int e = item >> rb_shift, rb = item & (RB - 1);
    const uint8_t *st = ring + (k % S) * Tl::STAGE;

    uint4 sv[8];  // gate_s r0, r1, gate_b r0, r1, up_s r0, r1, up_b r0, r1
    {
      const int s0 = G0 >> GS;
#pragma unroll
      for (int a = 0; a < 8; ++a) {
        const int row = (a & 1) ? g + 8 : g;
        sv[a] = lds_scales(st + 2 * Tl::WBYTES + (a >> 1) * Tl::SBYTES + (row * Tl::NS + s0) * 2,
                           Tl::SC);
      }
    }
    float accg[4] = {0.f, 0.f, 0.f, 0.f}, accu[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
    for (int i = 0; i < GPW; ++i) {
      const int col = (G0 + i) * 32 + 8 * c;
      const uint2 ag0 = lds64(st + g * Tl::PITCH + col);
      const uint2 ag1 = lds64(st + (g + 8) * Tl::PITCH + col);
      const uint2 au0 = lds64(st + Tl::WBYTES + g * Tl::PITCH + col);
      const uint2 au1 = lds64(st + Tl::WBYTES + (g + 8) * Tl::PITCH + col);
      const int si = i >> GS;
      const float sg0 = bf_at(sv[0], si), sg1 = bf_at(sv[1], si);
      const float bg0 = bf_at(sv[2], si), bg1 = bf_at(sv[3], si);
      const float su0 = bf_at(sv[4], si), su1 = bf_at(sv[5], si);
      const float bu0 = bf_at(sv[6], si), bu1 = bf_at(sv[7], si);
      float dg[4] = {0.f, 0.f, 0.f, 0.f}, du[4] = {0.f, 0.f, 0.f, 0.f};
      const uint32_t xw[8] = {xb[i][0].x, xb[i][0].y, xb[i][0].z, xb[i][0].w,
                              xb[i][1].x, xb[i][1].y, xb[i][1].z, xb[i][1].w};
#pragma unroll
      for (int m = 0; m < 4; ++m) {
        const int i0 = 2 * (m & 1);
        const uint32_t wa = (m >> 1) ? ag0.y : ag0.x;
        const uint32_t wb = (m >> 1) ? ag1.y : ag1.x;
        mma_bf16(dg, nib_pair(wa, i0), nib_pair(wb, i0), nib_pair(wa, i0 + 1),
                 nib_pair(wb, i0 + 1), xw[2 * m], xw[2 * m + 1]);
        const uint32_t va = (m >> 1) ? au0.y : au0.x;
        const uint32_t vb2 = (m >> 1) ? au1.y : au1.x;
        mma_bf16(du, nib_pair(va, i0), nib_pair(vb2, i0), nib_pair(va, i0 + 1),
                 nib_pair(vb2, i0 + 1), xw[2 * m], xw[2 * m + 1]);
      }
      const float bpg0 = fmaf(-128.f, sg0, bg0), bpg1 = fmaf(-128.f, sg1, bg1);
      const float bpu0 = fmaf(-128.f, su0, bu0), bpu1 = fmaf(-128.f, su1, bu1);
      accg[0] += fmaf(sg0, dg[0], bpg0 * xs0[i]);
      accg[1] += fmaf(sg0, dg[1], bpg0 * xs1[i]);
      accg[2] += fmaf(sg1, dg[2], bpg1 * xs0[i]);
      accg[3] += fmaf(sg1, dg[3], bpg1 * xs1[i]);
      accu[0] += fmaf(su0, du[0], bpu0 * xs0[i]);
      accu[1] += fmaf(su0, du[1], bpu0 * xs1[i]);
      accu[2] += fmaf(su1, du[2], bpu1 * xs0[i]);
      accu[3] += fmaf(su1, du[3], bpu1 * xs1[i]);
    }
    float *rw = red[warp];
    *reinterpret_cast<float2 *>(rw + g * 8 + 2 * c) = make_float2(accg[0], accg[1]);
    *reinterpret_cast<float2 *>(rw + (g + 8) * 8 + 2 * c) = make_float2(accg[2], accg[3]);
    *reinterpret_cast<float2 *>(rw + 128 + g * 8 + 2 * c) = make_float2(accu[0], accu[1]);
    *reinterpret_cast<float2 *>(rw + 128 + (g + 8) * 8 + 2 * c) = make_float2(accu[2], accu[3]);
    __syncthreads();
    if (tid < 128) {
      // Add the warp partials in warp order, then SwiGLU (bf16 per op).
      float sg = 0.f, su = 0.f;
#pragma unroll
      for (int w = 0; w < WARPS; ++w) {
        sg += red[w][tid];
        su += red[w][128 + tid];
      }
      hval[tid] = (tid & 7) < T ? swiglu_bf16(rbf(sg), rbf(su)) : 0.f;
    }
    __syncthreads();
    if (tid < 64) {
      // The 16 rows of h form quarter c' = rb%4 of intermediate group rb/4.
      const int n = tid >> 3, w = tid & 7;
      const int m = w >> 1, pp = w & 1, j = m >> 1, i0 = 2 * (m & 1);
      const int olo = 8 * j + i0 + pp, ohi = olo + 4;
      const uint32_t word = pack_bf2(hval[olo * 8 + n], hval[ohi * 8 + n]);
      uint32_t *hperm = wsp<uint32_t>(p, p.L.hperm);
      hperm[((((size_t)e * DEC_MAX_T + n) * NI + (rb >> 2)) * 4 + (rb & 3)) * 8 + w] = word;
    } else if (tid < 72) {
      const int n = tid - 64;
      float sh = 0.f;
#pragma unroll
      for (int o = 0; o < 16; ++o) sh += hval[o * 8 + n];
      wsp<float>(p, p.L.hsum)[((size_t)e * DEC_MAX_T + n) * (p.I / 16) + rb] = sh;
    }
    if (k == 0) trace_mark(p.trace, 7);
  }
  cp_async_wait<0>();
  span.end();
}

// ----------------------------------------------------------------------------
// K3: down projection + fused combine. One CTA per (entry, 128 output rows),
// warp w owns rows [16w, 16w+16). Weights are requested before the PDL wait;
// h is staged in shared memory after it. The last CTA of a 128-row block
// (atomic ticket per block) adds the routes of every token in rank order
// (exact double sum of bf16 values, rounded to float32 then bf16), then the
// gated shared expert and the optional residual.
// ----------------------------------------------------------------------------
constexpr int K3_THREADS = 256;

template <int I>
__global__ void __launch_bounds__(K3_THREADS, 2) moe_down_kernel(DecodeParams p) {
  constexpr int NGI = I / 64;
  constexpr int HW = I / 2 + 4;  // words per staged h column (+16 B pad)
  __shared__ __align__(16) uint32_t hsm[DEC_MAX_T][HW];
  __shared__ __align__(16) float hs_sm[DEC_MAX_T][I / 16];
  __shared__ int s_slot, s_n, s_flags;
  __shared__ int s_rank[DEC_MAX_T];
  __shared__ float s_score[DEC_MAX_T];
  __shared__ unsigned s_ticket;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int g = lane >> 2, c = lane & 3;
  const int T = p.T, H = p.H;
  SpanTrace span(p.trace, 2);
  const int e = blockIdx.x, rb = blockIdx.y;

  // Entry list (written by the router two launches back) and weights do not
  // depend on the gate/up kernel: read them before the PDL wait.
  if (tid == 0) s_n = *wsp<const int32_t>(p, p.L.n_entries);
  if (tid < 2 + 2 * DEC_MAX_T) {
    const int32_t *ent = reinterpret_cast<const int32_t *>(wsp<const DecEntry>(p, p.L.entries) + e);
    // words: 0 slot, 1 flags, 4..11 rank, 12..19 score
    const int wi = tid < 2 ? tid : (tid < 2 + DEC_MAX_T ? 4 + (tid - 2) : 12 + (tid - 2 - DEC_MAX_T));
    if (e < p.L.max_entries) {
      const int v = ent[wi];
      if (tid == 0) s_slot = v;
      else if (tid == 1) s_flags = v;
      else if (tid < 2 + DEC_MAX_T) s_rank[tid - 2] = v;
      else s_score[tid - 2 - DEC_MAX_T] = __int_as_float(v);
    }
  }
  __syncthreads();
  const int n_entries = s_n;
  if (e >= n_entries) {
    span.end();
    return;
  }
  const bool is_shared = s_flags & 1;
  const VbQuantPool &pool = is_shared ? p.shared : p.pool;
  const int slot = is_shared ? 0 : s_slot;
  const int r0 = 128 * rb + 16 * warp + g, r1 = r0 + 8;
  const int NSI = I >> (6 + p.gshift);
  uint2 a0[NGI], a1[NGI];
  {
    const uint8_t *dw = pool_ptr(pool, 6, slot);
#pragma unroll
    for (int G = 0; G < NGI; ++G) {
      a0[G] = ldg_nc_v2(dw + (size_t)r0 * (I / 2) + G * 32 + 8 * c);
      a1[G] = ldg_nc_v2(dw + (size_t)r1 * (I / 2) + G * 32 + 8 * c);
    }
  }
  uint4 sv[4];  // down_s r0, r1, down_b r0, r1
  {
    const uint16_t *ds = reinterpret_cast<const uint16_t *>(pool_ptr(pool, 7, slot));
    const uint16_t *db = reinterpret_cast<const uint16_t *>(pool_ptr(pool, 8, slot));
    sv[0] = ld_scales(ds + (size_t)r0 * NSI, NSI);
    sv[1] = ld_scales(ds + (size_t)r1 * NSI, NSI);
    sv[2] = ld_scales(db + (size_t)r0 * NSI, NSI);
    sv[3] = ld_scales(db + (size_t)r1 * NSI, NSI);
  }
  pdl_wait();
  pdl_launch_dependents();
  {
    // Stage h (fragment order) and its 16-row chunk sums for the T columns.
    const uint4 *hp = reinterpret_cast<const uint4 *>(wsp<const uint32_t>(p, p.L.hperm) +
                                                      (size_t)e * DEC_MAX_T * (I / 2));
    for (int q = tid; q < T * (I / 8); q += K3_THREADS) {
      const int n = q / (I / 8), j = q % (I / 8);
      *reinterpret_cast<uint4 *>(&hsm[n][4 * j]) = __ldcg(hp + q);
    }
    const float *hs = wsp<const float>(p, p.L.hsum) + (size_t)e * DEC_MAX_T * (I / 16);
    for (int q = tid; q < T * (I / 16); q += K3_THREADS) (&hs_sm[0][0])[q] = __ldcg(hs + q);
  }
  __syncthreads();
  float acc[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
  for (int G = 0; G < NGI; ++G) {
    uint4 hb0 = make_uint4(0, 0, 0, 0), hb1 = make_uint4(0, 0, 0, 0);
    if (g < T) {
      const uint4 *hp = reinterpret_cast<const uint4 *>(&hsm[g][(G * 4 + c) * 8]);
      hb0 = hp[0];
      hb1 = hp[1];
    }
    const uint32_t hw[8] = {hb0.x, hb0.y, hb0.z, hb0.w, hb1.x, hb1.y, hb1.z, hb1.w};
    float dd[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
    for (int m = 0; m < 4; ++m) {
      const int i0 = 2 * (m & 1);
      const uint32_t wa = (m >> 1) ? a0[G].y : a0[G].x;
      const uint32_t wb = (m >> 1) ? a1[G].y : a1[G].x;
      mma_bf16(dd, nib_pair(wa, i0), nib_pair(wb, i0), nib_pair(wa, i0 + 1),
               nib_pair(wb, i0 + 1), hw[2 * m], hw[2 * m + 1]);
    }
    const int si = G >> p.gshift;
    const float s0 = bf_at(sv[0], si), s1 = bf_at(sv[1], si);
    const float b0 = bf_at(sv[2], si), b1 = bf_at(sv[3], si);
    float h0 = 0.f, h1 = 0.f;
    if (2 * c < T) {
      const float4 v = *reinterpret_cast<const float4 *>(&hs_sm[2 * c][4 * G]);
      h0 = ((v.x + v.y) + v.z) + v.w;
    }
    if (2 * c + 1 < T) {
      const float4 v = *reinterpret_cast<const float4 *>(&hs_sm[2 * c + 1][4 * G]);
      h1 = ((v.x + v.y) + v.z) + v.w;
    }
    const float bp0 = fmaf(-128.f, s0, b0), bp1 = fmaf(-128.f, s1, b1);
    acc[0] += fmaf(s0, dd[0], bp0 * h0);
    acc[1] += fmaf(s0, dd[1], bp0 * h1);
    acc[2] += fmaf(s1, dd[2], bp1 * h0);
    acc[3] += fmaf(s1, dd[3], bp1 * h1);
  }
  uint16_t *wparts = wsp<uint16_t>(p, p.L.wparts);
  uint16_t *sparts = wsp<uint16_t>(p, p.L.sparts);
#pragma unroll
  for (int q = 0; q < 4; ++q) {
    const int n = 2 * c + (q & 1);
    if (n >= T) continue;
    const int row = (q >> 1) ? r1 : r0;
    const float yb = rbf(acc[q]);
    if (is_shared) {
      sparts[(size_t)n * H + row] = f2bf(yb);
    } else if (s_rank[n] >= 0) {
      wparts[((size_t)n * p.k + s_rank[n]) * H + row] = f2bf(__fmul_rn(yb, s_score[n]));
    }
  }

  // ---- fused combine: the last entry CTA of this row block adds the routes.
  __threadfence();
  __syncthreads();
  unsigned *cnt = wsp<unsigned>(p, p.L.rb_count) + rb;
  if (tid == 0) s_ticket = atomicAdd(cnt, 1u);
  __syncthreads();
  if (s_ticket == (unsigned)n_entries - 1) {
    __threadfence();
    const int k = p.k;
    const uint32_t *wp = wsp<const uint32_t>(p, p.L.wparts);
    const int32_t *ok = wsp<const int32_t>(p, p.L.route_ok);
    for (int q = tid; q < T * 64; q += K3_THREADS) {  // (token, column pair)
      const int t = q >> 6, c2 = 64 * rb + (q & 63);
      uint32_t wv[DEC_MAX_K];
      int okv[DEC_MAX_K];
#pragma unroll
      for (int j = 0; j < DEC_MAX_K; ++j) {
        if (j < k) {
          okv[j] = __ldcg(ok + t * k + j);
          wv[j] = __ldcg(wp + ((size_t)t * k + j) * (H / 2) + c2);
        }
      }
      double s0 = 0.0, s1 = 0.0;
#pragma unroll
      for (int j = 0; j < DEC_MAX_K; ++j) {
        if (j < k && okv[j]) {
          s0 += (double)bf2f(wv[j] & 0xFFFF);
          s1 += (double)bf2f(wv[j] >> 16);
        }
      }
      float y0 = rbf((float)s0), y1 = rbf((float)s1);
      if (p.has_shared) {
        const float gate = __ldcg(wsp<const float>(p, p.L.sgate) + t);
        const uint32_t sw = __ldcg(wsp<const uint32_t>(p, p.L.sparts) + (size_t)t * (H / 2) + c2);
        y0 = rbf(__fadd_rn(y0, rbf(__fmul_rn(gate, bf2f(sw & 0xFFFF)))));
        y1 = rbf(__fadd_rn(y1, rbf(__fmul_rn(gate, bf2f(sw >> 16)))));
      }
      const size_t oi = (size_t)t * (H / 2) + c2;
      if (p.residual) {
        const uint32_t rr = reinterpret_cast<const uint32_t *>(p.residual)[oi];
        y0 = rbf(__fadd_rn(bf2f(rr & 0xFFFF), y0));
        y1 = rbf(__fadd_rn(bf2f(rr >> 16), y1));
      }
      reinterpret_cast<uint32_t *>(p.out)[oi] = pack_bf2(y0, y1);
    }
    if (tid == 0) *cnt = 0u;  // ready for the next launch
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
  switch (I) {
    case 128: k3 = moe_down_kernel<128>; break;
    case 256: k3 = moe_down_kernel<256>; break;
    default: k3 = moe_down_kernel<512>; break;
  }

  cudaStream_t s = as_stream(stream);
  cudaEvent_t *ev = a->timing_events ? (cudaEvent_t *)a->timing_events : nullptr;
  const bool pdl = ev == nullptr;  // event records would break the PDL chain
  // K1 is a PDL secondary of whatever ran before it on the stream (the
  // previous block's down kernel): it only reads weights before the wait.
  if (ev) cudaEventRecord(ev[0], s);
  const size_t smem1 = (size_t)T * H * 2;
  cudaError_t err = decode_kernel_attrs((const void *)k1, smem1);
  if (err == cudaSuccess) err = decode_kernel_attrs((const void *)k2, k2_smem);
  if (err == cudaSuccess) err = decode_kernel_attrs((const void *)k3, 0);
  if (err != cudaSuccess) return set_error(VB_ERR_CUDA, "decode kernel attributes: %s", cudaGetErrorString(err));
  const int grid1 = (E + DEC_ROUTER_WARPS - 1) / DEC_ROUTER_WARPS;
  err = vb_launch(k1, dim3(grid1), dim3(DEC_ROUTER_WARPS * 32), smem1, s, pdl, p);
  if (err != cudaSuccess) return set_error(VB_ERR_CUDA, "moe_router_kernel: %s", cudaGetErrorString(err));
  if (ev) cudaEventRecord(ev[1], s);

  {
    const int grid2 = std::min(sm_count(), L.max_entries * (I / 16));
    err = vb_launch(k2, dim3(grid2), dim3(k2_threads), k2_smem, s, pdl, p);
  }
  if (err != cudaSuccess) return set_error(VB_ERR_CUDA, "moe_gateup_kernel: %s", cudaGetErrorString(err));
  if (ev) cudaEventRecord(ev[2], s);

  err = vb_launch(k3, dim3(L.max_entries, H / 128), dim3(K3_THREADS), 0, s, pdl, p);
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
  const size_t clear = L.rb_count + sizeof(unsigned) * (size_t)(a->hidden / 128);
  const cudaError_t e = cudaMemsetAsync(scratch, 0, clear, as_stream(stream));
  if (e != cudaSuccess)
    return set_error(VB_ERR_CUDA, "vb_moe_decode_noalloc: clearing scratch: %s", cudaGetErrorString(e));
  VbMoeDecodeArgs b = *a;
  b.workspace = scratch;
  b.workspace_bytes = VB_MOE_DECODE_NOALLOC_SCRATCH_BYTES;
  return vb_moe_decode(&b, stream);
}

}  // extern "C"
