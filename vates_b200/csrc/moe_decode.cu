// Decode / MTP-verify fused MoE block (T <= 8 tokens), MLX bf16 dtype chain.
//
// Reference: FileStreamingMoeBlock.__call__ (mlx_streaming/core/moe/block.py
// :245-1013) with PersistentSubGLU.forward (compute.py:145-199) and the
// shared expert (block.py:102-109, 1009-1012).
//
// Three kernels per block:
//  K1 router: logits = bf16(x.Wr^T [+bias]) with one warp per expert row.
//     The last CTA to finish (atomic ticket) runs the precise softmax, top-k
//     with lower-id tie break, renormalisation, slot gather, and builds the
//     list of unique expert "entries" (+ the shared expert). CTA 0 also
//     writes x in MMA-fragment order (xperm) and per-64 column sums (xsum).
//  K2 gate/up: one CTA per (entry, 16 intermediate rows). Weights are the A
//     operand of mma.m16n8k16 (16 rows x 16 columns), tokens are the 8 B
//     columns. 4-bit codes become exact bf16 values 128+q with one LOP3 per
//     pair, so the tensor core sums (128+q)*x per 64-column group; the
//     epilogue applies y += s*D + (b - 128*s)*sum(x) per group. 8 warps
//     split the hidden dimension; partial sums are added in warp order.
//     SwiGLU (bf16 per op) follows, h is written in fragment order (hperm).
//  K3 down + combine: one CTA per 16 output rows loops over all entries,
//     rounds y to bf16, multiplies by the route score (bf16), and adds the
//     routes of each token in rank order (exact double sum of bf16 values,
//     rounded to float32 then bf16), then the sigmoid-gated shared expert.
#include "common.cuh"

namespace vb {

constexpr int DEC_MAX_T = 8;
constexpr int DEC_MAX_K = 16;
constexpr int DEC_MAX_E = 1024;
constexpr int DEC_ROUTER_WARPS = 4;

struct DecEntry {
  int32_t slot;
  int32_t flags;  // bit0 = shared expert
  int32_t pad[2];
  int32_t rank[DEC_MAX_T];   // route rank of token n, -1 = not routed here
  float score[DEC_MAX_T];    // bf16 route score
};

struct DecodeLayout {
  size_t counter, n_entries, sgate, logits, entries, xperm, xsum, hperm, hsum,
      total;
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
  off = align_up(off, 256);
  L.logits = off; off += sizeof(float) * (size_t)T * E;
  off = align_up(off, 256);
  L.entries = off; off += sizeof(DecEntry) * (size_t)L.max_entries;
  off = align_up(off, 256);
  L.xperm = off; off += sizeof(uint32_t) * (size_t)T * (H / 2);
  off = align_up(off, 256);
  L.xsum = off; off += sizeof(float) * (size_t)T * (H / 64);
  off = align_up(off, 256);
  L.hperm = off; off += sizeof(uint32_t) * (size_t)L.max_entries * DEC_MAX_T * (I / 2);
  off = align_up(off, 256);
  L.hsum = off; off += sizeof(float) * (size_t)L.max_entries * DEC_MAX_T * (I / 16);
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
  DecodeLayout L;
};

template <typename T>
__device__ __forceinline__ T *wsp(const DecodeParams &p, size_t off) {
  return reinterpret_cast<T *>(p.ws + off);
}

// Position of value `o` (0..63) of a 64-group inside the fragment-ordered
// layout: returns (quarter c, word w, high half?).
__device__ __forceinline__ void frag_pos(int o, int &c, int &w, int &hi) {
  c = o >> 4;
  int o16 = o & 15;
  int j = o16 >> 3;
  int rem = o16 & 7;
  int i0 = (rem & 2);         // {0,1,4,5} -> 0, {2,3,6,7} -> 2
  int d = rem - i0;           // 0,1,4,5
  int m = 2 * j + (i0 >> 1);
  w = 2 * m + (d & 1);
  hi = d >> 2;
}

// ----------------------------------------------------------------------------
// K1: router GEMV (+ xperm/xsum/shared gate in CTA 0) + last-CTA top-k
// ----------------------------------------------------------------------------
__global__ void __launch_bounds__(DEC_ROUTER_WARPS * 32)
moe_router_kernel(DecodeParams p) {
  extern __shared__ __align__(16) uint8_t smem_raw[];
  uint16_t *xs = reinterpret_cast<uint16_t *>(smem_raw);  // [T][H] bf16
  const int T = p.T, H = p.H, E = p.E;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;

  // Stage x in shared memory (16-byte vectors).
  {
    const uint4 *src = reinterpret_cast<const uint4 *>(p.x);
    uint4 *dst = reinterpret_cast<uint4 *>(xs);
    int nvec = T * H / 8;
    for (int i = tid; i < nvec; i += blockDim.x) dst[i] = src[i];
  }
  __syncthreads();
  if (p.norm_eps > 0.f) {
    // Unit-weight RMSNorm of the block input (decoder post-attention norm):
    // y = bf16(x * (1/sqrt(mean(x^2) + eps))), float32 math with an exact
    // (double) sum of squares. Every CTA computes it identically.
    __shared__ float s_inv[DEC_MAX_T];
    for (int t = warp; t < T; t += DEC_ROUTER_WARPS) {
      double ss = 0.0;
      for (int q = lane; q < H; q += 32) {
        const float v = bf2f(xs[(size_t)t * H + q]);
        ss += (double)v * (double)v;
      }
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
      if (lane == 0) {
        const float ms = __fdiv_rn((float)ss, (float)H);
        s_inv[t] = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(ms, p.norm_eps)));
      }
    }
    __syncthreads();
    for (int i = tid; i < T * H; i += blockDim.x) {
      const int t = i / H;
      xs[i] = f2bf(__fmul_rn(bf2f(xs[i]), s_inv[t]));
    }
    __syncthreads();
  }

  // Router rows: one warp per expert.
  const int e = blockIdx.x * DEC_ROUTER_WARPS + warp;
  if (e < E) {
    float acc[DEC_MAX_T];
#pragma unroll
    for (int t = 0; t < DEC_MAX_T; ++t) acc[t] = 0.f;
    const uint4 *wrow = reinterpret_cast<const uint4 *>(p.router_w + (size_t)e * H);
    const int nv = H / 8;  // uint4 per row
    for (int v0 = 0; v0 < nv; v0 += 32 * 8) {
      uint4 wv[8];
#pragma unroll
      for (int u = 0; u < 8; ++u) {
        int v = v0 + u * 32 + lane;
        wv[u] = v < nv ? ldg_nc_v4(wrow + v) : make_uint4(0, 0, 0, 0);
      }
#pragma unroll
      for (int u = 0; u < 8; ++u) {
        int v = v0 + u * 32 + lane;
        if (v >= nv) break;
        const uint32_t wr[4] = {wv[u].x, wv[u].y, wv[u].z, wv[u].w};
        for (int t = 0; t < T; ++t) {
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
    for (int t = 0; t < T; ++t) {
      float a = acc[t];
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) a += __shfl_xor_sync(0xffffffffu, a, o);
      if (lane == 0) {
        if (p.router_bias) a = a + p.router_bias[e];
        wsp<float>(p, p.L.logits)[(size_t)t * E + e] = rbf(a);
      }
    }
  }

  if (blockIdx.x == 0) {
    // x in MMA fragment order + per-64-column sums (float32).
    uint32_t *xperm = wsp<uint32_t>(p, p.L.xperm);
    float *xsum = wsp<float>(p, p.L.xsum);
    const int NG = H / 64;
    for (int i = tid; i < T * H / 2; i += blockDim.x) {
      int n = i / (H / 2);
      int r = i - n * (H / 2);
      int G = r / 32, cw = r % 32, c = cw >> 3, w = cw & 7;
      int m = w >> 1, pp = w & 1, j = m >> 1, i0 = 2 * (m & 1);
      int base = 64 * G + 16 * c + 8 * j + i0 + pp;
      uint32_t lo = xs[(size_t)n * H + base], hi = xs[(size_t)n * H + base + 4];
      xperm[i] = lo | (hi << 16);
    }
    for (int i = tid; i < T * NG; i += blockDim.x) {
      int n = i / NG, G = i % NG;
      float s = 0.f;
      for (int q = 0; q < 64; ++q) s += bf2f(xs[(size_t)n * H + 64 * G + q]);
      xsum[i] = s;
    }
    if (p.has_shared) {
      for (int t = warp; t < T; t += DEC_ROUTER_WARPS) {
        float a = 0.f;
        for (int q = lane; q < H; q += 32)
          a = fmaf(bf2f(p.shared_gate_w[q]), bf2f(xs[(size_t)t * H + q]), a);
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) a += __shfl_xor_sync(0xffffffffu, a, o);
        if (lane == 0) wsp<float>(p, p.L.sgate)[t] = rbf(mlx_sigmoid(rbf(a)));
      }
    }
  }

  // Last-CTA ticket.
  __shared__ unsigned s_ticket;
  __threadfence();
  __syncthreads();
  if (tid == 0) s_ticket = atomicAdd(wsp<unsigned>(p, p.L.counter), 1u);
  __syncthreads();
  if (s_ticket != gridDim.x - 1) return;
  __threadfence();

  // ---- softmax + top-k per token (one warp per token) ----
  __shared__ int s_exp[DEC_MAX_T * DEC_MAX_K];
  __shared__ int s_slot[DEC_MAX_T * DEC_MAX_K];
  __shared__ float s_score[DEC_MAX_T * DEC_MAX_K];
  const int k = p.k;
  const float *logits = wsp<float>(p, p.L.logits);
  constexpr int PER = DEC_MAX_E / 32;
  for (int t = warp; t < T; t += DEC_ROUTER_WARPS) {
    float v[PER];
    float m = -INFINITY;
#pragma unroll
    for (int i = 0; i < PER; ++i) {
      int idx = lane + 32 * i;
      v[i] = idx < E ? __ldcg(logits + (size_t)t * E + idx) : -INFINITY;
      m = fmaxf(m, v[i]);
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
    double s = 0.0;
#pragma unroll
    for (int i = 0; i < PER; ++i) {
      int idx = lane + 32 * i;
      float ex = idx < E ? expf(__fsub_rn(v[i], m)) : 0.f;
      v[i] = ex;
      s += (double)ex;
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
    const float inv = __frcp_rn((float)s);
#pragma unroll
    for (int i = 0; i < PER; ++i) {
      int idx = lane + 32 * i;
      v[i] = idx < E ? rbf(__fmul_rn(v[i], inv)) : -INFINITY;
    }
    double ssum = 0.0;
    float sel_p = 0.f;
    for (int r = 0; r < k; ++r) {
      float bv = -INFINITY;
      int bi = 0x7fffffff;
#pragma unroll
      for (int i = 0; i < PER; ++i) {
        if (v[i] > bv) { bv = v[i]; bi = lane + 32 * i; }
      }
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) {
        float ov = __shfl_xor_sync(0xffffffffu, bv, o);
        int oi = __shfl_xor_sync(0xffffffffu, bi, o);
        if (ov > bv || (ov == bv && oi < bi)) { bv = ov; bi = oi; }
      }
      if ((bi & 31) == lane) {
#pragma unroll
        for (int i = 0; i < PER; ++i)
          if (lane + 32 * i == bi) v[i] = -INFINITY;
      }
      if (lane == r) sel_p = bv;
      ssum += (double)bv;
      if (lane == 0) s_exp[t * k + r] = bi;
    }
    __syncwarp();
    float score = sel_p;
    if (p.norm_topk) {
      float denom = rbf((float)ssum);
      score = rbf(__fdiv_rn(sel_p, denom));
    }
    if (lane < k) {
      int ex = s_exp[t * k + lane];
      int slot = -1;
      if (ex >= 0 && ex < E) slot = p.table[ex];
      else flag_status(p.status, VB_STATUS_BOUNDS);
      if (slot < 0 || slot >= p.pool.cap) {
        if (slot >= p.pool.cap) flag_status(p.status, VB_STATUS_BOUNDS);
        else flag_status(p.status, VB_STATUS_MISS);
        slot = -1;
      }
      s_slot[t * k + lane] = slot;
      s_score[t * k + lane] = score;
      if (p.out_inds) p.out_inds[t * k + lane] = ex;
      if (p.out_scores) p.out_scores[t * k + lane] = f2bf(score);
      if (p.out_local) p.out_local[t * k + lane] = slot;
    }
  }
  __syncthreads();

  // ---- unique entries in route order (t, j) ----
  if (warp == 0) {
    const int R = T * k;
    DecEntry *entries = wsp<DecEntry>(p, p.L.entries);
    int n_unique = 0;
    for (int base = 0; base < R; base += 32) {
      int r = base + lane;
      int slot = r < R ? s_slot[r] : -1;
      bool first = slot >= 0;
      if (first) {
        for (int q = 0; q < r; ++q)
          if (s_slot[q] == slot) { first = false; break; }
      }
      unsigned mask = __ballot_sync(0xffffffffu, first);
      if (first) {
        int idx = n_unique + __popc(mask & ((1u << lane) - 1u));
        DecEntry en;
        en.slot = slot;
        en.flags = 0;
        en.pad[0] = en.pad[1] = 0;
#pragma unroll
        for (int n = 0; n < DEC_MAX_T; ++n) { en.rank[n] = -1; en.score[n] = 0.f; }
        for (int q = r; q < R; ++q) {
          if (s_slot[q] == slot) {
            int tt = q / k, jj = q % k;
            en.rank[tt] = jj;
            en.score[tt] = s_score[q];
          }
        }
        entries[idx] = en;
      }
      n_unique += __popc(mask);
    }
    if (lane == 0) {
      int n = n_unique;
      if (p.has_shared) {
        DecEntry en;
        en.slot = 0;
        en.flags = 1;
        en.pad[0] = en.pad[1] = 0;
        for (int q = 0; q < DEC_MAX_T; ++q) { en.rank[q] = q < T ? 0 : -1; en.score[q] = 1.f; }
        entries[n++] = en;
      }
      *wsp<int32_t>(p, p.L.n_entries) = n;
      *wsp<unsigned>(p, p.L.counter) = 0u;  // ready for the next launch
    }
  }
}

// ----------------------------------------------------------------------------
// K2: gate/up + SwiGLU for one (entry, 16-row block)
// ----------------------------------------------------------------------------
template <int GPW>
__global__ void __launch_bounds__(256, 2) moe_gateup_kernel(DecodeParams p) {
  const int e = blockIdx.x;
  const int n_entries = *wsp<const int32_t>(p, p.L.n_entries);
  if (e >= n_entries) return;
  const DecEntry ent = wsp<const DecEntry>(p, p.L.entries)[e];
  const int rb = blockIdx.y;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int g = lane >> 2, c = lane & 3;
  const int H = p.H, T = p.T;
  const int NG = H / 64;
  const bool is_shared = ent.flags & 1;
  const VbQuantPool &pool = is_shared ? p.shared : p.pool;
  const int slot = is_shared ? 0 : ent.slot;

  __shared__ float red[8][2][16][8];
  __shared__ float fin[2][16][8];
  __shared__ float hval[16][8];

  float accg[4] = {0.f, 0.f, 0.f, 0.f}, accu[4] = {0.f, 0.f, 0.f, 0.f};
  const int G0 = warp * GPW;
  if (G0 < NG && slot >= 0) {
    const int row0 = 16 * rb + g, row1 = row0 + 8;
    const size_t wrow = (size_t)H / 2;  // bytes per packed row (4-bit)
    const uint8_t *gw = (const uint8_t *)pool.ptr[0] + (size_t)slot * pool.slot_stride[0];
    const uint8_t *uw = (const uint8_t *)pool.ptr[3] + (size_t)slot * pool.slot_stride[3];
    uint2 ag0[GPW], ag1[GPW], au0[GPW], au1[GPW];
#pragma unroll
    for (int i = 0; i < GPW; ++i) {
      const size_t col = (size_t)(G0 + i) * 32 + 8 * c;
      if (G0 + i < NG) {
        ag0[i] = ldg_nc_v2(gw + row0 * wrow + col);
        ag1[i] = ldg_nc_v2(gw + row1 * wrow + col);
        au0[i] = ldg_nc_v2(uw + row0 * wrow + col);
        au1[i] = ldg_nc_v2(uw + row1 * wrow + col);
      }
    }
    // Scales / biases (bf16) for rows row0/row1, groups G0..G0+GPW-1.
    const int NS = H >> (6 + p.gshift);  // scales per row
    const uint16_t *gs = (const uint16_t *)((const uint8_t *)pool.ptr[1] + (size_t)slot * pool.slot_stride[1]);
    const uint16_t *gb = (const uint16_t *)((const uint8_t *)pool.ptr[2] + (size_t)slot * pool.slot_stride[2]);
    const uint16_t *us = (const uint16_t *)((const uint8_t *)pool.ptr[4] + (size_t)slot * pool.slot_stride[4]);
    const uint16_t *ub = (const uint16_t *)((const uint8_t *)pool.ptr[5] + (size_t)slot * pool.slot_stride[5]);
    float sg0[GPW], sg1[GPW], bg0[GPW], bg1[GPW], su0[GPW], su1[GPW], bu0[GPW], bu1[GPW];
#pragma unroll
    for (int i = 0; i < GPW; ++i) {
      int si = (G0 + i) >> p.gshift;
      if (G0 + i < NG) {
        sg0[i] = bf2f(__ldg(gs + (size_t)row0 * NS + si));
        sg1[i] = bf2f(__ldg(gs + (size_t)row1 * NS + si));
        bg0[i] = bf2f(__ldg(gb + (size_t)row0 * NS + si));
        bg1[i] = bf2f(__ldg(gb + (size_t)row1 * NS + si));
        su0[i] = bf2f(__ldg(us + (size_t)row0 * NS + si));
        su1[i] = bf2f(__ldg(us + (size_t)row1 * NS + si));
        bu0[i] = bf2f(__ldg(ub + (size_t)row0 * NS + si));
        bu1[i] = bf2f(__ldg(ub + (size_t)row1 * NS + si));
      }
    }
    // B operand: x column n = g in fragment order; inactive columns are 0.
    const bool col_active = g < T && (is_shared || ent.rank[g] >= 0);
    const uint32_t *xperm = wsp<const uint32_t>(p, p.L.xperm);
    const float *xsum = wsp<const float>(p, p.L.xsum);
    uint4 xb[GPW][2];
    float xs0[GPW], xs1[GPW];
#pragma unroll
    for (int i = 0; i < GPW; ++i) {
      if (col_active && G0 + i < NG) {
        const uint4 *src = reinterpret_cast<const uint4 *>(
            xperm + (((size_t)g * NG + G0 + i) * 4 + c) * 8);
        xb[i][0] = src[0];
        xb[i][1] = src[1];
      } else {
        xb[i][0] = xb[i][1] = make_uint4(0, 0, 0, 0);
      }
      const int n0 = 2 * c, n1 = 2 * c + 1;
      const bool a0 = n0 < T && (is_shared || ent.rank[n0] >= 0);
      const bool a1 = n1 < T && (is_shared || ent.rank[n1] >= 0);
      xs0[i] = (a0 && G0 + i < NG) ? xsum[n0 * NG + G0 + i] : 0.f;
      xs1[i] = (a1 && G0 + i < NG) ? xsum[n1 * NG + G0 + i] : 0.f;
    }
#pragma unroll
    for (int i = 0; i < GPW; ++i) {
      if (G0 + i >= NG) break;
      float dg[4] = {0.f, 0.f, 0.f, 0.f}, du[4] = {0.f, 0.f, 0.f, 0.f};
      const uint32_t xw[8] = {xb[i][0].x, xb[i][0].y, xb[i][0].z, xb[i][0].w,
                              xb[i][1].x, xb[i][1].y, xb[i][1].z, xb[i][1].w};
#pragma unroll
      for (int m = 0; m < 4; ++m) {
        const int i0 = 2 * (m & 1);
        const uint32_t wa = (m >> 1) ? ag0[i].y : ag0[i].x;
        const uint32_t wb = (m >> 1) ? ag1[i].y : ag1[i].x;
        mma_bf16(dg, nib_pair(wa, i0), nib_pair(wb, i0), nib_pair(wa, i0 + 1),
                 nib_pair(wb, i0 + 1), xw[2 * m], xw[2 * m + 1]);
        const uint32_t va = (m >> 1) ? au0[i].y : au0[i].x;
        const uint32_t vb2 = (m >> 1) ? au1[i].y : au1[i].x;
        mma_bf16(du, nib_pair(va, i0), nib_pair(vb2, i0), nib_pair(va, i0 + 1),
                 nib_pair(vb2, i0 + 1), xw[2 * m], xw[2 * m + 1]);
      }
      const float bpg0 = fmaf(-128.f, sg0[i], bg0[i]), bpg1 = fmaf(-128.f, sg1[i], bg1[i]);
      const float bpu0 = fmaf(-128.f, su0[i], bu0[i]), bpu1 = fmaf(-128.f, su1[i], bu1[i]);
      accg[0] += fmaf(sg0[i], dg[0], bpg0 * xs0[i]);
      accg[1] += fmaf(sg0[i], dg[1], bpg0 * xs1[i]);
      accg[2] += fmaf(sg1[i], dg[2], bpg1 * xs0[i]);
      accg[3] += fmaf(sg1[i], dg[3], bpg1 * xs1[i]);
      accu[0] += fmaf(su0[i], du[0], bpu0 * xs0[i]);
      accu[1] += fmaf(su0[i], du[1], bpu0 * xs1[i]);
      accu[2] += fmaf(su1[i], du[2], bpu1 * xs0[i]);
      accu[3] += fmaf(su1[i], du[3], bpu1 * xs1[i]);
    }
  }
  red[warp][0][g][2 * c] = accg[0];
  red[warp][0][g][2 * c + 1] = accg[1];
  red[warp][0][g + 8][2 * c] = accg[2];
  red[warp][0][g + 8][2 * c + 1] = accg[3];
  red[warp][1][g][2 * c] = accu[0];
  red[warp][1][g][2 * c + 1] = accu[1];
  red[warp][1][g + 8][2 * c] = accu[2];
  red[warp][1][g + 8][2 * c + 1] = accu[3];
  __syncthreads();
  {
    const int P = tid >> 7, row = (tid >> 3) & 15, col = tid & 7;
    float s = 0.f;
#pragma unroll
    for (int w = 0; w < 8; ++w) s += red[w][P][row][col];
    fin[P][row][col] = s;
  }
  __syncthreads();
  if (tid < 128) {
    const int row = tid >> 3, col = tid & 7;
    const bool active = col < T && (is_shared || ent.rank[col] >= 0) && slot >= 0;
    float h = 0.f;
    if (active) h = swiglu_bf16(rbf(fin[0][row][col]), rbf(fin[1][row][col]));
    hval[row][col] = h;
  }
  __syncthreads();
  if (tid < 64) {
    // 16 rows of h are quarter c' = rb%4 of intermediate group G' = rb/4.
    const int n = tid >> 3, w = tid & 7;
    const int m = w >> 1, pp = w & 1, j = m >> 1, i0 = 2 * (m & 1);
    const int olo = 8 * j + i0 + pp, ohi = olo + 4;
    const uint32_t word = pack_bf2(hval[olo][n], hval[ohi][n]);
    const int NGI = p.I / 64;
    uint32_t *hperm = wsp<uint32_t>(p, p.L.hperm);
    const size_t idx = ((((size_t)e * DEC_MAX_T + n) * NGI + (rb >> 2)) * 4 + (rb & 3)) * 8 + w;
    hperm[idx] = word;
  } else if (tid < 72) {
    const int n = tid - 64;
    float s = 0.f;
#pragma unroll
    for (int o = 0; o < 16; ++o) s += hval[o][n];
    wsp<float>(p, p.L.hsum)[((size_t)e * DEC_MAX_T + n) * (p.I / 16) + rb] = s;
  }
}

// ----------------------------------------------------------------------------
// K3: down projection + weighted combine + shared expert, 16 output rows/CTA
// ----------------------------------------------------------------------------
template <int NGI>
__global__ void __launch_bounds__(256, 1) moe_down_kernel(DecodeParams p) {
  const int rb = blockIdx.x;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int g = lane >> 2, c = lane & 3;
  const int T = p.T, k = p.k, I = p.I;
  __shared__ float contrib[DEC_MAX_T][DEC_MAX_K][16];
  __shared__ float shy[DEC_MAX_T][16];
  for (int i = tid; i < DEC_MAX_T * DEC_MAX_K * 16; i += blockDim.x)
    (&contrib[0][0][0])[i] = 0.f;
  for (int i = tid; i < DEC_MAX_T * 16; i += blockDim.x) (&shy[0][0])[i] = 0.f;
  __syncthreads();

  const int n_entries = *wsp<const int32_t>(p, p.L.n_entries);
  const DecEntry *entries = wsp<const DecEntry>(p, p.L.entries);
  const uint32_t *hperm = wsp<const uint32_t>(p, p.L.hperm);
  const float *hsum = wsp<const float>(p, p.L.hsum);
  const int row0 = 16 * rb + g, row1 = row0 + 8;
  const size_t wrow = (size_t)I / 2;
  const int NS = I >> (6 + p.gshift);

  for (int e = warp; e < n_entries; e += 8) {
    const DecEntry ent = entries[e];
    const bool is_shared = ent.flags & 1;
    const VbQuantPool &pool = is_shared ? p.shared : p.pool;
    const int slot = is_shared ? 0 : ent.slot;
    if (slot < 0) continue;
    // Prefetch the next entry's rows into L2 while this one computes.
    if (e + 8 < n_entries) {
      const DecEntry nx = entries[e + 8];
      const bool ns = nx.flags & 1;
      const VbQuantPool &np = ns ? p.shared : p.pool;
      const int nslot = ns ? 0 : nx.slot;
      if (nslot >= 0 && lane < 16) {
        const uint8_t *nd = (const uint8_t *)np.ptr[6] + (size_t)nslot * np.slot_stride[6];
        const uint8_t *rowp = nd + (size_t)(16 * rb + lane) * wrow;
        for (size_t off = 0; off < wrow; off += 128) prefetch_l2(rowp + off);
      }
    }
    const uint8_t *dw = (const uint8_t *)pool.ptr[6] + (size_t)slot * pool.slot_stride[6];
    const uint16_t *ds = (const uint16_t *)((const uint8_t *)pool.ptr[7] + (size_t)slot * pool.slot_stride[7]);
    const uint16_t *db = (const uint16_t *)((const uint8_t *)pool.ptr[8] + (size_t)slot * pool.slot_stride[8]);
    uint2 a0[NGI], a1[NGI];
#pragma unroll
    for (int G = 0; G < NGI; ++G) {
      a0[G] = ldg_nc_v2(dw + row0 * wrow + G * 32 + 8 * c);
      a1[G] = ldg_nc_v2(dw + row1 * wrow + G * 32 + 8 * c);
    }
    float s0[NGI], s1[NGI], b0[NGI], b1[NGI];
#pragma unroll
    for (int G = 0; G < NGI; ++G) {
      const int si = G >> p.gshift;
      s0[G] = bf2f(__ldg(ds + (size_t)row0 * NS + si));
      s1[G] = bf2f(__ldg(ds + (size_t)row1 * NS + si));
      b0[G] = bf2f(__ldg(db + (size_t)row0 * NS + si));
      b1[G] = bf2f(__ldg(db + (size_t)row1 * NS + si));
    }
    const bool col_active = g < T && (is_shared || ent.rank[g] >= 0);
    uint4 hb[NGI][2];
#pragma unroll
    for (int G = 0; G < NGI; ++G) {
      if (col_active) {
        const uint4 *src = reinterpret_cast<const uint4 *>(
            hperm + ((((size_t)e * DEC_MAX_T + g) * NGI + G) * 4 + c) * 8);
        hb[G][0] = __ldcg(src);
        hb[G][1] = __ldcg(src + 1);
      } else {
        hb[G][0] = hb[G][1] = make_uint4(0, 0, 0, 0);
      }
    }
    const int n0 = 2 * c, n1 = 2 * c + 1;
    const bool act0 = n0 < T && (is_shared || ent.rank[n0] >= 0);
    const bool act1 = n1 < T && (is_shared || ent.rank[n1] >= 0);
    float acc[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
    for (int G = 0; G < NGI; ++G) {
      float d[4] = {0.f, 0.f, 0.f, 0.f};
      const uint32_t hw[8] = {hb[G][0].x, hb[G][0].y, hb[G][0].z, hb[G][0].w,
                              hb[G][1].x, hb[G][1].y, hb[G][1].z, hb[G][1].w};
#pragma unroll
      for (int m = 0; m < 4; ++m) {
        const int i0 = 2 * (m & 1);
        const uint32_t wa = (m >> 1) ? a0[G].y : a0[G].x;
        const uint32_t wb = (m >> 1) ? a1[G].y : a1[G].x;
        mma_bf16(d, nib_pair(wa, i0), nib_pair(wb, i0), nib_pair(wa, i0 + 1),
                 nib_pair(wb, i0 + 1), hw[2 * m], hw[2 * m + 1]);
      }
      float hs0 = 0.f, hs1 = 0.f;
      if (act0) {
        const float *h = hsum + ((size_t)e * DEC_MAX_T + n0) * (I / 16) + 4 * G;
        hs0 = ((__ldcg(h) + __ldcg(h + 1)) + __ldcg(h + 2)) + __ldcg(h + 3);
      }
      if (act1) {
        const float *h = hsum + ((size_t)e * DEC_MAX_T + n1) * (I / 16) + 4 * G;
        hs1 = ((__ldcg(h) + __ldcg(h + 1)) + __ldcg(h + 2)) + __ldcg(h + 3);
      }
      const float bp0 = fmaf(-128.f, s0[G], b0[G]), bp1 = fmaf(-128.f, s1[G], b1[G]);
      acc[0] += fmaf(s0[G], d[0], bp0 * hs0);
      acc[1] += fmaf(s0[G], d[1], bp0 * hs1);
      acc[2] += fmaf(s1[G], d[2], bp1 * hs0);
      acc[3] += fmaf(s1[G], d[3], bp1 * hs1);
    }
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      const int n = 2 * c + (q & 1);
      const int r = g + 8 * (q >> 1);
      if (n >= T) continue;
      const float yb = rbf(acc[q]);
      if (is_shared) {
        shy[n][r] = yb;
      } else if (ent.rank[n] >= 0) {
        contrib[n][ent.rank[n]][r] = rbf(__fmul_rn(yb, ent.score[n]));
      }
    }
  }
  __syncthreads();
  if (tid < T * 16) {
    const int t = tid >> 4, r = tid & 15;
    double s = 0.0;
    for (int j = 0; j < k; ++j) s += (double)contrib[t][j][r];
    float y = rbf((float)s);
    if (p.has_shared) {
      const float gate = wsp<const float>(p, p.L.sgate)[t];
      y = rbf(__fadd_rn(y, rbf(__fmul_rn(gate, shy[t][r]))));
    }
    const size_t oi = (size_t)t * p.H + 16 * rb + r;
    if (p.residual) y = rbf(__fadd_rn(bf2f(p.residual[oi]), y));
    p.out[oi] = f2bf(y);
  }
}

}  // namespace vb

using namespace vb;

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
  VB_REQUIRE(H % 512 == 0 && H >= 512 && H <= 8192, "vb_moe_decode: hidden=%d", H);
  VB_REQUIRE(I == 128 || I == 256 || I == 512, "vb_moe_decode: inter=%d", I);
  VB_REQUIRE(E >= k && E <= DEC_MAX_E, "vb_moe_decode: num_experts=%d", E);
  VB_REQUIRE(k >= 1 && k <= DEC_MAX_K && k <= 32, "vb_moe_decode: top_k=%d", k);
  VB_REQUIRE(a->x && a->router_w && a->slot_table && a->out, "vb_moe_decode: null tensor");
  VB_REQUIRE(a->pool.ptr[0] && a->pool.cap > 0, "vb_moe_decode: empty pool");
  const bool has_shared = a->shared.ptr[0] != nullptr;
  VB_REQUIRE(!has_shared || a->shared_gate_w, "vb_moe_decode: shared expert without gate");
  DecodeLayout L = decode_layout(T, H, I, E, k);
  VB_REQUIRE(a->workspace && a->workspace_bytes >= L.total,
             "vb_moe_decode: workspace %zu < %zu", a->workspace_bytes, L.total);

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
  p.L = L;
  cudaStream_t s = as_stream(stream);

  // The router's last-CTA ticket counter lives in the first workspace word:
  // callers zero-fill the workspace once; every call leaves it at zero.
  cudaEvent_t *ev = a->timing_events ? (cudaEvent_t *)a->timing_events : nullptr;
  if (ev) cudaEventRecord(ev[0], s);
  const size_t smem1 = (size_t)T * H * 2;
  if (smem1 > 48 * 1024) {
    cudaFuncSetAttribute(moe_router_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                         (int)smem1);
  }
  const int grid1 = (E + DEC_ROUTER_WARPS - 1) / DEC_ROUTER_WARPS;
  moe_router_kernel<<<grid1, DEC_ROUTER_WARPS * 32, smem1, s>>>(p);
  int rc = check_launch("moe_router_kernel");
  if (rc) return rc;
  if (ev) cudaEventRecord(ev[1], s);

  dim3 grid2(L.max_entries, I / 16);
  const int NG = H / 64;
  if (NG <= 8) moe_gateup_kernel<1><<<grid2, 256, 0, s>>>(p);
  else if (NG <= 16) moe_gateup_kernel<2><<<grid2, 256, 0, s>>>(p);
  else if (NG <= 32) moe_gateup_kernel<4><<<grid2, 256, 0, s>>>(p);
  else if (NG <= 64) moe_gateup_kernel<8><<<grid2, 256, 0, s>>>(p);
  else moe_gateup_kernel<16><<<grid2, 256, 0, s>>>(p);
  rc = check_launch("moe_gateup_kernel");
  if (rc) return rc;
  if (ev) cudaEventRecord(ev[2], s);

  const int grid3 = H / 16;
  if (I == 128) moe_down_kernel<2><<<grid3, 256, 0, s>>>(p);
  else if (I == 256) moe_down_kernel<4><<<grid3, 256, 0, s>>>(p);
  else moe_down_kernel<8><<<grid3, 256, 0, s>>>(p);
  rc = check_launch("moe_down_kernel");
  if (rc) return rc;
  if (ev) cudaEventRecord(ev[3], s);
  return VB_OK;
}

}  // extern "C"
