// Dense layers of the decode stack around the MoE block: the 4-bit quantized
// linear projection (with an optional RMSNorm of its input and an optional
// residual add), RMSNorm, row argmax and the quantized embedding lookup.
//
// Reference: every nn.QuantizedLinear / nn.QuantizedEmbedding of the
// Qwen3-Next model the reference runs (mlx-lm 0.31.3 models/qwen3_next.py,
// quantized 4-bit group 64 as in mtp/qwen3_next_mtp.py:170-181), i.e. MLX's
// quantized_matmul(x, w, scales, biases, transpose=True): per 64-column group
// s * sum(x q) + b * sum(x), float32 accumulation, one rounding to bf16; the
// decoder's residual adds (h = x + r in bf16) and mx.fast.rms_norm.
//
// vb_qlinear, T <= 8 tokens (HBM-bound, 0.5 B per weight): a persistent grid
// (two CTAs of 8 warps per SM) walks items of 16 output rows over the whole K.
// A CTA stages x once (RMS-normalised when asked) in MMA fragment order with
// per-group sums; for an item, warp w takes groups [w*GPW, (w+1)*GPW) of the
// 16 rows: each lane loads its 8-byte share of every group of rows g and g+8
// plus a vector of scales and biases, turns the codes into exact bf16 pairs
// 128 + q (LOP3) and runs mma.m16n8k16 against x; the group's scale and bias
// are applied as s * D + (b - 128 s) * sum(x). The eight warps' partial sums
// meet in shared memory and warp 0 adds them in warp order (deterministic).
// The next item's codes are loaded while the current one is computed.
#include "common.cuh"

namespace vb {

constexpr int QL_THREADS = 256;
constexpr int QL_MAX_T = 8;
constexpr int QL_MAX_K = 4096;

struct QlParams {
  const uint16_t *x;            // bf16 [T, K]
  const uint32_t *codes;        // [N, K/8]
  const uint16_t *scales, *biases;  // bf16 [N, K/64]
  const uint16_t *norm_w;       // nullable bf16 [K]: x -> rms_norm(x) * w
  const uint16_t *residual;     // nullable bf16 [T, N]
  uint16_t *y;                  // bf16 [T, N]
  float eps;
  int T, K, N, items;
};

template <int GPW>
struct QlItem {
  uint2 wa[GPW], wb[GPW];
  uint32_t sa[(GPW + 1) / 2], sb[(GPW + 1) / 2], ba[(GPW + 1) / 2], bb[(GPW + 1) / 2];
};

// Codes and scales of item `it` for this lane (rows 16 it + g, + 8; groups
// g0 .. g0 + GPW - 1, those past ng zero).
template <int GPW>
__device__ __forceinline__ void ql_load(const QlParams &p, int it, int g0, int ng, int lane,
                                        QlItem<GPW> &d) {
  const int g = lane >> 2, c = lane & 3;
  const int ra = it * 16 + g, rb = ra + 8;
  const bool va = ra < p.N, vb = rb < p.N;
  const int wpr = p.K >> 3, gpr = p.K >> 6;
#pragma unroll
  for (int j = 0; j < GPW; ++j) {
    const bool ok = j < ng;
    const int off = (g0 + j) * 8 + 2 * c;
    d.wa[j] = (va && ok) ? ldg_nc_v2(p.codes + (size_t)ra * wpr + off) : make_uint2(0, 0);
    d.wb[j] = (vb && ok) ? ldg_nc_v2(p.codes + (size_t)rb * wpr + off) : make_uint2(0, 0);
  }
  const size_t oa = (size_t)ra * gpr + g0, ob = (size_t)rb * gpr + g0;
  // warps past the last group load no scales (their vectors would run past
  // the row); a warp with groups has all GPW of them (G % GPW == 0)
  const bool va_s = va && ng > 0, vb_s = vb && ng > 0;
  if constexpr (GPW >= 8) {
#pragma unroll
    for (int h = 0; h < GPW / 8; ++h) {
      const uint4 z = make_uint4(0, 0, 0, 0);
      const uint4 s0 = va_s ? ldg_nc_v4(p.scales + oa + 8 * h) : z;
      const uint4 b0 = va_s ? ldg_nc_v4(p.biases + oa + 8 * h) : z;
      const uint4 s1 = vb_s ? ldg_nc_v4(p.scales + ob + 8 * h) : z;
      const uint4 b1 = vb_s ? ldg_nc_v4(p.biases + ob + 8 * h) : z;
      d.sa[4 * h] = s0.x; d.sa[4 * h + 1] = s0.y; d.sa[4 * h + 2] = s0.z; d.sa[4 * h + 3] = s0.w;
      d.ba[4 * h] = b0.x; d.ba[4 * h + 1] = b0.y; d.ba[4 * h + 2] = b0.z; d.ba[4 * h + 3] = b0.w;
      d.sb[4 * h] = s1.x; d.sb[4 * h + 1] = s1.y; d.sb[4 * h + 2] = s1.z; d.sb[4 * h + 3] = s1.w;
      d.bb[4 * h] = b1.x; d.bb[4 * h + 1] = b1.y; d.bb[4 * h + 2] = b1.z; d.bb[4 * h + 3] = b1.w;
    }
  } else if constexpr (GPW == 4) {
    const uint2 z = make_uint2(0, 0);
    const uint2 s0 = va_s ? ldg_nc_v2(p.scales + oa) : z, b0 = va_s ? ldg_nc_v2(p.biases + oa) : z;
    const uint2 s1 = vb_s ? ldg_nc_v2(p.scales + ob) : z, b1 = vb_s ? ldg_nc_v2(p.biases + ob) : z;
    d.sa[0] = s0.x; d.sa[1] = s0.y; d.ba[0] = b0.x; d.ba[1] = b0.y;
    d.sb[0] = s1.x; d.sb[1] = s1.y; d.bb[0] = b1.x; d.bb[1] = b1.y;
  } else if constexpr (GPW == 2) {
    d.sa[0] = va_s ? __ldg(reinterpret_cast<const uint32_t *>(p.scales + oa)) : 0u;
    d.ba[0] = va_s ? __ldg(reinterpret_cast<const uint32_t *>(p.biases + oa)) : 0u;
    d.sb[0] = vb_s ? __ldg(reinterpret_cast<const uint32_t *>(p.scales + ob)) : 0u;
    d.bb[0] = vb_s ? __ldg(reinterpret_cast<const uint32_t *>(p.biases + ob)) : 0u;
  } else {
    d.sa[0] = (va_s) ? (uint32_t)__ldg(p.scales + oa) : 0u;
    d.ba[0] = (va_s) ? (uint32_t)__ldg(p.biases + oa) : 0u;
    d.sb[0] = (vb_s) ? (uint32_t)__ldg(p.scales + ob) : 0u;
    d.bb[0] = (vb_s) ? (uint32_t)__ldg(p.biases + ob) : 0u;
  }
}

// bf16 value of group j (low half: even j) of a packed scale/bias word array.
template <int GPW>
__device__ __forceinline__ float ql_half(const uint32_t (&w)[(GPW + 1) / 2], int j) {
  const uint32_t v = w[j >> 1];
  return __uint_as_float((j & 1) ? (v & 0xFFFF0000u) : (v << 16));
}

// This warp's x fragments and group sums (its groups are the same for every
// item): in registers when GPW <= 4, read from shared memory otherwise.
template <int GPW>
struct QlX {
  static constexpr bool REG = GPW <= 4;
  uint2 f[REG ? GPW : 1][4];
  float s[REG ? GPW : 1][2];
};

template <int GPW>
__device__ __forceinline__ void ql_compute(const QlItem<GPW> &d, const uint2 *xfrag,
                                           const float *xsum, const QlX<GPW> &xr, int g0, int ng,
                                           int lane, float (&acc)[4]) {
  const int c = lane & 3;
#pragma unroll
  for (int j = 0; j < GPW; ++j) {
    if (j >= ng) break;
    const int grp = g0 + j;
    float dd[4] = {0.f, 0.f, 0.f, 0.f};
    uint32_t pa[2][4], pb[2][4];
    nib_pairs4(d.wa[j].x, pa[0]);
    nib_pairs4(d.wa[j].y, pa[1]);
    nib_pairs4(d.wb[j].x, pb[0]);
    nib_pairs4(d.wb[j].y, pb[1]);
#pragma unroll
    for (int mm = 0; mm < 4; ++mm) {
      const int jw = mm >> 1, h = mm & 1;
      const uint2 bf = QlX<GPW>::REG ? xr.f[QlX<GPW>::REG ? j : 0][mm]
                                     : xfrag[(grp * 4 + mm) * 32 + lane];
      mma_bf16(dd, pa[jw][2 * h], pb[jw][2 * h], pa[jw][2 * h + 1], pb[jw][2 * h + 1], bf.x,
               bf.y);
    }
    const float s_a = ql_half<GPW>(d.sa, j), s_b = ql_half<GPW>(d.sb, j);
    const float c_a = ql_half<GPW>(d.ba, j) - 128.f * s_a, c_b = ql_half<GPW>(d.bb, j) - 128.f * s_b;
    const float x0 = QlX<GPW>::REG ? xr.s[QlX<GPW>::REG ? j : 0][0] : xsum[grp * QL_MAX_T + 2 * c];
    const float x1 = QlX<GPW>::REG ? xr.s[QlX<GPW>::REG ? j : 0][1]
                                   : xsum[grp * QL_MAX_T + 2 * c + 1];
    acc[0] += fmaf(s_a, dd[0], c_a * x0);
    acc[1] += fmaf(s_a, dd[1], c_a * x1);
    acc[2] += fmaf(s_b, dd[2], c_b * x0);
    acc[3] += fmaf(s_b, dd[3], c_b * x1);
  }
}

// Dynamic shared memory: xfrag [K/16][32] uint2 and xsum [K/64][8] f32.
template <int GPW>
__global__ void __launch_bounds__(QL_THREADS, 2) qlinear_kernel(QlParams p) {
  extern __shared__ __align__(16) uint8_t ql_smem[];
  __shared__ float inv_rms[QL_MAX_T];
  __shared__ float red[2][8][32][4];
  const int K = p.K, T = p.T;
  uint2 *xfrag = reinterpret_cast<uint2 *>(ql_smem);
  float *xsum = reinterpret_cast<float *>(ql_smem + (size_t)K * 16);
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int G = K >> 6;
  const int g0 = warp * GPW, ng = max(0, min(GPW, G - g0));

  // First item's weights (independent of earlier kernels) before anything else.
  QlItem<GPW> cur, nxt;
  int it = blockIdx.x;
  if (it < p.items) ql_load<GPW>(p, it, g0, ng, lane, cur);
  pdl_launch_dependents();
  pdl_wait();

  // x: inverse RMS per row (warp t takes row t), then the rows staged as
  // bf16(bf16(x * inv) * w) (or x), then fragments and group sums.
  if (p.norm_w) {
    for (int t = warp; t < T; t += QL_THREADS / 32) {
      const uint16_t *xr = p.x + (size_t)t * K;
      float ss = 0.f;
#pragma unroll 4
      for (int k = lane * 8; k < K; k += 256) {
        const uint4 v = *reinterpret_cast<const uint4 *>(xr + k);
        const uint32_t w4[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          const float lo = __uint_as_float(w4[i] << 16), hi = __uint_as_float(w4[i] & 0xFFFF0000u);
          ss = fmaf(lo, lo, ss);
          ss = fmaf(hi, hi, ss);
        }
      }
#pragma unroll
      for (int o = 16; o; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
      if (lane == 0) inv_rms[t] = rsqrtf(ss / (float)K + p.eps);
    }
    __syncthreads();
  }
  // Fragments straight from x: work item (row n, group grp, word w) loads
  // the 8 columns kb = 64 grp + 8 w of row n and writes the two fragments
  // that word feeds. Fragment of MMA m = 4 grp + mm (mm = 2 jw + h) for lane
  // (n, c): the lane's code word covers columns 64 grp + 8 (2c + jw) .. +7,
  // its A pairs are nibbles (2h, 2h+4) and (2h+1, 2h+5), so b0 = x[n][kb+2h],
  // x[n][kb+2h+4] and b1 = x[n][kb+2h+1], x[n][kb+2h+5] with w = 2c + jw.
  // The 8 words of (n, grp) are 8 consecutive lanes: their sum by shuffles
  // (fixed order) is the group sum. Only rows n < T are staged (the MMA
  // columns of rows past T are never stored), and each thread issues the
  // loads of four work items before it uses the first, so a CTA waits for
  // x about once instead of once per work item.
  {
    const int total = T * G * 8;  // a multiple of 32: the bounds below are warp-uniform
    for (int i0 = 0; i0 < total; i0 += 4 * QL_THREADS) {
      uint4 raw[4];
#pragma unroll
      for (int b = 0; b < 4; ++b) {
        const int i = i0 + b * QL_THREADS + tid;
        if (i < total) {
          const int w = i & 7, grp = (i >> 3) % G, n = (i >> 3) / G;
          raw[b] = *reinterpret_cast<const uint4 *>(p.x + (size_t)n * K + grp * 64 + w * 8);
        }
      }
#pragma unroll
      for (int b = 0; b < 4; ++b) {
        const int i = i0 + b * QL_THREADS + tid;
        if (i >= total) break;
        const int w = i & 7, grp = (i >> 3) % G, n = (i >> 3) / G;
        const uint32_t xv[4] = {raw[b].x, raw[b].y, raw[b].z, raw[b].w};
        float v[8];
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          v[2 * q] = __uint_as_float(xv[q] << 16);
          v[2 * q + 1] = __uint_as_float(xv[q] & 0xFFFF0000u);
        }
        if (p.norm_w) {
          const uint4 wr = *reinterpret_cast<const uint4 *>(p.norm_w + grp * 64 + w * 8);
          const uint32_t wv[4] = {wr.x, wr.y, wr.z, wr.w};
          const float inv = inv_rms[n];
#pragma unroll
          for (int q = 0; q < 4; ++q) {
            v[2 * q] = rbf(rbf(v[2 * q] * inv) * __uint_as_float(wv[q] << 16));
            v[2 * q + 1] = rbf(rbf(v[2 * q + 1] * inv) * __uint_as_float(wv[q] & 0xFFFF0000u));
          }
        }
        const int cc = w >> 1, jw = w & 1, l = n * 4 + cc;
#pragma unroll
        for (int h = 0; h < 2; ++h)
          xfrag[(grp * 4 + 2 * jw + h) * 32 + l] =
              make_uint2(pack_bf2(v[2 * h], v[2 * h + 4]), pack_bf2(v[2 * h + 1], v[2 * h + 5]));
        float sum = 0.f;
#pragma unroll
        for (int q = 0; q < 8; ++q) sum += v[q];
        sum += __shfl_xor_sync(0xffffffffu, sum, 1);
        sum += __shfl_xor_sync(0xffffffffu, sum, 2);
        sum += __shfl_xor_sync(0xffffffffu, sum, 4);
        if (w == 0) xsum[grp * QL_MAX_T + n] = sum;
      }
    }
  }
  __syncthreads();

  const int c = lane & 3, g = lane >> 2;
  QlX<GPW> xr;
  if constexpr (QlX<GPW>::REG) {
#pragma unroll
    for (int j = 0; j < GPW; ++j) {
      const int grp = j < ng ? g0 + j : 0;
#pragma unroll
      for (int mm = 0; mm < 4; ++mm) xr.f[j][mm] = xfrag[(grp * 4 + mm) * 32 + lane];
      xr.s[j][0] = xsum[grp * QL_MAX_T + 2 * c];
      xr.s[j][1] = xsum[grp * QL_MAX_T + 2 * c + 1];
    }
  }
  int buf = 0;
  for (; it < p.items; it += gridDim.x) {
    const int next = it + gridDim.x;
    if (next < p.items) ql_load<GPW>(p, next, g0, ng, lane, nxt);
    float acc[4] = {0.f, 0.f, 0.f, 0.f};
    ql_compute<GPW>(cur, xfrag, xsum, xr, g0, ng, lane, acc);
    *reinterpret_cast<float4 *>(red[buf][warp][lane]) = make_float4(acc[0], acc[1], acc[2], acc[3]);
    __syncthreads();
    if (warp == 0) {
      float o[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
      for (int w = 0; w < 8; ++w) {
        const float4 v = *reinterpret_cast<const float4 *>(red[buf][w][lane]);
        o[0] += v.x; o[1] += v.y; o[2] += v.z; o[3] += v.w;
      }
      const int rows[2] = {it * 16 + g, it * 16 + g + 8};
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        const int row = rows[q >> 1], n = 2 * c + (q & 1);
        if (row < p.N && n < T) {
          float v = rbf(o[q]);
          if (p.residual) v = bf2f(p.residual[(size_t)n * p.N + row]) + v;
          p.y[(size_t)n * p.N + row] = f2bf(v);
        }
      }
    }
    buf ^= 1;  // the next item writes the other partial buffer: one barrier per item
    cur = nxt;
  }
}

// RMSNorm with an optional residual add: h = bf16(x + r) (written to h_out
// when given), y = bf16(bf16(h * rsqrt(mean(h^2) + eps)) * w), y rows
// y_stride elements apart. One CTA per row.
__global__ void __launch_bounds__(256) rms_norm_kernel(const uint16_t *__restrict__ x,
                                                       const uint16_t *__restrict__ r,
                                                       const uint16_t *__restrict__ w, int D,
                                                       float eps, uint16_t *__restrict__ h_out,
                                                       uint16_t *__restrict__ y, int y_stride) {
  __shared__ float red[8];
  pdl_launch_dependents();
  pdl_wait();
  const size_t row = blockIdx.x;
  const uint16_t *xr = x + row * D;
  float ss = 0.f;
  for (int k = threadIdx.x; k < D; k += 256) {
    float v = bf2f(xr[k]);
    if (r) v = rbf(v + bf2f(r[row * D + k]));
    ss = fmaf(v, v, ss);
  }
#pragma unroll
  for (int o = 16; o; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = ss;
  __syncthreads();
  float tot = 0.f;
#pragma unroll
  for (int i = 0; i < 8; ++i) tot += red[i];
  const float inv = rsqrtf(tot / (float)D + eps);
  for (int k = threadIdx.x; k < D; k += 256) {
    float v = bf2f(xr[k]);
    if (r) v = rbf(v + bf2f(r[row * D + k]));
    if (h_out) h_out[row * D + k] = f2bf(v);
    const float nv = rbf(v * inv);
    y[row * y_stride + k] = f2bf(w ? nv * bf2f(w[k]) : nv);
  }
}

// Row argmax of bf16 values, ties to the smallest index (mx.argmax). Grid
// (rows, parts): every CTA reduces a strided share of its row, the last CTA of
// the row (ticket) reduces the parts in order and resets the ticket.
constexpr int AM_PARTS = 16;
__global__ void __launch_bounds__(256) argmax_kernel(const uint16_t *__restrict__ v, int n,
                                                     float *__restrict__ part_val,
                                                     int32_t *__restrict__ part_idx,
                                                     uint32_t *__restrict__ tickets,
                                                     int32_t *__restrict__ out) {
  __shared__ float sv[8];
  __shared__ int si[8];
  __shared__ int last;
  const int row = blockIdx.x, part = blockIdx.y, tid = threadIdx.x;
  pdl_launch_dependents();
  pdl_wait();
  const uint16_t *r = v + (size_t)row * n;
  float best = -INFINITY;
  int bi = INT_MAX;
  const int per = (n + AM_PARTS - 1) / AM_PARTS;
  const int lo = part * per, hi = min(n, lo + per);
  for (int i = lo + tid; i < hi; i += 256) {
    const float f = bf2f(r[i]);
    if (f > best) { best = f; bi = i; }
  }
#pragma unroll
  for (int o = 16; o; o >>= 1) {
    const float ov = __shfl_xor_sync(0xffffffffu, best, o);
    const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
    if (ov > best || (ov == best && oi < bi)) { best = ov; bi = oi; }
  }
  if ((tid & 31) == 0) { sv[tid >> 5] = best; si[tid >> 5] = bi; }
  __syncthreads();
  if (tid == 0) {
    for (int i = 1; i < 8; ++i)
      if (sv[i] > best || (sv[i] == best && si[i] < bi)) { best = sv[i]; bi = si[i]; }
    part_val[row * AM_PARTS + part] = best;
    part_idx[row * AM_PARTS + part] = bi;
    __threadfence();
    last = atomicAdd(tickets + row, 1u) == AM_PARTS - 1;
  }
  __syncthreads();
  if (!last || tid != 0) return;
  __threadfence();
  float b = -INFINITY;
  int id = INT_MAX;
  for (int i = 0; i < AM_PARTS; ++i) {
    const float pv = __ldcg(part_val + row * AM_PARTS + i);
    const int pi = __ldcg(part_idx + row * AM_PARTS + i);
    if (pv > b || (pv == b && pi < id)) { b = pv; id = pi; }
  }
  out[row] = id == INT_MAX ? 0 : id;
  tickets[row] = 0u;
}

// Quantized embedding rows (nn.QuantizedEmbedding: mx.dequantize of the
// gathered rows), 4-bit group 64: out[t] = dequant(table[ids[t]]) in bf16.
// Ids outside [0, vocab) write zeros and flag VB_STATUS_BOUNDS.
__global__ void __launch_bounds__(256) embed4_kernel(const int32_t *__restrict__ ids,
                                                     const uint32_t *__restrict__ codes,
                                                     const uint16_t *__restrict__ scales,
                                                     const uint16_t *__restrict__ biases,
                                                     int vocab, int H,
                                                     uint16_t *__restrict__ out,
                                                     int32_t *status) {
  const int t = blockIdx.x;
  pdl_launch_dependents();
  pdl_wait();
  const int id = ids[t];
  const bool ok = id >= 0 && id < vocab;
  if (!ok && threadIdx.x == 0) flag_status(status, VB_STATUS_BOUNDS);
  const int wpr = H >> 3;
  for (int wi = threadIdx.x; wi < wpr; wi += 256) {
    uint4 o4 = make_uint4(0, 0, 0, 0);
    if (ok) {
      const size_t gi = (size_t)id * (H >> 6) + (wi >> 3);
      const uint32_t sc = scales[gi], bi = biases[gi];
      uint32_t o[4];
      dequant4_bf16x2(codes[(size_t)id * wpr + wi], sc | (sc << 16), bi | (bi << 16), o);
      o4 = make_uint4(__byte_perm(o[0], o[1], 0x5410), __byte_perm(o[2], o[3], 0x5410),
                      __byte_perm(o[0], o[1], 0x7632), __byte_perm(o[2], o[3], 0x7632));
    }
    *reinterpret_cast<uint4 *>(out + (size_t)t * H + wi * 8) = o4;
  }
}

// The MTP head's fc input in one launch (qwen3_next_mtp.py:40-46): row t of
// out [T, 2H] = [rms_norm(embed(ids[t])) * w_emb | rms_norm(hidden[t]) * w_hid].
// CTA (t, half) stages its source row in shared memory as bf16 (the
// embedding row dequantized exactly as embed4_kernel does it), then
// normalises it with rms_norm_kernel's arithmetic and summation order, so
// the result equals vb_embed_rows followed by two vb_rms_norm calls.
constexpr int MTPI_MAX_H = 8192;
__global__ void __launch_bounds__(256) mtp_fc_input_kernel(
    const int32_t *__restrict__ ids, const uint32_t *__restrict__ codes,
    const uint16_t *__restrict__ scales, const uint16_t *__restrict__ biases, int vocab, int H,
    const uint16_t *__restrict__ w_emb, const uint16_t *__restrict__ hidden,
    const uint16_t *__restrict__ w_hid, float eps, uint16_t *__restrict__ out,
    int32_t *status) {
  __shared__ __align__(16) uint16_t row[MTPI_MAX_H];
  __shared__ float red[8];
  const int t = blockIdx.x, half = blockIdx.y, tid = threadIdx.x;
  pdl_launch_dependents();
  pdl_wait();
  if (half == 0) {
    const int id = ids[t];
    const bool ok = id >= 0 && id < vocab;
    if (!ok && tid == 0) flag_status(status, VB_STATUS_BOUNDS);
    const int wpr = H >> 3;
    for (int wi = tid; wi < wpr; wi += 256) {
      uint4 o4 = make_uint4(0, 0, 0, 0);
      if (ok) {
        const size_t gi = (size_t)id * (H >> 6) + (wi >> 3);
        const uint32_t sc = scales[gi], bi = biases[gi];
        uint32_t o[4];
        dequant4_bf16x2(codes[(size_t)id * wpr + wi], sc | (sc << 16), bi | (bi << 16), o);
        o4 = make_uint4(__byte_perm(o[0], o[1], 0x5410), __byte_perm(o[2], o[3], 0x5410),
                        __byte_perm(o[0], o[1], 0x7632), __byte_perm(o[2], o[3], 0x7632));
      }
      *reinterpret_cast<uint4 *>(row + wi * 8) = o4;
    }
  } else {
    for (int k = tid * 8; k < H; k += 256 * 8)
      *reinterpret_cast<uint4 *>(row + k) =
          *reinterpret_cast<const uint4 *>(hidden + (size_t)t * H + k);
  }
  __syncthreads();
  float ss = 0.f;
  for (int k = tid; k < H; k += 256) {
    const float v = bf2f(row[k]);
    ss = fmaf(v, v, ss);
  }
#pragma unroll
  for (int o = 16; o; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
  if ((tid & 31) == 0) red[tid >> 5] = ss;
  __syncthreads();
  float tot = 0.f;
#pragma unroll
  for (int i = 0; i < 8; ++i) tot += red[i];
  const float inv = rsqrtf(tot / (float)H + eps);
  const uint16_t *w = half == 0 ? w_emb : w_hid;
  uint16_t *y = out + (size_t)t * 2 * H + half * H;
  for (int k = tid; k < H; k += 256) {
    const float nv = rbf(bf2f(row[k]) * inv);
    y[k] = f2bf(w ? nv * bf2f(w[k]) : nv);
  }
}

static size_t ql_smem_bytes(int K) {
  return (size_t)K * 16 + (size_t)(K / 64) * QL_MAX_T * 4;
}

static int ql_sm_count() {
  static int n = 0;
  if (!n) {
    int dev = 0;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
    if (n <= 0) n = 148;
  }
  return n;
}

template <int GPW>
static cudaError_t ql_launch(const QlParams &p, cudaStream_t s) {
  static bool attr_done = false;
  const size_t smem = ql_smem_bytes(p.K);
  if (!attr_done) {
    cudaFuncSetAttribute(qlinear_kernel<GPW>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                         (int)ql_smem_bytes(QL_MAX_K));
    attr_done = true;
  }
  const int grid = min(p.items, 2 * ql_sm_count());
  return vb_launch(qlinear_kernel<GPW>, dim3(grid), dim3(QL_THREADS), smem, s, false, p);
}

}  // namespace vb

using namespace vb;

extern "C" {

size_t vb_qlinear_workspace_size(int32_t tokens, int32_t in_features, int32_t out_features) {
  (void)tokens; (void)in_features; (void)out_features;
  return 0;  // no scratch: the K reduction stays inside a CTA
}

int vb_qlinear(const uint16_t *x, int32_t tokens, int32_t in_features,
               const uint32_t *codes, const uint16_t *scales, const uint16_t *biases,
               int32_t out_features, int32_t group, int32_t bits, const uint16_t *norm_w,
               float norm_eps, const uint16_t *residual, uint16_t *y, void *workspace,
               size_t workspace_bytes, vb_stream_t stream) {
  (void)workspace; (void)workspace_bytes;
  VB_REQUIRE(tokens >= 1 && tokens <= QL_MAX_T, "vb_qlinear: tokens=%d (1..%d)", tokens,
             QL_MAX_T);
  VB_REQUIRE(group == 64 && bits == 4, "vb_qlinear: group %d bits %d (64, 4 only)", group, bits);
  VB_REQUIRE(in_features >= 256 && in_features % 256 == 0 && in_features <= QL_MAX_K &&
                 (in_features <= 2048 || in_features % 512 == 0),
             "vb_qlinear: in_features %d (a multiple of 256 up to 2048, of 512 up to %d)",
             in_features, QL_MAX_K);
  VB_REQUIRE(out_features >= 1, "vb_qlinear: out_features %d", out_features);
  VB_REQUIRE(x && codes && scales && biases && y, "vb_qlinear: null tensor");
  VB_REQUIRE(((uintptr_t)x % 16) == 0 && ((uintptr_t)codes % 8) == 0 &&
                 (!norm_w || ((uintptr_t)norm_w % 16) == 0),
             "vb_qlinear: x and norm weights 16-byte aligned, codes 8-byte aligned");
  VB_REQUIRE(!norm_w || norm_eps > 0.f, "vb_qlinear: norm_eps %g", (double)norm_eps);
  VB_REQUIRE(((uintptr_t)scales % 16) == 0 && ((uintptr_t)biases % 16) == 0,
             "vb_qlinear: scales and biases 16-byte aligned");
  QlParams p;
  p.x = x; p.codes = codes; p.scales = scales; p.biases = biases; p.norm_w = norm_w;
  p.residual = residual; p.y = y; p.eps = norm_eps;
  p.T = tokens; p.K = in_features; p.N = out_features;
  p.items = (out_features + 15) / 16;
  const int G = in_features / 64;   // groups; eight warps share them
  const cudaStream_t s = as_stream(stream);
  if (G <= 8)
    ql_launch<1>(p, s);
  else if (G <= 16)
    ql_launch<2>(p, s);
  else if (G <= 32)
    ql_launch<4>(p, s);
  else
    ql_launch<8>(p, s);
  return check_launch("qlinear_kernel");
}

int vb_rms_norm(const uint16_t *x, const uint16_t *residual, const uint16_t *weight,
                int32_t rows, int32_t dim, float eps, uint16_t *h_out, uint16_t *y,
                int32_t y_stride, vb_stream_t stream) {
  VB_REQUIRE(rows >= 1 && dim >= 1 && eps > 0.f, "vb_rms_norm: rows=%d dim=%d eps=%g", rows,
             dim, (double)eps);
  VB_REQUIRE(y_stride == 0 || y_stride >= dim, "vb_rms_norm: y_stride %d < dim %d", y_stride,
             dim);
  VB_REQUIRE(x && y, "vb_rms_norm: null tensor");
  vb_launch(rms_norm_kernel, dim3(rows), dim3(256), 0, as_stream(stream), false, x, residual,
            weight, dim, eps, h_out, y, (int)(y_stride ? y_stride : dim));
  return check_launch("rms_norm_kernel");
}

size_t vb_argmax_workspace_size(int32_t rows) {
  if (rows < 1) return 0;
  return align_up((size_t)rows * sizeof(uint32_t), 256) +
         (size_t)rows * AM_PARTS * (sizeof(float) + sizeof(int32_t));
}

int vb_argmax(const uint16_t *values, int32_t rows, int32_t n, int32_t *out, void *workspace,
              size_t workspace_bytes, vb_stream_t stream) {
  VB_REQUIRE(rows >= 1 && n >= 1, "vb_argmax: rows=%d n=%d", rows, n);
  VB_REQUIRE(values && out, "vb_argmax: null tensor");
  const size_t need = vb_argmax_workspace_size(rows);
  VB_REQUIRE(workspace && workspace_bytes >= need,
             "vb_argmax: workspace %zu bytes, %zu needed (zero-filled once)", workspace_bytes,
             need);
  uint32_t *tickets = reinterpret_cast<uint32_t *>(workspace);
  float *pv = reinterpret_cast<float *>((char *)workspace +
                                        align_up((size_t)rows * sizeof(uint32_t), 256));
  int32_t *pi = reinterpret_cast<int32_t *>(pv + (size_t)rows * AM_PARTS);
  vb_launch(argmax_kernel, dim3(rows, AM_PARTS), dim3(256), 0, as_stream(stream), false, values,
            (int)n, pv, pi, tickets, out);
  return check_launch("argmax_kernel");
}

int vb_mtp_fc_input(const int32_t *ids, int32_t tokens, const uint32_t *codes,
                    const uint16_t *scales, const uint16_t *biases, int32_t vocab,
                    int32_t hidden, const uint16_t *emb_norm_w, const uint16_t *prev_hidden,
                    const uint16_t *hid_norm_w, float eps, uint16_t *out, int32_t *status,
                    vb_stream_t stream) {
  VB_REQUIRE(tokens >= 1 && vocab >= 1 && hidden >= 64 && hidden % 64 == 0 &&
                 hidden <= MTPI_MAX_H && eps > 0.f,
             "vb_mtp_fc_input: tokens=%d vocab=%d hidden=%d", tokens, vocab, hidden);
  VB_REQUIRE(ids && codes && scales && biases && prev_hidden && out,
             "vb_mtp_fc_input: null tensor");
  VB_REQUIRE(((uintptr_t)prev_hidden % 16) == 0, "vb_mtp_fc_input: hidden rows 16-byte aligned");
  vb_launch(mtp_fc_input_kernel, dim3(tokens, 2), dim3(256), 0, as_stream(stream), false, ids,
            codes, scales, biases, (int)vocab, (int)hidden, emb_norm_w, prev_hidden, hid_norm_w,
            eps, out, status);
  return check_launch("mtp_fc_input_kernel");
}

int vb_embed_rows(const int32_t *ids, int32_t tokens, const uint32_t *codes,
                  const uint16_t *scales, const uint16_t *biases, int32_t vocab,
                  int32_t hidden, int32_t group, int32_t bits, uint16_t *out, int32_t *status,
                  vb_stream_t stream) {
  VB_REQUIRE(tokens >= 1 && vocab >= 1 && hidden >= 64 && hidden % 64 == 0,
             "vb_embed_rows: tokens=%d vocab=%d hidden=%d", tokens, vocab, hidden);
  VB_REQUIRE(group == 64 && bits == 4, "vb_embed_rows: group %d bits %d (64, 4 only)", group,
             bits);
  VB_REQUIRE(ids && codes && scales && biases && out, "vb_embed_rows: null tensor");
  VB_REQUIRE(((uintptr_t)out % 16) == 0, "vb_embed_rows: out must be 16-byte aligned");
  vb_launch(embed4_kernel, dim3(tokens), dim3(256), 0, as_stream(stream), false, ids, codes, scales,
            biases, (int)vocab, (int)hidden, out, status);
  return check_launch("embed4_kernel");
}

}  // extern "C"
