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
// vb_qlinear, T <= 8 tokens (HBM-bound, 0.5 B per weight): a CTA of 8 warps
// owns 128 output rows (16 per warp) and a K slice of KS groups of 64
// columns; the K slices of one row block are separate CTAs whose float32
// partials are added, in slice order, by the last CTA to finish (a ticket per
// row block, reset by that CTA, so the kernel is deterministic and replayable
// in a CUDA graph). Each lane loads its 8-byte share of every group of rows
// g and g+8 up front, turns the codes into exact bf16 pairs 128 + q (LOP3)
// and runs mma.m16n8k16 against x staged in shared memory in fragment order;
// the group's scale and bias are applied as s * D + (b - 128 s) * sum(x).
#include "common.cuh"

namespace vb {

constexpr int QL_THREADS = 256;
constexpr int QL_ROWS = 128;     // output rows per CTA (16 per warp)
constexpr int QL_MAX_T = 8;
constexpr int QL_MAX_S = 16;     // K slices per row block (K <= 4096)

struct QlParams {
  const uint16_t *x;            // bf16 [T, K]
  const uint32_t *codes;        // [N, K/8]
  const uint16_t *scales, *biases;  // bf16 [N, K/64]
  const uint16_t *norm_w;       // nullable bf16 [K]: x -> rms_norm(x) * w
  const uint16_t *residual;     // nullable bf16 [T, N]
  uint16_t *y;                  // bf16 [T, N]
  float *partial;               // [S, T, N] when S > 1
  uint32_t *tickets;            // [ceil(N/128)] when S > 1, zero between launches
  float eps;
  int T, K, N, S;
};

// Stage the K slice of x (optionally RMS-normalised) in fragment order.
// Fragment of MMA m = 4 j + mm (group j of the slice, mm = 2 jw + h) for lane
// (n = lane / 4, c = lane % 4): the word of 8 codes this lane holds for that
// MMA covers columns kb .. kb+7 with kb = 64 (slice group) + 8 (2c + jw); the
// A pairs it feeds are nibbles (2h, 2h+4) and (2h+1, 2h+5) of that word, so
// b0 = x[n][kb + 2h], x[n][kb + 2h + 4] and b1 = x[n][kb + 2h + 1],
// x[n][kb + 2h + 5].
template <int KS>
__global__ void __launch_bounds__(QL_THREADS) qlinear_kernel(QlParams p) {
  __shared__ __align__(16) uint16_t xs_raw[QL_MAX_T][KS * 64];
  __shared__ __align__(16) uint2 xfrag[KS * 4][32];
  __shared__ float xsum[KS][QL_MAX_T];
  __shared__ float inv_rms[QL_MAX_T];
  __shared__ int last_cta;

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int g = lane >> 2, c = lane & 3;
  const int rb = blockIdx.x, s = blockIdx.y;
  const int K = p.K, N = p.N, T = p.T;
  const int wpr = K >> 3, gpr = K >> 6;
  const int grp0 = s * KS;
  const int ra = rb * QL_ROWS + warp * 16 + g, rb8 = ra + 8;
  const bool va = ra < N, vb8 = rb8 < N;

  // 1. Weight codes of both rows for every group of the slice, then scales
  //    and biases (KS consecutive bf16 per row).
  uint2 wa[KS], wb[KS];
#pragma unroll
  for (int j = 0; j < KS; ++j) {
    const int off = (grp0 + j) * 8 + 2 * c;
    wa[j] = va ? ldg_nc_v2(p.codes + (size_t)ra * wpr + off) : make_uint2(0, 0);
    wb[j] = vb8 ? ldg_nc_v2(p.codes + (size_t)rb8 * wpr + off) : make_uint2(0, 0);
  }
  // KS consecutive bf16 scales (biases) of a row: one 16-byte (KS = 8) or
  // 8-byte (KS = 4) load each; word i holds groups 2i (low) and 2i+1 (high)
  uint32_t sa[KS / 2], sb[KS / 2], ba[KS / 2], bb[KS / 2];
  {
    const size_t oa = (size_t)ra * gpr + grp0, ob = (size_t)rb8 * gpr + grp0;
    if constexpr (KS == 8) {
      const uint4 z = make_uint4(0, 0, 0, 0);
      const uint4 s0 = va ? ldg_nc_v4(p.scales + oa) : z, b0 = va ? ldg_nc_v4(p.biases + oa) : z;
      const uint4 s1 = vb8 ? ldg_nc_v4(p.scales + ob) : z, b1 = vb8 ? ldg_nc_v4(p.biases + ob) : z;
      sa[0] = s0.x; sa[1] = s0.y; sa[2] = s0.z; sa[3] = s0.w;
      ba[0] = b0.x; ba[1] = b0.y; ba[2] = b0.z; ba[3] = b0.w;
      sb[0] = s1.x; sb[1] = s1.y; sb[2] = s1.z; sb[3] = s1.w;
      bb[0] = b1.x; bb[1] = b1.y; bb[2] = b1.z; bb[3] = b1.w;
    } else {
      const uint2 z = make_uint2(0, 0);
      const uint2 s0 = va ? ldg_nc_v2(p.scales + oa) : z, b0 = va ? ldg_nc_v2(p.biases + oa) : z;
      const uint2 s1 = vb8 ? ldg_nc_v2(p.scales + ob) : z, b1 = vb8 ? ldg_nc_v2(p.biases + ob) : z;
      sa[0] = s0.x; sa[1] = s0.y; ba[0] = b0.x; ba[1] = b0.y;
      sb[0] = s1.x; sb[1] = s1.y; bb[0] = b1.x; bb[1] = b1.y;
    }
  }
  // Everything above is weights. The kernels of the decode stack are
  // launched plainly (a programmatic-dependent launch of every kernel was
  // measured slower in the 48-layer graph), so pdl_wait is a no-op; the
  // trigger lets a programmatic dependent (the MoE block kernel) launch
  // while this grid drains.
  pdl_launch_dependents();
  pdl_wait();

  // 2. x: inverse RMS over the whole row (warp t takes token t), then the
  //    slice, normalised as bf16(bf16(x * inv) * w).
  if (p.norm_w) {
    for (int t = warp; t < T; t += QL_THREADS / 32) {
      const uint16_t *xr = p.x + (size_t)t * K;
      float ss = 0.f;
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
  for (int i = tid; i < QL_MAX_T * KS * 8; i += QL_THREADS) {
    const int t = i / (KS * 8), k8 = (i % (KS * 8)) * 8;
    uint4 v = make_uint4(0, 0, 0, 0);
    if (t < T) {
      v = *reinterpret_cast<const uint4 *>(p.x + (size_t)t * K + grp0 * 64 + k8);
      if (p.norm_w) {
        const uint4 w = *reinterpret_cast<const uint4 *>(p.norm_w + grp0 * 64 + k8);
        uint32_t xv[4] = {v.x, v.y, v.z, v.w};
        const uint32_t wv[4] = {w.x, w.y, w.z, w.w};
        const float inv = inv_rms[t];
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          const float lo = rbf(__uint_as_float(xv[q] << 16) * inv);
          const float hi = rbf(__uint_as_float(xv[q] & 0xFFFF0000u) * inv);
          xv[q] = pack_bf2(lo * __uint_as_float(wv[q] << 16),
                           hi * __uint_as_float(wv[q] & 0xFFFF0000u));
        }
        v = make_uint4(xv[0], xv[1], xv[2], xv[3]);
      }
    }
    *reinterpret_cast<uint4 *>(&xs_raw[t][k8]) = v;
  }
  __syncthreads();
  for (int i = tid; i < KS * 4 * 32; i += QL_THREADS) {
    const int m = i >> 5, l = i & 31;
    const int j = m >> 2, mm = m & 3, jw = mm >> 1, h = mm & 1;
    const int n = l >> 2, cc = l & 3;
    const int kb = j * 64 + 8 * (2 * cc + jw) + 2 * h;
    const uint16_t *xr = xs_raw[n];
    xfrag[m][l] = make_uint2((uint32_t)xr[kb] | ((uint32_t)xr[kb + 4] << 16),
                             (uint32_t)xr[kb + 1] | ((uint32_t)xr[kb + 5] << 16));
  }
  // per-group sums of x: warp j takes group j, lane (n, quarter) 16 columns,
  // the quarters added by shuffles (fixed order)
  if (warp < KS) {
    const int n = lane >> 2, qq = lane & 3;
    float sum = 0.f;
#pragma unroll
    for (int k = 0; k < 16; ++k) sum += bf2f(xs_raw[n][warp * 64 + qq * 16 + k]);
    sum += __shfl_xor_sync(0xffffffffu, sum, 1);
    sum += __shfl_xor_sync(0xffffffffu, sum, 2);
    if (qq == 0) xsum[warp][n] = sum;
  }
  __syncthreads();

  // 3. Four MMAs per group, then the group's scale and bias.
  float acc[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
  for (int j = 0; j < KS; ++j) {
    float d[4] = {0.f, 0.f, 0.f, 0.f};
    uint32_t pa[2][4], pb[2][4];
    nib_pairs4(wa[j].x, pa[0]);
    nib_pairs4(wa[j].y, pa[1]);
    nib_pairs4(wb[j].x, pb[0]);
    nib_pairs4(wb[j].y, pb[1]);
#pragma unroll
    for (int mm = 0; mm < 4; ++mm) {
      const int jw = mm >> 1, h = mm & 1;
      const uint2 bf = xfrag[j * 4 + mm][lane];
      mma_bf16(d, pa[jw][2 * h], pb[jw][2 * h], pa[jw][2 * h + 1], pb[jw][2 * h + 1], bf.x, bf.y);
    }
    const int sh = (j & 1) ? 0 : 16;  // low half: even group
    const float s_a = __uint_as_float((sa[j >> 1] << sh) & 0xFFFF0000u);
    const float s_b = __uint_as_float((sb[j >> 1] << sh) & 0xFFFF0000u);
    const float c_a = __uint_as_float((ba[j >> 1] << sh) & 0xFFFF0000u) - 128.f * s_a;
    const float c_b = __uint_as_float((bb[j >> 1] << sh) & 0xFFFF0000u) - 128.f * s_b;
    const float x0 = xsum[j][2 * c], x1 = xsum[j][2 * c + 1];
    acc[0] += fmaf(s_a, d[0], c_a * x0);
    acc[1] += fmaf(s_a, d[1], c_a * x1);
    acc[2] += fmaf(s_b, d[2], c_b * x0);
    acc[3] += fmaf(s_b, d[3], c_b * x1);
  }

  // 4. Output: directly when the row block has one slice, else partials and
  //    the last CTA's ordered reduction.
  const int n0 = 2 * c, n1 = 2 * c + 1;
  if (p.S == 1) {
    const int rows[2] = {ra, rb8};
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      const int row = rows[q >> 1], n = (q & 1) ? n1 : n0;
      if (row < N && n < T) {
        float v = rbf(acc[q]);
        if (p.residual) v = bf2f(p.residual[(size_t)n * N + row]) + v;
        p.y[(size_t)n * N + row] = f2bf(v);
      }
    }
    return;
  }
  {
    const int rows[2] = {ra, rb8};
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      const int row = rows[q >> 1], n = (q & 1) ? n1 : n0;
      if (row < N && n < T) p.partial[((size_t)s * T + n) * N + row] = acc[q];
    }
  }
  __threadfence();
  __syncthreads();
  if (tid == 0) {
    const uint32_t ticket = atomicAdd(p.tickets + rb, 1u);
    last_cta = ticket == (uint32_t)(p.S - 1);
  }
  __syncthreads();
  if (!last_cta) return;
  __threadfence();
  const int row0 = rb * QL_ROWS;
  for (int i = tid; i < QL_ROWS * T; i += QL_THREADS) {
    const int n = i / QL_ROWS, row = row0 + i % QL_ROWS;
    if (row >= N) continue;
    float part[QL_MAX_S];
#pragma unroll
    for (int ss = 0; ss < QL_MAX_S; ++ss)
      part[ss] = ss < p.S ? __ldcg(p.partial + ((size_t)ss * T + n) * N + row) : 0.f;
    float v = 0.f;
#pragma unroll
    for (int ss = 0; ss < QL_MAX_S; ++ss) v += part[ss];
    v = rbf(v);
    if (p.residual) v = bf2f(p.residual[(size_t)n * N + row]) + v;
    p.y[(size_t)n * N + row] = f2bf(v);
  }
  if (tid == 0) p.tickets[rb] = 0u;
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

// Groups per K slice: 8 when the grid still has two CTAs per SM with it,
// else 4 (more slices for narrow outputs).
static int ql_slice_groups(int K, int N) {
  const long blocks = (N + QL_ROWS - 1) / QL_ROWS;
  return (K % 512 == 0 && blocks * (K / 512) >= 2 * 148) ? 8 : 4;
}

}  // namespace vb

using namespace vb;

extern "C" {

size_t vb_qlinear_workspace_size(int32_t tokens, int32_t in_features, int32_t out_features) {
  if (tokens < 1 || in_features < 256 || out_features < 1) return 0;
  const int S = in_features / 64 / ql_slice_groups(in_features, out_features);
  const size_t blocks = (size_t)(out_features + QL_ROWS - 1) / QL_ROWS;
  if (S <= 1) return 0;
  return align_up(blocks * sizeof(uint32_t), 256) +
         (size_t)S * tokens * out_features * sizeof(float);
}

int vb_qlinear(const uint16_t *x, int32_t tokens, int32_t in_features,
               const uint32_t *codes, const uint16_t *scales, const uint16_t *biases,
               int32_t out_features, int32_t group, int32_t bits, const uint16_t *norm_w,
               float norm_eps, const uint16_t *residual, uint16_t *y, void *workspace,
               size_t workspace_bytes, vb_stream_t stream) {
  VB_REQUIRE(tokens >= 1 && tokens <= QL_MAX_T, "vb_qlinear: tokens=%d (1..%d)", tokens,
             QL_MAX_T);
  VB_REQUIRE(group == 64 && bits == 4, "vb_qlinear: group %d bits %d (64, 4 only)", group, bits);
  VB_REQUIRE(in_features >= 256 && in_features % 256 == 0,
             "vb_qlinear: in_features %d (a multiple of 256)", in_features);
  VB_REQUIRE(out_features >= 1, "vb_qlinear: out_features %d", out_features);
  VB_REQUIRE(x && codes && scales && biases && y, "vb_qlinear: null tensor");
  VB_REQUIRE(((uintptr_t)x % 16) == 0 && ((uintptr_t)codes % 8) == 0 &&
                 (!norm_w || ((uintptr_t)norm_w % 16) == 0),
             "vb_qlinear: x and norm weights 16-byte aligned, codes 8-byte aligned");
  VB_REQUIRE(!norm_w || norm_eps > 0.f, "vb_qlinear: norm_eps %g", (double)norm_eps);
  VB_REQUIRE(((uintptr_t)scales % 16) == 0 && ((uintptr_t)biases % 16) == 0,
             "vb_qlinear: scales and biases 16-byte aligned");
  const int KS = ql_slice_groups(in_features, out_features);
  QlParams p;
  p.x = x; p.codes = codes; p.scales = scales; p.biases = biases; p.norm_w = norm_w;
  p.residual = residual; p.y = y; p.eps = norm_eps;
  p.T = tokens; p.K = in_features; p.N = out_features;
  p.S = in_features / 64 / KS;
  p.partial = nullptr; p.tickets = nullptr;
  const int blocks = (out_features + QL_ROWS - 1) / QL_ROWS;
  if (p.S > 1) {
    const size_t need = vb_qlinear_workspace_size(tokens, in_features, out_features);
    VB_REQUIRE(workspace && workspace_bytes >= need,
               "vb_qlinear: workspace %zu bytes, %zu needed (zero-filled once)", workspace_bytes,
               need);
    p.tickets = reinterpret_cast<uint32_t *>(workspace);
    p.partial = reinterpret_cast<float *>((char *)workspace +
                                          align_up((size_t)blocks * sizeof(uint32_t), 256));
  }
  VB_REQUIRE(p.S <= QL_MAX_S, "vb_qlinear: %d K slices (in_features <= %d)", p.S,
             QL_MAX_S * 4 * 64);
  const dim3 grid(blocks, p.S);
  cudaError_t e;
  if (KS == 8)
    e = vb_launch(qlinear_kernel<8>, grid, dim3(QL_THREADS), 0, as_stream(stream), false, p);
  else
    e = vb_launch(qlinear_kernel<4>, grid, dim3(QL_THREADS), 0, as_stream(stream), false, p);
  if (e != cudaSuccess) return check_launch("qlinear_kernel");
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
