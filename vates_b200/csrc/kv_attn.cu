// Quantized GQA decode attention directly over the packed IsoQuant cache.
//
// Reference: asym_quantized_sdpa (mlx_streaming/core/cache/quant_kv.py:
// 212-249): q*scale (bf16) -> quantized_matmul(q, K^T) (bf16 scores) ->
// causal mask -> precise softmax -> quantized_matmul(p, V) -> bf16, then the
// inverse V rotation (kv_quant_patch.py:67-68).
//
// Split-K ("flash decoding"): each CTA owns one (batch, kv head) and a
// contiguous key range processed in 16-key tiles; a combine kernel merges the
// per-split (max, sum, output) triples in split order. Two partial kernels:
// kv_attn1_kernel for up to 8 query rows per kv head (decode, T = 1; every
// warp owns whole tiles) and kv_attn4_kernel for 9..32 rows (MTP verify,
// T = 4; the CTA shares each unpacked tile, warp w takes rows 8w..8w+7).
// Both compute S^T = K Q^T and O^T += V^T P^T on mma.sync with the codes as
// exact bf16 values 128 + code, the per-64-dim-group scale and bias applied
// as s*D + (b - 128 s)*sum and the V bias term sum(p*b) on the CUDA cores;
// scores and P are rounded to bf16 as MLX does.
#include "common.cuh"

namespace vb {

constexpr int ATT_ROUND = 64;

struct AttnParams {
  const uint16_t *q;
  const uint32_t *kc, *vc;
  const uint16_t *ks, *kb, *vs, *vb;
  const float *rv;
  const int32_t *pos_dev;  // nullable: S = *pos_dev + pos_add + L read on the device
  int pos_add;
  int B, Hq, Hkv, L, S, cap, rep, QR, causal, nsplit, kps;
  float scale;
  float *opart, *mpart, *lpart;
  // gate (nullable, batch 1): out receives bf16(o * bf16(sigmoid(g))) in
  // [L, Hq * 256] with g = gate[l * gate_stride + hq * 512 + 256 + d] (the
  // gate half of each query head's projection), else o in [B, Hq, L, 256]
  const uint16_t *gate;
  int gate_stride;
  uint16_t *out;
};

__device__ __forceinline__ void ldsm_x4_trans(uint32_t &r0, uint32_t &r1, uint32_t &r2,
                                              uint32_t &r3, const void *smem_ptr) {
  const uint32_t a = (uint32_t)__cvta_generic_to_shared(smem_ptr);
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3) : "r"(a));
}

__device__ __forceinline__ float bf_at2(const uint2 &v, int i) {
  const uint32_t w = i < 2 ? v.x : v.y;
  return (i & 1) ? __uint_as_float(w & 0xFFFF0000u) : __uint_as_float(w << 16);
}

constexpr int ATT_MAX_SPLITS = 1024;

__global__ void __launch_bounds__(256, 4) kv_attn_combine_kernel(AttnParams p) {
  pdl_launch_dependents();
  pdl_wait();  // no-op unless launched as a programmatic dependent
  __shared__ float s_red[256];
  __shared__ float s_e[ATT_MAX_SPLITS];
  __shared__ float s_num[8][32];
  __shared__ float ov[32];
  const int row_id = blockIdx.x;  // ((b*Hq + hq)*L + l)
  const int chunk = blockIdx.y;   // dims [32 chunk, 32 chunk + 32)
  const int l = row_id % p.L;
  const int bhq = row_id / p.L;
  const int b = bhq / p.Hq, hq = bhq % p.Hq;
  const int hkv = hq / p.rep, rep_i = hq % p.rep;
  const int r = rep_i * p.L + l;
  const size_t bh = (size_t)b * p.Hkv + hkv;
  const int tid = threadIdx.x;
  const int ns = p.nsplit;
  // the gate value of this thread's output dim, loaded before the reductions
  float gv = 0.f;
  if (p.gate && tid < 32)
    gv = bf2f(p.gate[(size_t)l * p.gate_stride + hq * 512 + 256 + 32 * chunk + tid]);
  // The first 256 splits' maxima and sums and this thread's first 16
  // partial outputs are loaded before any of them is used (one memory round
  // trip instead of three); the sums below keep the split order.
  const int wid = tid >> 5;
  const int dl = tid & 31, sl = tid >> 5;
  const int d = 32 * chunk + dl;
  // splits sl + 8 j, j < CB_PRE, in registers: 16 keeps the kernel at 64
  // registers, four CTAs per SM (32 raised it to 70 and three CTAs, slower on
  // short caches with few splits)
  constexpr int CB_PRE = 16;
  const float mp0 = tid < ns ? p.mpart[(bh * ns + tid) * 32 + r] : -INFINITY;
  const float lp0 = tid < ns ? p.lpart[(bh * ns + tid) * 32 + r] : 0.f;
  float opre[CB_PRE];
#pragma unroll
  for (int j = 0; j < CB_PRE; ++j) {
    const int s = sl + 8 * j;
    opre[j] = s < ns ? p.opart[((bh * ns + s) * 32 + r) * 256 + d] : 0.f;
  }
  // maximum and denominator: per-thread partials, warp shuffles, then the 8
  // warp values in warp order (one block barrier each)
  float m = mp0;
  for (int s = tid + 256; s < ns; s += 256) m = fmaxf(m, p.mpart[(bh * ns + s) * 32 + r]);
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
  if ((tid & 31) == 0) s_red[wid] = m;
  __syncthreads();
  float M = s_red[0];
#pragma unroll
  for (int w = 1; w < 8; ++w) M = fmaxf(M, s_red[w]);
  float dn = 0.f;
  for (int s = tid; s < ns; s += 256) {
    const size_t cta = bh * ns + s;
    const float ms = s == tid ? mp0 : p.mpart[cta * 32 + r];
    const float e = ms == -INFINITY ? 0.f : expf(ms - M);
    s_e[s] = e;
    dn = fmaf(s == tid ? lp0 : p.lpart[cta * 32 + r], e, dn);
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) dn += __shfl_xor_sync(0xffffffffu, dn, o);
  if ((tid & 31) == 0) s_red[8 + wid] = dn;
  __syncthreads();
  float den = 0.f;
#pragma unroll
  for (int w = 0; w < 8; ++w) den += s_red[8 + w];
  float num = 0.f;
#pragma unroll
  for (int j = 0; j < CB_PRE; ++j) {
    const int s = sl + 8 * j;
    if (s < ns) num = fmaf(opre[j], s_e[s], num);
  }
#pragma unroll 4
  for (int s = sl + 8 * CB_PRE; s < ns; s += 8)
    num = fmaf(p.opart[((bh * ns + s) * 32 + r) * 256 + d], s_e[s], num);
  s_num[sl][dl] = num;
  __syncthreads();
  if (tid < 32) {
    float nm = 0.f;
#pragma unroll
    for (int i = 0; i < 8; ++i) nm += s_num[i][tid];
    float o = rbf(den > 0.f ? nm / den : 0.f);
    ov[tid] = o;
    __syncwarp();
    if (p.rv) {
      const int blk = d >> 2, i = d & 3;
      const float *R = p.rv + (size_t)blk * 16;
      float acc = 0.f;
#pragma unroll
      for (int kk = 0; kk < 4; ++kk)
        acc = __fadd_rn(acc, __fmul_rn(ov[(tid & ~3) + kk], rbf(__ldg(R + i * 4 + kk))));
      o = rbf(acc);
    }
    if (p.gate)  // attention output times the sigmoid gate (kv_quant_patch.py:70-71)
      p.out[((size_t)l * p.Hq + hq) * 256 + d] = f2bf(o * rbf(mlx_sigmoid(gv)));
    else
      p.out[(size_t)row_id * 256 + d] = f2bf(o);
  }
}

// ----------------------------------------------------------------------------
// Single-query-position path (rep * L <= 8 query rows per kv head, i.e. GQA
// decode at T=1): every warp owns whole 16-key tiles. Scores are computed
// transposed, S^T[key][row] = K * Q^T, with the 4-bit K codes as the A
// operand (exact bf16 128+q by one LOP3 per pair) and the 8 query rows as
// the N=8 columns; per 64-dim group the epilogue applies s*D + (b-128s)*sum(q)
// and the group partials are added in group order, then rounded to bf16.
// The output is accumulated transposed too, O^T[dim][row] += V^T * P^T, with
// V unpacked to exact bf16 in shared memory (read as A by ldmatrix.trans)
// and P (bf16, times the key's V scale of the dim group) moved from the S^T
// accumulator layout to the B layout with movmatrix.trans. Raw K/V codes and
// scales of the next tile are prefetched with cp.async. The 4 warps' partial
// softmax states are merged in shared memory into the CTA's split partial.
// ----------------------------------------------------------------------------
constexpr int A1_WARPS = 4;
constexpr int A1_VPITCH = 256 + 8;                       // bf16 per unpacked V row
constexpr int A1_VBYTES = 16 * A1_VPITCH * 2;            // 8448
constexpr int A1_RAW = 16 * 128 + 16 * 96 + 4 * 16 * 8;  // K codes, V codes, 4 scale tensors
constexpr int A1_WARP_SMEM = A1_VBYTES + 2 * A1_RAW;     // 16640
constexpr int A1_SMEM = A1_WARPS * A1_WARP_SMEM;

// Codes at bits s0 and s0+3 of u (3-bit) -> bf16 pair (128 + c0, 128 + c1).
__device__ __forceinline__ uint32_t v3_pair128(uint32_t u, int s0) {
  const uint32_t a = u >> s0;
  return lop_and_or(a << 13, 0x00070000u, lop_and_or(a, 0x7u, 0x43004300u));
}

__device__ __forceinline__ uint32_t movmatrix_trans(uint32_t x) {
  uint32_t y;
  asm volatile("movmatrix.sync.aligned.m8n8.trans.b16 %0, %1;" : "=r"(y) : "r"(x));
  return y;
}
__device__ __forceinline__ uint2 lds_u2(const uint8_t *p) {
  return *reinterpret_cast<const uint2 *>(p);
}

// Raw tile (16 keys from key0; keys past S-1 read key S-1 and are masked
// later) -> staging buffer: K codes [16][128 B], V codes [16][96 B], then
// the K scale, K bias, V scale, V bias of each key [4][16][8 B]. A lane's
// chunks are fixed: keys key0 + kq[i] at byte offsets that do not change
// from tile to tile.
__device__ __forceinline__ void a1_fetch(const uint8_t *kbase, const uint8_t *vbase,
                                         const uint8_t *s0, const uint8_t *s1, int S, int key0,
                                         uint8_t *raw, int lane) {
  // K codes: piece lane + 32 i, i < 4 -> key (lane >> 3) + 4 i, offset (lane & 7) * 16
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const int key = min(key0 + (lane >> 3) + 4 * i, S - 1);
    cp_async16(raw + (lane + 32 * i) * 16, kbase + (size_t)key * 128 + (lane & 7) * 16);
  }
  // V codes: pieces 128 + lane + 32 i -> key qq / 6, offset (qq % 6) * 16
#pragma unroll
  for (int i = 0; i < 3; ++i) {
    const int qq = lane + 32 * i;
    const int key = min(key0 + qq / 6, S - 1);
    cp_async16(raw + 2048 + qq * 16, vbase + (size_t)key * 96 + (qq % 6) * 16);
  }
  // scales: piece lane + 32 i -> tensor (lane >> 4) + 2 i, key lane & 15
#pragma unroll
  for (int i = 0; i < 2; ++i) {
    const int key = min(key0 + (lane & 15), S - 1);
    cp_async8(raw + 3584 + (lane + 32 * i) * 8, (i ? s1 : s0) + (size_t)key * 8);
  }
}

template <bool DEV_POS>
__global__ void __launch_bounds__(A1_WARPS * 32, 3) kv_attn1_kernel(AttnParams p) {
  extern __shared__ __align__(16) uint8_t smem_raw[];
  if (DEV_POS) {  // launched as a programmatic dependent by the *_at entries
    pdl_launch_dependents();
    pdl_wait();
  }
  const int S_ = DEV_POS ? min(max(*p.pos_dev + p.pos_add, 0) + p.L, p.cap) : p.S;
  const int bh = blockIdx.x, split = blockIdx.y;
  const int b = bh / p.Hkv, hkv = bh % p.Hkv;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int g = lane >> 2, c = lane & 3;
  const int k_begin = split * p.kps;
  const int k_end = min(S_, k_begin + p.kps);
  uint8_t *wsm = smem_raw + warp * A1_WARP_SMEM;
  uint16_t *Vt = reinterpret_cast<uint16_t *>(wsm);
  uint8_t *raw0 = wsm + A1_VBYTES;

  // Q^T as B fragments (row g; zero for rows >= QR) and the per-group q sums
  // of rows 2c, 2c+1. The fragments are the same in every warp of the CTA;
  // they live in shared memory (warp w writes group w), which keeps the tile
  // loop within the register budget of three CTAs per SM without spills.
  __shared__ uint2 s_qb[4][4][32];
  float qs[4][2];
  {
    float vals[64];
    const int r = g;
    float part[4] = {0.f, 0.f, 0.f, 0.f};
    if (r < p.QR) {
      const int rep_i = r / p.L, l = r % p.L;
      const int hq = hkv * p.rep + rep_i;
      const uint16_t *qp = p.q + (((size_t)b * p.Hq + hq) * p.L + l) * 256;
#pragma unroll
      for (int G = 0; G < 4; ++G)
#pragma unroll
        for (int i = 0; i < 16; ++i) {
          const float v = rbf(__fmul_rn(bf2f(qp[64 * G + 16 * c + i]), p.scale));
          vals[16 * G + i] = v;
          part[G] += v;
        }
    } else {
#pragma unroll
      for (int i = 0; i < 64; ++i) vals[i] = 0.f;
    }
#pragma unroll
    for (int G = 0; G < 4; ++G) {
      if (G == warp) {
#pragma unroll
        for (int m = 0; m < 4; ++m) {
          const int d0 = 16 * G + 8 * (m >> 1) + 2 * (m & 1);
          s_qb[G][m][lane] = make_uint2(pack_bf2(vals[d0], vals[d0 + 4]),
                                        pack_bf2(vals[d0 + 1], vals[d0 + 5]));
        }
      }
      float t = part[G];
      t += __shfl_xor_sync(0xffffffffu, t, 1);
      t += __shfl_xor_sync(0xffffffffu, t, 2);
      // row g's sum -> lanes needing rows 2c, 2c+1
      qs[G][0] = __shfl_sync(0xffffffffu, t, (2 * c) * 4);
      qs[G][1] = __shfl_sync(0xffffffffu, t, (2 * c + 1) * 4);
    }
  }
  static_assert(A1_WARPS == 4, "warp w stores the Q fragments of group w");
  __syncthreads();

  float O[16][4];
#pragma unroll
  for (int i = 0; i < 16; ++i) O[i][0] = O[i][1] = O[i][2] = O[i][3] = 0.f;
  float m_run[2] = {-INFINITY, -INFINITY}, l_run[2] = {0.f, 0.f};
  float bsum[4][2], psum[4][2];
#pragma unroll
  for (int G = 0; G < 4; ++G) bsum[G][0] = bsum[G][1] = psum[G][0] = psum[G][1] = 0.f;
  // Last key each of this lane's rows (2c, 2c+1) may see: -1 past the query
  // rows, S - L + position under the causal mask.
  int klim[2];
#pragma unroll
  for (int h = 0; h < 2; ++h) {
    const int row = 2 * c + h;
    klim[h] = row >= p.QR ? -1 : (p.causal ? S_ - p.L + row % p.L : INT_MAX);
  }

  const size_t head_row0 = (size_t)bh * p.cap;
  const int n_tiles = (k_end - k_begin + 15) / 16;
  const uint8_t *kbase = reinterpret_cast<const uint8_t *>(p.kc + head_row0 * 32);
  const uint8_t *vbase = reinterpret_cast<const uint8_t *>(p.vc + head_row0 * 24);
  // scale tensors of this lane's two pieces: (lane >> 4) and (lane >> 4) + 2
  const uint16_t *sc_t[4] = {p.ks, p.kb, p.vs, p.vb};
  const uint8_t *sb0 = reinterpret_cast<const uint8_t *>(((lane >> 4) ? sc_t[1] : sc_t[0]) + head_row0 * 4);
  const uint8_t *sb1 = reinterpret_cast<const uint8_t *>(((lane >> 4) ? sc_t[3] : sc_t[2]) + head_row0 * 4);
  int it = 0;
  int t_cur = warp;
  if (t_cur < n_tiles) a1_fetch(kbase, vbase, sb0, sb1, S_, k_begin + 16 * t_cur, raw0, lane);
  cp_async_commit();
  for (; t_cur < n_tiles; t_cur += A1_WARPS, ++it) {
    const int t_next = t_cur + A1_WARPS;
    if (t_next < n_tiles)
      a1_fetch(kbase, vbase, sb0, sb1, S_, k_begin + 16 * t_next,
               raw0 + ((it + 1) & 1) * A1_RAW, lane);
    cp_async_commit();
    cp_async_wait<1>();
    __syncwarp();
    const uint8_t *rw = raw0 + (it & 1) * A1_RAW;
    const uint8_t *Kr = rw, *Vr = rw + 2048, *Sk = rw + 3584, *Bk = Sk + 128, *Sv = Sk + 256,
                  *Bv = Sk + 384;
    const int key0 = k_begin + 16 * t_cur;

    // ---- scores S^T for keys g, g+8 and rows 2c, 2c+1 ----
    float sc[4] = {0.f, 0.f, 0.f, 0.f};
    const uint2 ksg = lds_u2(Sk + g * 8), ks8 = lds_u2(Sk + (g + 8) * 8);
    const uint2 kbg = lds_u2(Bk + g * 8), kb8 = lds_u2(Bk + (g + 8) * 8);
#pragma unroll
    for (int G = 0; G < 4; ++G) {
      const uint2 wa = lds_u2(Kr + g * 128 + G * 32 + 8 * c);
      const uint2 wb = lds_u2(Kr + (g + 8) * 128 + G * 32 + 8 * c);
      uint32_t pa[2][4], pb[2][4];
      nib_pairs4(wa.x, pa[0]);
      nib_pairs4(wa.y, pa[1]);
      nib_pairs4(wb.x, pb[0]);
      nib_pairs4(wb.y, pb[1]);
      float d[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
      for (int m = 0; m < 4; ++m) {
        const int i0 = 2 * (m & 1), h = m >> 1;
        const uint2 qf = s_qb[G][m][lane];
        mma_bf16(d, pa[h][i0], pb[h][i0], pa[h][i0 + 1], pb[h][i0 + 1], qf.x, qf.y);
      }
      const float s_g = bf_at2(ksg, G), s_8 = bf_at2(ks8, G);
      const float bp_g = fmaf(-128.f, s_g, bf_at2(kbg, G));
      const float bp_8 = fmaf(-128.f, s_8, bf_at2(kb8, G));
      sc[0] += fmaf(s_g, d[0], bp_g * qs[G][0]);
      sc[1] += fmaf(s_g, d[1], bp_g * qs[G][1]);
      sc[2] += fmaf(s_8, d[2], bp_8 * qs[G][0]);
      sc[3] += fmaf(s_8, d[3], bp_8 * qs[G][1]);
    }
    // bf16 scores; mask keys outside [k_begin, k_end), rows >= QR and the
    // causal bound key <= S - L + l.
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const int key = key0 + g + 8 * (j >> 1);
      const bool ok = key < k_end && key <= klim[j & 1];
      sc[j] = ok ? rbf(sc[j]) : -INFINITY;
    }
    // ---- online softmax (rows 2c, 2c+1) ----
    float mx[2] = {fmaxf(sc[0], sc[2]), fmaxf(sc[1], sc[3])};
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      mx[h] = fmaxf(mx[h], __shfl_xor_sync(0xffffffffu, mx[h], 4));
      mx[h] = fmaxf(mx[h], __shfl_xor_sync(0xffffffffu, mx[h], 8));
      mx[h] = fmaxf(mx[h], __shfl_xor_sync(0xffffffffu, mx[h], 16));
    }
    float mnew[2], alpha[2];
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      mnew[h] = fmaxf(m_run[h], mx[h]);
      alpha[h] = (m_run[h] == -INFINITY) ? 0.f : __expf(m_run[h] - mnew[h]);
      if (mnew[h] == -INFINITY) alpha[h] = 1.f;
      m_run[h] = mnew[h];
    }
    if (__any_sync(0xffffffffu, alpha[0] != 1.f || alpha[1] != 1.f)) {
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        l_run[h] *= alpha[h];
#pragma unroll
        for (int G = 0; G < 4; ++G) {
          bsum[G][h] *= alpha[h];
          psum[G][h] *= alpha[h];
        }
      }
#pragma unroll
      for (int i = 0; i < 16; ++i) {
        O[i][0] *= alpha[0];
        O[i][1] *= alpha[1];
        O[i][2] *= alpha[0];
        O[i][3] *= alpha[1];
      }
    }
    float e[4];
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const int h = j & 1;
      e[j] = sc[j] == -INFINITY ? 0.f : __expf(sc[j] - mnew[h]);
      l_run[h] += e[j];
    }
    // P^T fragments per V group: p = bf16(e * vs); V bias term on the side.
    const uint2 vsg = lds_u2(Sv + g * 8), vs8 = lds_u2(Sv + (g + 8) * 8);
    const uint2 vbg = lds_u2(Bv + g * 8), vb8 = lds_u2(Bv + (g + 8) * 8);
    uint32_t pB[4][2];
#pragma unroll
    for (int G = 0; G < 4; ++G) {
      const float sg = bf_at2(vsg, G), s8 = bf_at2(vs8, G);
      const float bg = bf_at2(vbg, G), b8 = bf_at2(vb8, G);
      bsum[G][0] = fmaf(e[0], bg, fmaf(e[2], b8, bsum[G][0]));
      bsum[G][1] = fmaf(e[1], bg, fmaf(e[3], b8, bsum[G][1]));
      const uint32_t x0 = pack_bf2(e[0] * sg, e[1] * sg);  // key g: rows 2c, 2c+1
      const uint32_t x1 = pack_bf2(e[2] * s8, e[3] * s8);  // key g+8
      psum[G][0] += __uint_as_float(x0 << 16) + __uint_as_float(x1 << 16);
      psum[G][1] += __uint_as_float(x0 & 0xFFFF0000u) + __uint_as_float(x1 & 0xFFFF0000u);
      pB[G][0] = movmatrix_trans(x0);  // keys 2c, 2c+1 of row g
      pB[G][1] = movmatrix_trans(x1);  // keys 8+2c, 8+2c+1
    }
    // ---- V codes -> exact bf16 rows of Vt ----
    {
      const int kk = lane >> 1, hh = lane & 1;
      const uint32_t *vw = reinterpret_cast<const uint32_t *>(Vr + kk * 96 + hh * 48);
      uint32_t w[13];
#pragma unroll
      for (int i = 0; i < 12; ++i) w[i] = vw[i];
      w[12] = 0;
      uint16_t *dst = Vt + kk * A1_VPITCH + 128 * hh;
#pragma unroll
      for (int j = 0; j < 16; ++j) {
        const int bit = 24 * j, wi = bit >> 5, sh = bit & 31;
        const uint32_t u = __funnelshift_r(w[wi], w[wi + 1], sh) & 0xFFFFFFu;
        uint4 o;
        o.x = v3_pair128(u, 0);
        o.y = v3_pair128(u, 6);
        o.z = v3_pair128(u, 12);
        o.w = v3_pair128(u, 18);
        *reinterpret_cast<uint4 *>(dst + 8 * j) = o;
      }
    }
    __syncwarp();
    // ---- O^T += V^T P^T (V as 128 + c; 128 * sum(p) removed at the end) ----
    {
      const int q = lane >> 3, r = lane & 7;
      const int key = (q >> 1) * 8 + r, dq = (q & 1) * 8;
#pragma unroll
      for (int G = 0; G < 4; ++G) {
#pragma unroll
        for (int mt = 0; mt < 4; ++mt) {
          uint32_t a0, a1, a2, a3;
          ldsm_x4_trans(a0, a1, a2, a3, Vt + key * A1_VPITCH + 64 * G + 16 * mt + dq);
          mma_bf16(O[4 * G + mt], a0, a1, a2, a3, pB[G][0], pB[G][1]);
        }
      }
    }
    __syncwarp();
  }
  cp_async_wait<0>();

  // ---- reduce the lane partials of l and the V bias sums (over g) ----
#pragma unroll
  for (int h = 0; h < 2; ++h) {
#pragma unroll
    for (int o = 4; o < 32; o <<= 1) {
      l_run[h] += __shfl_xor_sync(0xffffffffu, l_run[h], o);
#pragma unroll
      for (int G = 0; G < 4; ++G) {
        bsum[G][h] += __shfl_xor_sync(0xffffffffu, bsum[G][h], o);
        psum[G][h] += __shfl_xor_sync(0xffffffffu, psum[G][h], o);
      }
    }
  }
  // ---- merge the 4 warps in shared memory: [warp][row 8][dim 256] + m, l ----
  __syncthreads();
  float *Om = reinterpret_cast<float *>(smem_raw);            // 4 x 8 x 256 floats (32 KB)
  float *Mm = Om + A1_WARPS * 8 * 256, *Lm = Mm + A1_WARPS * 8;
#pragma unroll
  for (int i = 0; i < 16; ++i) {
    const int G = i >> 2, mt = i & 3;
    const int d0 = 64 * G + 16 * mt + g;
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      const int row = 2 * c + h;
      const float off = fmaf(-128.f, psum[G][h], bsum[G][h]);
      Om[(warp * 8 + row) * 256 + d0] = O[i][h] + off;
      Om[(warp * 8 + row) * 256 + d0 + 8] = O[i][2 + h] + off;
    }
  }
  if (g == 0) {
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      Mm[warp * 8 + 2 * c + h] = m_run[h];
      Lm[warp * 8 + 2 * c + h] = l_run[h];
    }
  }
  __syncthreads();
  const size_t cta = (size_t)bh * p.nsplit + split;
  for (int i = threadIdx.x; i < 8 * 256; i += blockDim.x) {
    const int row = i >> 8, d = i & 255;
    if (row >= p.QR) continue;
    float M = -INFINITY;
#pragma unroll
    for (int w = 0; w < A1_WARPS; ++w) M = fmaxf(M, Mm[w * 8 + row]);
    float num = 0.f, den = 0.f;
#pragma unroll
    for (int w = 0; w < A1_WARPS; ++w) {
      const float mw = Mm[w * 8 + row];
      if (mw == -INFINITY) continue;
      const float sw = expf(mw - M);
      num = fmaf(Om[(w * 8 + row) * 256 + d], sw, num);
      den = fmaf(Lm[w * 8 + row], sw, den);
    }
    p.opart[(cta * 32 + row) * 256 + d] = num;
    if (d == 0) {
      p.mpart[cta * 32 + row] = M;
      p.lpart[cta * 32 + row] = den;
    }
  }
}

// ----------------------------------------------------------------------------
// Multi-position path (8 < rep * L <= 32 query rows per kv head: the MTP
// verify block, T = 4): the CTA walks 16-key tiles together. Its 128 threads
// unpack the tile's codes once into shared memory as exact bf16 128 + code
// (K in the (0,4,1,5,2,6,3,7) order of one LOP3 per pair inside every 8
// dims, V in dim order), and warp w takes query rows [8w, 8w + 8): scores
// S^T = K Q^T with K as the A operand (ldmatrix) and the 8 rows as N,
// per 64-dim group s*D + (b-128s)*sum(q); online softmax; O^T += V^T P^T
// with V^T by ldmatrix.trans. The rows of different warps are disjoint, so
// every warp writes its own rows of the split partial.
// ----------------------------------------------------------------------------
constexpr int A4_WARPS = 4;
constexpr int A4_PITCH = 256 + 8;                          // bf16 per unpacked row
constexpr int A4_TILE = 16 * A4_PITCH;                     // bf16 per unpacked 16-key tile
constexpr int A4_RAW = 16 * 128 + 16 * 96 + 4 * 16 * 8;    // K codes, V codes, 4 scale tensors
constexpr int A4_NRAW = 3;                                // staged tiles (two ahead)
constexpr int A4_SMEM = A4_NRAW * A4_RAW + 2 * 2 * A4_TILE * 2;  // raw, (K, V) unpacked x2

__device__ __forceinline__ void ldsm_x4(uint32_t &r0, uint32_t &r1, uint32_t &r2, uint32_t &r3,
                                        const void *smem_ptr) {
  const uint32_t a = (uint32_t)__cvta_generic_to_shared(smem_ptr);
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3) : "r"(a));
}

// Raw tile (16 keys from key0; keys past S-1 read key S-1 and are masked
// later) -> staging: K codes [16][128 B] (16-byte chunk j of key k at chunk
// j ^ (k % 8), so that eight keys' same chunk sit on distinct banks), V
// codes [16][96 B], then K scale, K bias, V scale, V bias [4][16][8 B]; 288
// copies over 128 threads.
__device__ __forceinline__ void a4_fetch(const uint8_t *kbase, const uint8_t *vbase,
                                         const uint8_t *const *sc, int S, int key0, uint8_t *raw,
                                         int tid) {
#pragma unroll
  for (int i = 0; i < 3; ++i) {
    const int q = tid + 128 * i;
    if (q < 128) {
      const int kr = q >> 3, j = q & 7, key = min(key0 + kr, S - 1);
      cp_async16(raw + kr * 128 + ((j ^ (kr & 7)) << 4), kbase + (size_t)key * 128 + j * 16);
    } else if (q < 224) {
      const int qq = q - 128, key = min(key0 + qq / 6, S - 1);
      cp_async16(raw + 2048 + qq * 16, vbase + (size_t)key * 96 + (qq % 6) * 16);
    } else if (q < 288) {
      const int qq = q - 224, t = qq >> 4, key = min(key0 + (qq & 15), S - 1);
      cp_async8(raw + 3584 + qq * 8, sc[t] + (size_t)key * 8);
    }
  }
}

template <bool DEV_POS>
__global__ void __launch_bounds__(A4_WARPS * 32, 3) kv_attn4_kernel(AttnParams p) {
  extern __shared__ __align__(16) uint8_t smem_raw[];
  if (DEV_POS) {  // launched as a programmatic dependent by the *_at entries
    pdl_launch_dependents();
    pdl_wait();
  }
  const int S_ = DEV_POS ? min(max(*p.pos_dev + p.pos_add, 0) + p.L, p.cap) : p.S;
  const int bh = blockIdx.x, split = blockIdx.y;
  const int b = bh / p.Hkv, hkv = bh % p.Hkv;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int g = lane >> 2, c = lane & 3;
  const int k_begin = split * p.kps;
  const int k_end = min(S_, k_begin + p.kps);
  uint8_t *raw0 = smem_raw;
  uint16_t *tiles = reinterpret_cast<uint16_t *>(smem_raw + A4_NRAW * A4_RAW);  // [2][K, V][16][PITCH]

  // Q^T B fragments of row 8w + g in the stored K order (k-step kk holds
  // dims 16kk + c, +4 and 16kk + 8 + c, +4 for lane c) and the per-group q
  // sums of rows 2c, 2c+1 of this warp.
  uint32_t qb[16][2];
  float qs[4][2];
  {
    const int r = 8 * warp + g;
    float part[4] = {0.f, 0.f, 0.f, 0.f};
    const uint16_t *qp = nullptr;
    if (r < p.QR) {
      const int rep_i = r / p.L, l = r % p.L;
      qp = p.q + (((size_t)b * p.Hq + hkv * p.rep + rep_i) * p.L + l) * 256;
    }
#pragma unroll
    for (int kk = 0; kk < 16; ++kk) {
      float v[4] = {0.f, 0.f, 0.f, 0.f};
      if (qp) {
#pragma unroll
        for (int j = 0; j < 4; ++j) v[j] = rbf(__fmul_rn(bf2f(qp[16 * kk + c + 4 * j]), p.scale));
      }
      qb[kk][0] = pack_bf2(v[0], v[1]);
      qb[kk][1] = pack_bf2(v[2], v[3]);
      part[kk >> 2] += (v[0] + v[1]) + (v[2] + v[3]);
    }
#pragma unroll
    for (int G = 0; G < 4; ++G) {
      float t = part[G];
      t += __shfl_xor_sync(0xffffffffu, t, 1);
      t += __shfl_xor_sync(0xffffffffu, t, 2);
      qs[G][0] = __shfl_sync(0xffffffffu, t, (2 * c) * 4);
      qs[G][1] = __shfl_sync(0xffffffffu, t, (2 * c + 1) * 4);
    }
  }

  float O[16][4];
#pragma unroll
  for (int i = 0; i < 16; ++i) O[i][0] = O[i][1] = O[i][2] = O[i][3] = 0.f;
  float m_run[2] = {-INFINITY, -INFINITY}, l_run[2] = {0.f, 0.f};
  float bsum[4][2], psum[4][2];
#pragma unroll
  for (int G = 0; G < 4; ++G) bsum[G][0] = bsum[G][1] = psum[G][0] = psum[G][1] = 0.f;

  const size_t head_row0 = (size_t)bh * p.cap;
  const int n_tiles = (k_end - k_begin + 15) / 16;
  const uint8_t *kbase = reinterpret_cast<const uint8_t *>(p.kc + head_row0 * 32);
  const uint8_t *vbase = reinterpret_cast<const uint8_t *>(p.vc + head_row0 * 24);
  const uint8_t *scb[4] = {reinterpret_cast<const uint8_t *>(p.ks + head_row0 * 4),
                           reinterpret_cast<const uint8_t *>(p.kb + head_row0 * 4),
                           reinterpret_cast<const uint8_t *>(p.vs + head_row0 * 4),
                           reinterpret_cast<const uint8_t *>(p.vb + head_row0 * 4)};
  const int row0 = 8 * warp + 2 * c;  // rows of this lane's score / output columns
  // Last key each of rows row0, row0+1 may see: -1 past the query rows,
  // S - L + position under the causal mask.
  int klim[2];
#pragma unroll
  for (int h = 0; h < 2; ++h) {
    const int row = row0 + h;
    klim[h] = row >= p.QR ? -1 : (p.causal ? S_ - p.L + row % p.L : INT_MAX);
  }
#pragma unroll 1
  for (int t = 0; t < A4_NRAW - 1; ++t) {
    if (t < n_tiles) a4_fetch(kbase, vbase, scb, S_, k_begin + 16 * t, raw0 + t * A4_RAW, tid);
    cp_async_commit();
  }
#pragma unroll 1
  for (int t = 0; t < n_tiles; ++t) {
    const int tn = t + A4_NRAW - 1;
    if (tn < n_tiles) a4_fetch(kbase, vbase, scb, S_, k_begin + 16 * tn, raw0 + (tn % A4_NRAW) * A4_RAW, tid);
    cp_async_commit();
    cp_async_wait<A4_NRAW - 1>();
    __syncthreads();  // tile t staged by every thread
    const uint8_t *rw = raw0 + (t % A4_NRAW) * A4_RAW;
    uint16_t *Kt = tiles + (t & 1) * 2 * A4_TILE, *Vt = Kt + A4_TILE;
    const int key0 = k_begin + 16 * t;
    {
      // K: thread -> key tid % 16, 32 codes (16 bytes) from byte 16 (tid / 16):
      // the eight lanes of a store phase hold eight different keys.
      const int key = tid & 15, part = tid >> 4;
      const uint4 w = *reinterpret_cast<const uint4 *>(rw + key * 128 + ((part ^ (key & 7)) << 4));
      const uint32_t ws[4] = {w.x, w.y, w.z, w.w};
      uint4 *dk = reinterpret_cast<uint4 *>(Kt + key * A4_PITCH + part * 32);
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        uint32_t pr[4];
        nib_pairs4(ws[j], pr);
        dk[j] = make_uint4(pr[0], pr[1], pr[2], pr[3]);
      }
      // V: thread -> key tid % 16, codes 32 (tid / 16) .. +32 (12 bytes)
      const uint32_t *vw = reinterpret_cast<const uint32_t *>(rw + 2048 + key * 96 + part * 12);
      const uint32_t v0 = vw[0], v1 = vw[1], v2 = vw[2];
      uint4 *dv = reinterpret_cast<uint4 *>(Vt + key * A4_PITCH + part * 32);
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const uint32_t u = j == 0 ? (v0 & 0xFFFFFFu)
                         : j == 1 ? (__funnelshift_r(v0, v1, 24) & 0xFFFFFFu)
                         : j == 2 ? (__funnelshift_r(v1, v2, 16) & 0xFFFFFFu)
                                  : (v2 >> 8);
        dv[j] = make_uint4(v3_pair128(u, 0), v3_pair128(u, 6), v3_pair128(u, 12), v3_pair128(u, 18));
      }
    }
    // Scales of keys g, g+8 (read before the barrier: the staging buffer is
    // refilled once every thread has passed it).
    const uint8_t *Sk = rw + 3584;
    const uint2 ksg = lds_u2(Sk + g * 8), ks8 = lds_u2(Sk + (g + 8) * 8);
    const uint2 kbg = lds_u2(Sk + 128 + g * 8), kb8 = lds_u2(Sk + 128 + (g + 8) * 8);
    const uint2 vsg = lds_u2(Sk + 256 + g * 8), vs8 = lds_u2(Sk + 256 + (g + 8) * 8);
    const uint2 vbg = lds_u2(Sk + 384 + g * 8), vb8 = lds_u2(Sk + 384 + (g + 8) * 8);
    __syncthreads();  // unpacked tile complete

    // ---- scores S^T for keys g, g+8 and rows row0, row0+1 ----
    float sc[4] = {0.f, 0.f, 0.f, 0.f};
    const uint16_t *ka = Kt + (lane & 15) * A4_PITCH + (lane >> 4) * 8;
#pragma unroll
    for (int G = 0; G < 4; ++G) {
      float d[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
      for (int k4 = 0; k4 < 4; ++k4) {
        const int kk = 4 * G + k4;
        uint32_t a0, a1, a2, a3;
        ldsm_x4(a0, a1, a2, a3, ka + 16 * kk);
        mma_bf16(d, a0, a1, a2, a3, qb[kk][0], qb[kk][1]);
      }
      const float s_g = bf_at2(ksg, G), s_8 = bf_at2(ks8, G);
      const float bp_g = fmaf(-128.f, s_g, bf_at2(kbg, G));
      const float bp_8 = fmaf(-128.f, s_8, bf_at2(kb8, G));
      sc[0] += fmaf(s_g, d[0], bp_g * qs[G][0]);
      sc[1] += fmaf(s_g, d[1], bp_g * qs[G][1]);
      sc[2] += fmaf(s_8, d[2], bp_8 * qs[G][0]);
      sc[3] += fmaf(s_8, d[3], bp_8 * qs[G][1]);
    }
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const int key = key0 + g + 8 * (j >> 1);
      const bool ok = key < k_end && key <= klim[j & 1];
      sc[j] = ok ? rbf(sc[j]) : -INFINITY;
    }
    // ---- online softmax (rows row0, row0+1) ----
    float mx[2] = {fmaxf(sc[0], sc[2]), fmaxf(sc[1], sc[3])};
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      mx[h] = fmaxf(mx[h], __shfl_xor_sync(0xffffffffu, mx[h], 4));
      mx[h] = fmaxf(mx[h], __shfl_xor_sync(0xffffffffu, mx[h], 8));
      mx[h] = fmaxf(mx[h], __shfl_xor_sync(0xffffffffu, mx[h], 16));
    }
    float mnew[2], alpha[2];
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      mnew[h] = fmaxf(m_run[h], mx[h]);
      alpha[h] = (m_run[h] == -INFINITY) ? 0.f : __expf(m_run[h] - mnew[h]);
      if (mnew[h] == -INFINITY) alpha[h] = 1.f;
      m_run[h] = mnew[h];
    }
    if (__any_sync(0xffffffffu, alpha[0] != 1.f || alpha[1] != 1.f)) {
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        l_run[h] *= alpha[h];
#pragma unroll
        for (int G = 0; G < 4; ++G) {
          bsum[G][h] *= alpha[h];
          psum[G][h] *= alpha[h];
        }
      }
#pragma unroll
      for (int i = 0; i < 16; ++i) {
        O[i][0] *= alpha[0];
        O[i][1] *= alpha[1];
        O[i][2] *= alpha[0];
        O[i][3] *= alpha[1];
      }
    }
    float e[4];
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const int h = j & 1;
      e[j] = sc[j] == -INFINITY ? 0.f : __expf(sc[j] - mnew[h]);
      l_run[h] += e[j];
    }
    // P^T fragments per V group: p = bf16(e * vs); V bias term on the side.
    uint32_t pB[4][2];
#pragma unroll
    for (int G = 0; G < 4; ++G) {
      const float sg = bf_at2(vsg, G), s8 = bf_at2(vs8, G);
      const float bg = bf_at2(vbg, G), b8 = bf_at2(vb8, G);
      bsum[G][0] = fmaf(e[0], bg, fmaf(e[2], b8, bsum[G][0]));
      bsum[G][1] = fmaf(e[1], bg, fmaf(e[3], b8, bsum[G][1]));
      const uint32_t x0 = pack_bf2(e[0] * sg, e[1] * sg);  // key g: rows row0, row0+1
      const uint32_t x1 = pack_bf2(e[2] * s8, e[3] * s8);  // key g+8
      psum[G][0] += __uint_as_float(x0 << 16) + __uint_as_float(x1 << 16);
      psum[G][1] += __uint_as_float(x0 & 0xFFFF0000u) + __uint_as_float(x1 & 0xFFFF0000u);
      pB[G][0] = movmatrix_trans(x0);
      pB[G][1] = movmatrix_trans(x1);
    }
    // ---- O^T += V^T P^T (V as 128 + c; 128 * sum(p) removed at the end) ----
    {
      const int q = lane >> 3, r = lane & 7;
      const int key = (q >> 1) * 8 + r, dq = (q & 1) * 8;
#pragma unroll
      for (int G = 0; G < 4; ++G) {
#pragma unroll
        for (int mt = 0; mt < 4; ++mt) {
          uint32_t a0, a1, a2, a3;
          ldsm_x4_trans(a0, a1, a2, a3, Vt + key * A4_PITCH + 64 * G + 16 * mt + dq);
          mma_bf16(O[4 * G + mt], a0, a1, a2, a3, pB[G][0], pB[G][1]);
        }
      }
    }
  }
  cp_async_wait<0>();

  // ---- reduce the lane partials of l and the V bias sums (over g) ----
#pragma unroll
  for (int h = 0; h < 2; ++h) {
#pragma unroll
    for (int o = 4; o < 32; o <<= 1) {
      l_run[h] += __shfl_xor_sync(0xffffffffu, l_run[h], o);
#pragma unroll
      for (int G = 0; G < 4; ++G) {
        bsum[G][h] += __shfl_xor_sync(0xffffffffu, bsum[G][h], o);
        psum[G][h] += __shfl_xor_sync(0xffffffffu, psum[G][h], o);
      }
    }
  }
  // ---- this warp's rows of the split partial ----
  const size_t cta = (size_t)bh * p.nsplit + split;
#pragma unroll
  for (int h = 0; h < 2; ++h) {
    const int row = row0 + h;
    if (row >= p.QR) continue;
    float *op = p.opart + (cta * 32 + row) * 256;
#pragma unroll
    for (int i = 0; i < 16; ++i) {
      const int G = i >> 2, mt = i & 3;
      const int d0 = 64 * G + 16 * mt + g;
      const float off = fmaf(-128.f, psum[G][h], bsum[G][h]);
      op[d0] = O[i][h] + off;
      op[d0 + 8] = O[i][2 + h] + off;
    }
    if (g == 0) {
      p.mpart[cta * 32 + row] = m_run[h];
      p.lpart[cta * 32 + row] = l_run[h];
    }
  }
}

// ----------------------------------------------------------------------------
// Plain bf16 cache (the MTP layer's mlx-lm KVCache, attended with
// mx.fast.scaled_dot_product_attention): q * scale, scores, softmax and P V in
// float32, one rounding of the output (in the combine). CUDA-core split-K
// kernel: a CTA walks its key range in 32-key chunks staged in shared memory;
// thread t scores key t % 32 against rows t / 32 + 8 i (conflict-free with
// the 258-element K pitch) and accumulates 4 output dims of 8 rows. The
// partials use the quantized kernels' layout, so the same combine merges them.
// ----------------------------------------------------------------------------
constexpr int B16_KP = 258;  // bf16 per staged K row
constexpr int B16_SMEM = 32 * 256 * 4 + 32 * B16_KP * 2 + 32 * 256 * 2 + 32 * 33 * 4 + 3 * 32 * 4;

template <bool DEV_POS>
__global__ void __launch_bounds__(256) kv_bf16_attn_kernel(AttnParams p) {
  extern __shared__ __align__(16) uint8_t smem_raw[];
  if (DEV_POS) {  // launched as a programmatic dependent by the *_at entries
    pdl_launch_dependents();
    pdl_wait();
  }
  const int S_ = DEV_POS ? min(max(*p.pos_dev + p.pos_add, 0) + p.L, p.cap) : p.S;
  float *qs = reinterpret_cast<float *>(smem_raw);                    // [32][256]
  uint16_t *ks = reinterpret_cast<uint16_t *>(qs + 32 * 256);         // [32][B16_KP]
  uint16_t *vs = ks + 32 * B16_KP;                                    // [32][256]
  float *sc = reinterpret_cast<float *>(vs + 32 * 256);               // [32][33]
  float *m_s = sc + 32 * 33, *l_s = m_s + 32, *f_s = l_s + 32;
  const int bh = blockIdx.x, split = blockIdx.y;
  const int b = bh / p.Hkv, hkv = bh % p.Hkv;
  const int tid = threadIdx.x;
  const int k_begin = split * p.kps;
  const int k_end = min(S_, k_begin + p.kps);
  const uint16_t *kc = reinterpret_cast<const uint16_t *>(p.kc) + (size_t)bh * p.cap * 256;
  const uint16_t *vc = reinterpret_cast<const uint16_t *>(p.vc) + (size_t)bh * p.cap * 256;
  for (int i = tid; i < 32 * 256; i += 256) {
    const int r = i >> 8, d = i & 255;
    float v = 0.f;
    if (r < p.QR) {
      const int hq = hkv * p.rep + r / p.L, l = r % p.L;
      v = bf2f(p.q[(((size_t)b * p.Hq + hq) * p.L + l) * 256 + d]) * p.scale;
    }
    qs[i] = v;
  }
  if (tid < 32) { m_s[tid] = -INFINITY; l_s[tid] = 0.f; }
  const int dq = (tid & 63) * 4, r0 = (tid >> 6) * 8;  // output dims, rows
  float O[8][4];
#pragma unroll
  for (int i = 0; i < 8; ++i) O[i][0] = O[i][1] = O[i][2] = O[i][3] = 0.f;
  for (int key0 = k_begin; key0 < k_end; key0 += 32) {
    const int nk = min(32, k_end - key0);
    __syncthreads();
    for (int i = tid; i < 32 * 128; i += 256) {  // 2 bf16 per step
      const int kk = i >> 7, d2 = (i & 127) * 2;
      uint32_t kw = 0, vw = 0;
      if (kk < nk) {
        kw = *reinterpret_cast<const uint32_t *>(kc + (size_t)(key0 + kk) * 256 + d2);
        vw = *reinterpret_cast<const uint32_t *>(vc + (size_t)(key0 + kk) * 256 + d2);
      }
      *reinterpret_cast<uint32_t *>(ks + kk * B16_KP + d2) = kw;
      *reinterpret_cast<uint32_t *>(vs + kk * 256 + d2) = vw;
    }
    __syncthreads();
    {  // scores
      const int kk = tid & 31, rb = tid >> 5;
      float acc[4] = {0.f, 0.f, 0.f, 0.f};
      const uint16_t *kr = ks + kk * B16_KP;
      for (int d = 0; d < 256; d += 2) {
        const uint32_t kw = *reinterpret_cast<const uint32_t *>(kr + d);
        const float k0 = __uint_as_float(kw << 16), k1 = __uint_as_float(kw & 0xFFFF0000u);
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          const float2 qv = *reinterpret_cast<const float2 *>(qs + (rb + 8 * i) * 256 + d);
          acc[i] = fmaf(qv.x, k0, acc[i]);
          acc[i] = fmaf(qv.y, k1, acc[i]);
        }
      }
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const int r = rb + 8 * i;
        const int key = key0 + kk;
        bool ok = kk < nk && r < p.QR;
        if (ok && p.causal) ok = key <= S_ - p.L + r % p.L;
        sc[r * 33 + kk] = ok ? acc[i] : -INFINITY;
      }
    }
    __syncthreads();
    if (tid < 32) {  // online softmax state of row tid
      const int r = tid;
      float mx = m_s[r];
      for (int kk = 0; kk < 32; ++kk) mx = fmaxf(mx, sc[r * 33 + kk]);
      const float mo = m_s[r];
      const float f = (mx == -INFINITY) ? 1.f : expf(mo - mx);
      float lsum = l_s[r] * (mo == -INFINITY ? 0.f : f);
      for (int kk = 0; kk < 32; ++kk) {
        const float sv = sc[r * 33 + kk];
        const float e = sv == -INFINITY ? 0.f : expf(sv - mx);
        sc[r * 33 + kk] = e;
        lsum += e;
      }
      m_s[r] = mx;
      l_s[r] = lsum;
      f_s[r] = (mo == -INFINITY) ? 0.f : f;
    }
    __syncthreads();
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const float f = f_s[r0 + i];
#pragma unroll
      for (int j = 0; j < 4; ++j) O[i][j] *= f;
    }
    for (int kk = 0; kk < 32; ++kk) {
      const uint2 vw = *reinterpret_cast<const uint2 *>(vs + kk * 256 + dq);
      const float v0 = __uint_as_float(vw.x << 16), v1 = __uint_as_float(vw.x & 0xFFFF0000u);
      const float v2 = __uint_as_float(vw.y << 16), v3 = __uint_as_float(vw.y & 0xFFFF0000u);
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        const float pv = sc[(r0 + i) * 33 + kk];
        O[i][0] = fmaf(pv, v0, O[i][0]);
        O[i][1] = fmaf(pv, v1, O[i][1]);
        O[i][2] = fmaf(pv, v2, O[i][2]);
        O[i][3] = fmaf(pv, v3, O[i][3]);
      }
    }
  }
  __syncthreads();
  const size_t cta = (size_t)bh * p.nsplit + split;
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    const int r = r0 + i;
    if (r >= p.QR) continue;
    *reinterpret_cast<float4 *>(p.opart + (cta * 32 + r) * 256 + dq) =
        make_float4(O[i][0], O[i][1], O[i][2], O[i][3]);
  }
  if (tid < p.QR) {
    p.mpart[cta * 32 + tid] = m_s[tid];
    p.lpart[cta * 32 + tid] = l_s[tid];
  }
}

// Keys per split: about three CTAs per SM over all (batch, kv head) pairs,
// in multiples of 64 keys.
static void attn_split(int bhk, int S, int &nsplit, int &kps) {
  int target = (3 * 148 + bhk - 1) / bhk;
  if (target < 1) target = 1;
  kps = (S + target - 1) / target;
  kps = (kps + ATT_ROUND - 1) / ATT_ROUND * ATT_ROUND;
  nsplit = (S + kps - 1) / kps;
}

}  // namespace vb

using namespace vb;

extern "C" {

size_t vb_kv_attn_workspace_size(int32_t batch, int32_t q_heads, int32_t L,
                                 int32_t dim, int32_t keys) {
  (void)q_heads; (void)L; (void)dim;
  if (batch <= 0 || keys <= 0) return 0;
  // Upper bound for kv_heads <= 64: at most 3 x 148 split CTAs overall plus
  // one per (batch, kv head) (the split rounds keys up to 64-key multiples).
  const size_t ctas = 3 * 148 + (size_t)batch * 64;
  return align_up(ctas * 32 * 256 * sizeof(float), 256) + 2 * align_up(ctas * 32 * sizeof(float), 256);
}

static int kv_decode_attn_impl(const uint16_t *q, const uint32_t *k_codes,
                               const uint16_t *k_scales, const uint16_t *k_biases,
                               const uint32_t *v_codes, const uint16_t *v_scales,
                               const uint16_t *v_biases, const float *rv_blocks,
                               int32_t batch, int32_t q_heads, int32_t kv_heads,
                               int32_t L, int32_t dim, int32_t keys, int32_t cap,
                               int32_t group, int32_t k_bits, int32_t v_bits,
                               float scale, int32_t causal, const int32_t *pos_dev,
                               const uint16_t *gate, int32_t gate_stride,
                               uint16_t *out, void *workspace, size_t workspace_bytes,
                               vb_stream_t stream) {
  VB_REQUIRE(dim == 256 && group == 64 && k_bits == 4 && v_bits == 3,
             "vb_kv_decode_attn: supports D=256, group 64, K4/V3 (got D=%d g=%d k%d v%d)",
             dim, group, k_bits, v_bits);
  VB_REQUIRE(batch > 0 && kv_heads > 0 && q_heads % kv_heads == 0,
             "vb_kv_decode_attn: heads %d/%d", q_heads, kv_heads);
  const int rep = q_heads / kv_heads;
  VB_REQUIRE(L >= 1 && L <= 4 && rep * L <= 32, "vb_kv_decode_attn: L=%d rep=%d", L, rep);
  VB_REQUIRE(keys >= L && keys <= cap, "vb_kv_decode_attn: keys=%d cap=%d L=%d", keys, cap, L);
  VB_REQUIRE(q && k_codes && k_scales && k_biases && v_codes && v_scales && v_biases && out,
             "vb_kv_decode_attn: null pointer");
  VB_REQUIRE(!gate || (batch == 1 && gate_stride >= q_heads * 512),
             "vb_kv_decode_attn: gate with batch %d, stride %d", batch, gate_stride);
  AttnParams p = {};
  p.q = q; p.kc = k_codes; p.vc = v_codes; p.ks = k_scales; p.kb = k_biases;
  p.vs = v_scales; p.vb = v_biases; p.rv = rv_blocks; p.pos_dev = pos_dev;
  p.gate = gate; p.gate_stride = gate_stride;
  p.B = batch; p.Hq = q_heads; p.Hkv = kv_heads; p.L = L; p.S = keys; p.cap = cap;
  p.rep = rep; p.QR = rep * L; p.causal = causal; p.scale = scale;
  attn_split(batch * kv_heads, keys, p.nsplit, p.kps);
  VB_REQUIRE(p.nsplit <= ATT_MAX_SPLITS, "vb_kv_decode_attn: %d splits", p.nsplit);
  const size_t ctas = (size_t)batch * kv_heads * p.nsplit;
  const size_t obytes = align_up(ctas * 32 * 256 * sizeof(float), 256);
  const size_t mbytes = align_up(ctas * 32 * sizeof(float), 256);
  VB_REQUIRE(workspace && workspace_bytes >= obytes + 2 * mbytes,
             "vb_kv_decode_attn: workspace %zu < %zu", workspace_bytes, obytes + 2 * mbytes);
  uint8_t *ws = static_cast<uint8_t *>(workspace);
  p.opart = reinterpret_cast<float *>(ws);
  p.mpart = reinterpret_cast<float *>(ws + obytes);
  p.lpart = reinterpret_cast<float *>(ws + obytes + mbytes);
  p.out = out;
  cudaStream_t s = as_stream(stream);
  const dim3 grid(batch * kv_heads, p.nsplit);
  static bool attr_done = false;
  if (!attr_done) {
    cudaFuncSetAttribute(kv_attn1_kernel<false>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                         A1_SMEM);
    cudaFuncSetAttribute(kv_attn1_kernel<true>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                         A1_SMEM);
    cudaFuncSetAttribute(kv_attn4_kernel<false>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                         A4_SMEM);
    cudaFuncSetAttribute(kv_attn4_kernel<true>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                         A4_SMEM);
    attr_done = true;
  }
  if (p.QR <= 8) {
    if (pos_dev)
      vb_launch(kv_attn1_kernel<true>, grid, dim3(A1_WARPS * 32), A1_SMEM, s, false, p);
    else
      kv_attn1_kernel<false><<<grid, A1_WARPS * 32, A1_SMEM, s>>>(p);
  } else {
    if (pos_dev)
      vb_launch(kv_attn4_kernel<true>, grid, dim3(A4_WARPS * 32), A4_SMEM, s, false, p);
    else
      kv_attn4_kernel<false><<<grid, A4_WARPS * 32, A4_SMEM, s>>>(p);
  }
  const int rc = check_launch(p.QR <= 8 ? "kv_attn1_kernel" : "kv_attn4_kernel");
  if (rc) return rc;
  if (pos_dev)
    vb_launch(kv_attn_combine_kernel, dim3(batch * q_heads * L, 8), dim3(256), 0, s, false, p);
  else
    kv_attn_combine_kernel<<<dim3(batch * q_heads * L, 8), 256, 0, s>>>(p);
  return check_launch("kv_attn_combine_kernel");
}

int vb_kv_decode_attn(const uint16_t *q, const uint32_t *k_codes,
                      const uint16_t *k_scales, const uint16_t *k_biases,
                      const uint32_t *v_codes, const uint16_t *v_scales,
                      const uint16_t *v_biases, const float *rv_blocks,
                      int32_t batch, int32_t q_heads, int32_t kv_heads,
                      int32_t L, int32_t dim, int32_t keys, int32_t cap,
                      int32_t group, int32_t k_bits, int32_t v_bits,
                      float scale, int32_t causal, uint16_t *out,
                      void *workspace, size_t workspace_bytes,
                      vb_stream_t stream) {
  return kv_decode_attn_impl(q, k_codes, k_scales, k_biases, v_codes, v_scales, v_biases,
                             rv_blocks, batch, q_heads, kv_heads, L, dim, keys, cap, group,
                             k_bits, v_bits, scale, causal, nullptr, nullptr, 0, out, workspace,
                             workspace_bytes, stream);
}

int vb_kv_bf16_attn_at(const uint16_t *q, const uint16_t *k_cache, const uint16_t *v_cache,
                       int32_t batch, int32_t q_heads, int32_t kv_heads, int32_t L,
                       int32_t dim, const int32_t *pos, int32_t pos_add, int32_t keys_max,
                       int32_t cap, float scale, int32_t causal, const uint16_t *gate_proj,
                       int32_t gate_stride, uint16_t *out, void *workspace,
                       size_t workspace_bytes, vb_stream_t stream) {
  VB_REQUIRE(dim == 256, "vb_kv_bf16_attn_at: D=%d (256 only)", dim);
  VB_REQUIRE(batch > 0 && kv_heads > 0 && q_heads % kv_heads == 0,
             "vb_kv_bf16_attn_at: heads %d/%d", q_heads, kv_heads);
  const int rep = q_heads / kv_heads;
  VB_REQUIRE(L >= 1 && rep * L <= 32, "vb_kv_bf16_attn_at: L=%d rep=%d", L, rep);
  VB_REQUIRE(keys_max >= L && keys_max <= cap, "vb_kv_bf16_attn_at: keys_max=%d cap=%d",
             keys_max, cap);
  VB_REQUIRE(q && k_cache && v_cache && out && pos, "vb_kv_bf16_attn_at: null pointer");
  VB_REQUIRE(!gate_proj || (batch == 1 && gate_stride >= q_heads * 512),
             "vb_kv_bf16_attn_at: gate with batch %d, stride %d", batch, gate_stride);
  AttnParams p = {};
  p.q = q; p.kc = reinterpret_cast<const uint32_t *>(k_cache);
  p.vc = reinterpret_cast<const uint32_t *>(v_cache);
  p.ks = p.kb = p.vs = p.vb = nullptr; p.rv = nullptr; p.pos_dev = pos; p.pos_add = pos_add;
  p.gate = gate_proj; p.gate_stride = gate_stride;
  p.B = batch; p.Hq = q_heads; p.Hkv = kv_heads; p.L = L; p.S = keys_max; p.cap = cap;
  p.rep = rep; p.QR = rep * L; p.causal = causal; p.scale = scale;
  attn_split(batch * kv_heads, keys_max, p.nsplit, p.kps);
  VB_REQUIRE(p.nsplit <= ATT_MAX_SPLITS, "vb_kv_bf16_attn_at: %d splits", p.nsplit);
  const size_t ctas = (size_t)batch * kv_heads * p.nsplit;
  const size_t obytes = align_up(ctas * 32 * 256 * sizeof(float), 256);
  const size_t mbytes = align_up(ctas * 32 * sizeof(float), 256);
  VB_REQUIRE(workspace && workspace_bytes >= obytes + 2 * mbytes + 256,
             "vb_kv_bf16_attn_at: workspace %zu < %zu", workspace_bytes,
             obytes + 2 * mbytes + 256);
  uint8_t *ws = static_cast<uint8_t *>(workspace);
  p.opart = reinterpret_cast<float *>(ws);
  p.mpart = reinterpret_cast<float *>(ws + obytes);
  p.lpart = reinterpret_cast<float *>(ws + obytes + mbytes);
  p.out = out;
  cudaStream_t s = as_stream(stream);
  static bool attr_done = false;
  if (!attr_done) {
    cudaFuncSetAttribute(kv_bf16_attn_kernel<true>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                         B16_SMEM);
    attr_done = true;
  }
  vb_launch(kv_bf16_attn_kernel<true>, dim3(batch * kv_heads, p.nsplit), dim3(256), B16_SMEM, s,
            true, p);
  const int rc = check_launch("kv_bf16_attn_kernel");
  if (rc) return rc;
  vb_launch(kv_attn_combine_kernel, dim3(batch * q_heads * L, 8), dim3(256), 0, s, false, p);
  return check_launch("kv_attn_combine_kernel");
}

int vb_kv_decode_attn_at(const uint16_t *q, const uint32_t *k_codes,
                         const uint16_t *k_scales, const uint16_t *k_biases,
                         const uint32_t *v_codes, const uint16_t *v_scales,
                         const uint16_t *v_biases, const float *rv_blocks,
                         int32_t batch, int32_t q_heads, int32_t kv_heads,
                         int32_t L, int32_t dim, const int32_t *pos, int32_t keys_max,
                         int32_t cap, int32_t group, int32_t k_bits, int32_t v_bits,
                         float scale, int32_t causal, const uint16_t *gate_proj,
                         int32_t gate_stride, uint16_t *out, void *workspace,
                         size_t workspace_bytes, vb_stream_t stream) {
  VB_REQUIRE(pos != nullptr, "vb_kv_decode_attn_at: null position");
  return kv_decode_attn_impl(q, k_codes, k_scales, k_biases, v_codes, v_scales, v_biases,
                             rv_blocks, batch, q_heads, kv_heads, L, dim, keys_max, cap, group,
                             k_bits, v_bits, scale, causal, pos, gate_proj, gate_stride, out,
                             workspace, workspace_bytes, stream);
}

}  // extern "C"
