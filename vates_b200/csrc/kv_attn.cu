// Quantized GQA decode attention directly over the packed IsoQuant cache.
//
// Reference: asym_quantized_sdpa (mlx_streaming/core/cache/quant_kv.py:
// 212-249): q*scale (bf16) -> quantized_matmul(q, K^T) (bf16 scores) ->
// causal mask -> precise softmax -> quantized_matmul(p, V) -> bf16, then the
// inverse V rotation (kv_quant_patch.py:67-68).
//
// Split-K ("flash decoding"): each CTA owns one (batch, kv head) and a
// contiguous key range, processed in rounds of 64 keys; a combine kernel
// merges the per-split (max, sum, output) triples in split order.
// Inside a CTA, warp w owns head-dim group w (64 dims, one scale/bias group):
//  - QK^T: A = q (16 query rows x 16 dims, kept in registers), B = K codes
//    of 8 keys as exact bf16 (128+q) built with one LOP3 per pair; per key
//    the group score is s*D + (b-128*s)*sum(q). The four group partials are
//    exchanged through shared memory and added in group order, so every warp
//    sees identical scores (rounded to bf16 as MLX does).
//  - Online softmax in float32; P is multiplied by the key's V scale of the
//    warp's group and rounded to bf16 as the A operand of P.V; the V bias
//    term sum(p*b) is accumulated on the CUDA cores.
//  - V codes (3-bit) of the warp's 64 dims are unpacked to exact bf16 in
//    shared memory and read as B fragments with ldmatrix.trans.
#include "common.cuh"

namespace vb {

constexpr int ATT_WARPS = 4;
constexpr int ATT_ROUND = 64;
constexpr int ATT_SX_STRIDE = 68;   // floats per score row (64 + pad)
constexpr int ATT_VS_STRIDE = 72;   // bf16 per unpacked V row (64 + pad)

struct AttnParams {
  const uint16_t *q;
  const uint32_t *kc, *vc;
  const uint16_t *ks, *kb, *vs, *vb;
  const float *rv;
  int B, Hq, Hkv, L, S, cap, rep, QR, causal, nsplit, kps;
  float scale;
  float *opart, *mpart, *lpart;
  uint16_t *out;
};

__device__ __forceinline__ void ldsm_x4_trans(uint32_t &r0, uint32_t &r1, uint32_t &r2,
                                              uint32_t &r3, const void *smem_ptr) {
  const uint32_t a = (uint32_t)__cvta_generic_to_shared(smem_ptr);
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3) : "r"(a));
}

__device__ __forceinline__ uint32_t v3_pair(uint32_t u, int s0) {
  // codes at bit s0 and s0+3 of u -> exact bf16 pair (c0, c1)
  const uint32_t lo = u >> s0;
  const uint32_t hi = (s0 + 3 <= 16) ? (u << (16 - s0 - 3)) : (u >> (s0 + 3 - 16));
  uint32_t pr = ((lo & 0x7u) | (hi & 0x70000u)) | 0x43004300u;
  __nv_bfloat162 v = *reinterpret_cast<__nv_bfloat162 *>(&pr);
  const __nv_bfloat162 off = __floats2bfloat162_rn(128.f, 128.f);
  v = __hsub2(v, off);
  return *reinterpret_cast<uint32_t *>(&v);
}

template <int MT>
__global__ void __launch_bounds__(ATT_WARPS * 32, 2) kv_attn_partial_kernel(AttnParams p) {
  extern __shared__ __align__(16) uint8_t smem_raw[];
  float *Sx = reinterpret_cast<float *>(smem_raw);  // [2][4][16*MT][68]
  uint16_t *Vs = reinterpret_cast<uint16_t *>(Sx + 2 * ATT_WARPS * 16 * MT * ATT_SX_STRIDE);
  float2 *ksc = reinterpret_cast<float2 *>(Vs + ATT_WARPS * ATT_ROUND * ATT_VS_STRIDE);
  float2 *vsc = ksc + ATT_WARPS * ATT_ROUND;

  const int bh = blockIdx.x;  // b * Hkv + hkv
  const int split = blockIdx.y;
  const int b = bh / p.Hkv, hkv = bh % p.Hkv;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int g = lane >> 2, c = lane & 3;
  const int G = warp;
  const int k_begin = split * p.kps;
  const int k_end = min(p.S, k_begin + p.kps);

  // ---- q fragments (scaled, bf16) for this warp's dim group ----
  uint32_t aq[MT][4][4];
  float qsum[MT][2];
#pragma unroll
  for (int mt = 0; mt < MT; ++mt) {
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      const int r = 16 * mt + g + 8 * h;
      float vals[16];
      float part = 0.f;
      if (r < p.QR) {
        const int rep_i = r / p.L, l = r % p.L;
        const int hq = hkv * p.rep + rep_i;
        const uint16_t *qp = p.q + (((size_t)b * p.Hq + hq) * p.L + l) * 256 + 64 * G + 16 * c;
#pragma unroll
        for (int i = 0; i < 16; ++i) {
          vals[i] = rbf(__fmul_rn(bf2f(qp[i]), p.scale));
          part += vals[i];
        }
      } else {
#pragma unroll
        for (int i = 0; i < 16; ++i) vals[i] = 0.f;
      }
#pragma unroll
      for (int m = 0; m < 4; ++m) {
        const int j = m >> 1, i0 = 2 * (m & 1);
        const int d0 = 8 * j + i0;
        aq[mt][m][h] = pack_bf2(vals[d0], vals[d0 + 4]);
        aq[mt][m][2 + h] = pack_bf2(vals[d0 + 1], vals[d0 + 5]);
      }
      part += __shfl_xor_sync(0xffffffffu, part, 1);
      part += __shfl_xor_sync(0xffffffffu, part, 2);
      qsum[mt][h] = part;
    }
  }

  float O[MT][8][4];
  float m_run[MT][2], l_run[MT][2], bsum[MT][2];
#pragma unroll
  for (int mt = 0; mt < MT; ++mt) {
#pragma unroll
    for (int nd = 0; nd < 8; ++nd)
#pragma unroll
      for (int q = 0; q < 4; ++q) O[mt][nd][q] = 0.f;
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      m_run[mt][h] = -INFINITY;
      l_run[mt][h] = 0.f;
      bsum[mt][h] = 0.f;
    }
  }

  const size_t head_row0 = (size_t)bh * p.cap;
  uint16_t *Vw = Vs + warp * ATT_ROUND * ATT_VS_STRIDE;
  float2 *kscw = ksc + warp * ATT_ROUND;
  float2 *vscw = vsc + warp * ATT_ROUND;
  int buf = 0;

  for (int kb = k_begin; kb < k_end; kb += ATT_ROUND, buf ^= 1) {
    // ---- per-warp loads: scales, K words, V unpack ----
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      const int kl = 2 * lane + h;
      const int key = min(kb + kl, p.S - 1);
      const size_t sidx = (head_row0 + key) * 4 + G;
      const float ks_ = bf2f(__ldg(p.ks + sidx)), kb_ = bf2f(__ldg(p.kb + sidx));
      const float vs_ = bf2f(__ldg(p.vs + sidx)), vb_ = bf2f(__ldg(p.vb + sidx));
      kscw[kl] = make_float2(ks_, fmaf(-128.f, ks_, kb_));
      vscw[kl] = make_float2(vs_, vb_);
      const uint32_t *vrow = p.vc + (head_row0 + key) * 24 + 6 * G;
      uint32_t w[7];
      const uint2 v01 = *reinterpret_cast<const uint2 *>(vrow);
      const uint2 v23 = *reinterpret_cast<const uint2 *>(vrow + 2);
      const uint2 v45 = *reinterpret_cast<const uint2 *>(vrow + 4);
      w[0] = v01.x; w[1] = v01.y; w[2] = v23.x; w[3] = v23.y; w[4] = v45.x; w[5] = v45.y; w[6] = 0;
      uint16_t *dst = Vw + kl * ATT_VS_STRIDE;
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        const int bit = 24 * i, wi = bit >> 5, sh = bit & 31;
        const uint32_t u = __funnelshift_r(w[wi], w[wi + 1], sh) & 0xFFFFFFu;
        uint4 o;
        o.x = v3_pair(u, 0);
        o.y = v3_pair(u, 6);
        o.z = v3_pair(u, 12);
        o.w = v3_pair(u, 18);
        *reinterpret_cast<uint4 *>(dst + 8 * i) = o;
      }
    }
    uint2 kw[8];
#pragma unroll
    for (int nt = 0; nt < 8; ++nt) {
      const int key = min(kb + 8 * nt + g, p.S - 1);
      kw[nt] = ldg_nc_v2(reinterpret_cast<const uint8_t *>(p.kc + (head_row0 + key) * 32) + 32 * G + 8 * c);
    }
    __syncwarp();

    // ---- partial scores of this group ----
    float *Sxw = Sx + ((size_t)buf * ATT_WARPS + warp) * 16 * MT * ATT_SX_STRIDE;
#pragma unroll
    for (int nt = 0; nt < 8; ++nt) {
      const float2 ks0 = kscw[8 * nt + 2 * c], ks1 = kscw[8 * nt + 2 * c + 1];
#pragma unroll
      for (int mt = 0; mt < MT; ++mt) {
        float d[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
        for (int m = 0; m < 4; ++m) {
          const int i0 = 2 * (m & 1);
          const uint32_t wv = (m >> 1) ? kw[nt].y : kw[nt].x;
          mma_bf16(d, aq[mt][m][0], aq[mt][m][1], aq[mt][m][2], aq[mt][m][3],
                   nib_pair(wv, i0), nib_pair(wv, i0 + 1));
        }
        const float s00 = fmaf(ks0.x, d[0], ks0.y * qsum[mt][0]);
        const float s01 = fmaf(ks1.x, d[1], ks1.y * qsum[mt][0]);
        const float s10 = fmaf(ks0.x, d[2], ks0.y * qsum[mt][1]);
        const float s11 = fmaf(ks1.x, d[3], ks1.y * qsum[mt][1]);
        float *r0 = Sxw + (16 * mt + g) * ATT_SX_STRIDE + 8 * nt + 2 * c;
        float *r1 = r0 + 8 * ATT_SX_STRIDE;
        *reinterpret_cast<float2 *>(r0) = make_float2(s00, s01);
        *reinterpret_cast<float2 *>(r1) = make_float2(s10, s11);
      }
    }
    __syncthreads();

    // ---- full scores, online softmax, P fragments ----
    const float *Sxb = Sx + (size_t)buf * ATT_WARPS * 16 * MT * ATT_SX_STRIDE;
#pragma unroll
    for (int mt = 0; mt < MT; ++mt) {
      float sv[8][4];
      float mx[2] = {-INFINITY, -INFINITY};
#pragma unroll
      for (int nt = 0; nt < 8; ++nt) {
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          const int row = 16 * mt + g + 8 * (q >> 1);
          const int kl = 8 * nt + 2 * c + (q & 1);
          float s = 0.f;
#pragma unroll
          for (int w = 0; w < ATT_WARPS; ++w)
            s += Sxb[((size_t)w * 16 * MT + row) * ATT_SX_STRIDE + kl];
          s = rbf(s);
          const int key = kb + kl;
          bool ok = row < p.QR && key < k_end;
          if (p.causal && ok) ok = key <= p.S - p.L + (row % p.L);
          s = ok ? s : -INFINITY;
          sv[nt][q] = s;
          mx[q >> 1] = fmaxf(mx[q >> 1], s);
        }
      }
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        mx[h] = fmaxf(mx[h], __shfl_xor_sync(0xffffffffu, mx[h], 1));
        mx[h] = fmaxf(mx[h], __shfl_xor_sync(0xffffffffu, mx[h], 2));
      }
      float mnew[2], alpha[2];
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        mnew[h] = fmaxf(m_run[mt][h], mx[h]);
        alpha[h] = (m_run[mt][h] == -INFINITY) ? 0.f : expf(m_run[mt][h] - mnew[h]);
        if (mnew[h] == -INFINITY) alpha[h] = 1.f;
        m_run[mt][h] = mnew[h];
        l_run[mt][h] *= alpha[h];
        bsum[mt][h] *= alpha[h];
      }
#pragma unroll
      for (int nd = 0; nd < 8; ++nd) {
        O[mt][nd][0] *= alpha[0];
        O[mt][nd][1] *= alpha[0];
        O[mt][nd][2] *= alpha[1];
        O[mt][nd][3] *= alpha[1];
      }
      uint32_t ap[4][4];
#pragma unroll
      for (int nt = 0; nt < 8; ++nt) {
        float pr[4];
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          const int h = q >> 1;
          const float e = sv[nt][q] == -INFINITY ? 0.f : expf(sv[nt][q] - mnew[h]);
          const float2 vsb = vscw[8 * nt + 2 * c + (q & 1)];
          l_run[mt][h] += e;
          bsum[mt][h] = fmaf(e, vsb.y, bsum[mt][h]);
          pr[q] = e * vsb.x;
        }
        const int ks = nt >> 1, hi = nt & 1;
        ap[ks][2 * hi + 0] = pack_bf2(pr[0], pr[1]);
        ap[ks][2 * hi + 1] = pack_bf2(pr[2], pr[3]);
      }
      // ---- P.V over this warp's 64 dims ----
#pragma unroll
      for (int ks = 0; ks < 4; ++ks) {
        const int mi = lane >> 3, ri = lane & 7;
#pragma unroll
        for (int nd = 0; nd < 8; nd += 2) {
          const int key = 16 * ks + ri + 8 * (mi & 1);
          const int dim = 8 * (nd + (mi >> 1));
          uint32_t b0, b1, b2, b3;
          ldsm_x4_trans(b0, b1, b2, b3, Vw + key * ATT_VS_STRIDE + dim);
          mma_bf16(O[mt][nd], ap[ks][0], ap[ks][1], ap[ks][2], ap[ks][3], b0, b1);
          mma_bf16(O[mt][nd + 1], ap[ks][0], ap[ks][1], ap[ks][2], ap[ks][3], b2, b3);
        }
      }
    }
    __syncwarp();
  }

  // ---- write split partials ----
  const size_t cta = (size_t)bh * p.nsplit + split;
#pragma unroll
  for (int mt = 0; mt < MT; ++mt) {
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      float l = l_run[mt][h], bs = bsum[mt][h];
      l += __shfl_xor_sync(0xffffffffu, l, 1);
      l += __shfl_xor_sync(0xffffffffu, l, 2);
      bs += __shfl_xor_sync(0xffffffffu, bs, 1);
      bs += __shfl_xor_sync(0xffffffffu, bs, 2);
      const int row = 16 * mt + g + 8 * h;
      if (row < p.QR) {
        float *orow = p.opart + (cta * 32 + row) * 256 + 64 * G;
#pragma unroll
        for (int nd = 0; nd < 8; ++nd) {
          *reinterpret_cast<float2 *>(orow + 8 * nd + 2 * c) =
              make_float2(O[mt][nd][2 * h] + bs, O[mt][nd][2 * h + 1] + bs);
        }
        if (warp == 0 && c == 0) {
          p.mpart[cta * 32 + row] = m_run[mt][h];
          p.lpart[cta * 32 + row] = l;
        }
      }
    }
  }
}

// One CTA (256 threads = dims) per query row: merge splits, round to bf16,
// optional inverse V rotation (4x4 blocks of R_v^T, R rounded to bf16).
__global__ void __launch_bounds__(256) kv_attn_combine_kernel(AttnParams p) {
  const int row_id = blockIdx.x;  // ((b*Hq + hq)*L + l)
  const int l = row_id % p.L;
  const int bhq = row_id / p.L;
  const int b = bhq / p.Hq, hq = bhq % p.Hq;
  const int hkv = hq / p.rep, rep_i = hq % p.rep;
  const int r = rep_i * p.L + l;
  const size_t bh = (size_t)b * p.Hkv + hkv;
  const int d = threadIdx.x;
  float M = -INFINITY;
  for (int s = 0; s < p.nsplit; ++s) M = fmaxf(M, p.mpart[(bh * p.nsplit + s) * 32 + r]);
  float num = 0.f, den = 0.f;
  for (int s = 0; s < p.nsplit; ++s) {
    const size_t cta = bh * p.nsplit + s;
    const float ms = p.mpart[cta * 32 + r];
    if (ms == -INFINITY) continue;
    const float e = expf(ms - M);
    den = fmaf(p.lpart[cta * 32 + r], e, den);
    num = fmaf(p.opart[(cta * 32 + r) * 256 + d], e, num);
  }
  float o = rbf(den > 0.f ? num / den : 0.f);
  if (p.rv) {
    __shared__ float ov[256];
    ov[d] = o;
    __syncthreads();
    const int blk = d >> 2, i = d & 3;
    const float *R = p.rv + (size_t)blk * 16;
    float acc = 0.f;
#pragma unroll
    for (int kk = 0; kk < 4; ++kk)
      acc = __fadd_rn(acc, __fmul_rn(ov[4 * blk + kk], rbf(__ldg(R + i * 4 + kk))));
    o = rbf(acc);
  }
  p.out[(size_t)row_id * 256 + d] = f2bf(o);
}

static void attn_split(int bhk, int S, int &nsplit, int &kps) {
  int target = (2 * 148 + bhk - 1) / bhk;
  if (target < 1) target = 1;
  kps = (S + target - 1) / target;
  kps = (kps + ATT_ROUND - 1) / ATT_ROUND * ATT_ROUND;
  if (kps < ATT_ROUND) kps = ATT_ROUND;
  nsplit = (S + kps - 1) / kps;
}

}  // namespace vb

using namespace vb;

extern "C" {

size_t vb_kv_attn_workspace_size(int32_t batch, int32_t q_heads, int32_t L,
                                 int32_t dim, int32_t keys) {
  (void)q_heads; (void)L; (void)dim;
  if (batch <= 0 || keys <= 0) return 0;
  // Upper bound over kv_heads >= 1: splits <= 296 per (batch, kv head) and
  // at most 296 CTAs overall plus one per (batch, kv head).
  const size_t ctas = 2 * 148 + (size_t)batch * 64;
  return align_up(ctas * 32 * 256 * sizeof(float), 256) + 2 * align_up(ctas * 32 * sizeof(float), 256);
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
  AttnParams p;
  p.q = q; p.kc = k_codes; p.vc = v_codes; p.ks = k_scales; p.kb = k_biases;
  p.vs = v_scales; p.vb = v_biases; p.rv = rv_blocks;
  p.B = batch; p.Hq = q_heads; p.Hkv = kv_heads; p.L = L; p.S = keys; p.cap = cap;
  p.rep = rep; p.QR = rep * L; p.causal = causal; p.scale = scale;
  attn_split(batch * kv_heads, keys, p.nsplit, p.kps);
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
  const int MT = p.QR > 16 ? 2 : 1;
  const size_t smem = (size_t)2 * ATT_WARPS * 16 * MT * ATT_SX_STRIDE * sizeof(float) +
                      (size_t)ATT_WARPS * ATT_ROUND * ATT_VS_STRIDE * sizeof(uint16_t) +
                      (size_t)2 * ATT_WARPS * ATT_ROUND * sizeof(float2);
  dim3 grid(batch * kv_heads, p.nsplit);
  if (MT == 1) {
    cudaFuncSetAttribute(kv_attn_partial_kernel<1>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    kv_attn_partial_kernel<1><<<grid, ATT_WARPS * 32, smem, s>>>(p);
  } else {
    cudaFuncSetAttribute(kv_attn_partial_kernel<2>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    kv_attn_partial_kernel<2><<<grid, ATT_WARPS * 32, smem, s>>>(p);
  }
  int rc = check_launch("kv_attn_partial_kernel");
  if (rc) return rc;
  kv_attn_combine_kernel<<<batch * q_heads * L, 256, 0, s>>>(p);
  return check_launch("kv_attn_combine_kernel");
}

}  // extern "C"
