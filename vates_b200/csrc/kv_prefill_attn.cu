// Prefill attention over the packed IsoQuant K4/V3 cache on the 5th-generation
// tensor cores (tcgen05, accumulators in TMEM).
//
// Reference: _tiled_asymmetric_attention (mlx_streaming/core/attention/
// expert_major.py:32-95), called per query tile by the prefill branch of the
// rotated quantized attention (expert_major.py:107-182): q*scale (bf16) ->
// quantized_matmul(q, K^T) (bf16 scores) -> causal mask -> precise softmax
// -> quantized_matmul(p, V) -> bf16, then the inverse V rotation
// (kv_quant_patch.py:67-68). The reference materialises score tiles under a
// 16 M-score budget; here one CTA owns 128 query rows (128 / rep positions x
// the rep query heads of one kv head, so every dequantised key tile serves
// all of them) and streams the visible keys in 128-key tiles with an online
// softmax:
//   1. all 8 warps dequantise the K tile (s * code + b in fp32, rounded to
//      bf16) into a K-major 128-byte-swizzled operand; thread 0 issues
//      S = Q K^T (M=128, N=128, K=256) into TMEM;
//   2. meanwhile the V tile is dequantised into the same swizzled layout,
//      read by the tensor core as an MN-major operand (keys along K);
//   3. warps 0-3 (one query row per thread = TMEM lane) round the scores to
//      bf16, mask, update the running maximum (the reference value moves only
//      when the tile maximum exceeds it by 8 in log2 units; O and the sum are
//      then rescaled in place), write P = exp2(s - m) as bf16 into shared
//      memory and add the fp32 values to the row sum;
//   4. thread 0 issues O += P V (M=128, N=256, K=128) into TMEM.
// The epilogue divides by the row sum, rounds to bf16, applies the optional
// inverse V rotation (bf16 4x4 blocks) and writes the rows. Every mbarrier
// wait is bounded (2 s, then VB_STATUS_TIMEOUT); TMEM is freed only after
// the MMAs this CTA issued have completed.
#include "common.cuh"
#include "tc100.cuh"

namespace vb {
namespace {

constexpr int PA_THREADS = 256;
constexpr int PA_ROWS = 128;          // query rows per CTA
constexpr int PA_KT = 128;            // keys per tile
constexpr int PA_BLOCK = 16384;       // 128 rows x 64 bf16, 128-byte swizzle
constexpr int PA_Q = 0;               // 4 blocks: Q [row][dim]
constexpr int PA_K = 4 * PA_BLOCK;    // 4 blocks: K [key][dim]
constexpr int PA_V = 8 * PA_BLOCK;    // 4 blocks: V [key][dim]
constexpr int PA_P = 12 * PA_BLOCK;   // 2 blocks: P [row][key]
constexpr int PA_SMEM = 14 * PA_BLOCK + 1024;
constexpr uint64_t PA_WAIT_NS = 2000000000ull;
constexpr uint32_t PA_TS = 0, PA_TO = 128;  // TMEM columns of S and O
constexpr float PA_RESCALE = 8.f;           // log2 units

struct PrefillAttnParams {
  const uint16_t *q;
  const uint32_t *kc, *vc;
  const uint16_t *ks, *kb, *vs, *vb;
  const float *rv;
  int B, Hq, Hkv, Lq, keys, cap, rep, P, causal, n_row_tiles;
  float scale;
  uint16_t *out;
  int32_t *status;
};

// Byte offset of 16-byte chunk c of row r in a 128-row x 64-column block.
__device__ __forceinline__ uint32_t sw_off(int r, int c) {
  return (uint32_t)((r >> 3) * 1024 + (r & 7) * 128 + ((c ^ (r & 7)) << 4));
}

// MN-major descriptor, 128-byte swizzle: 64-element lines along N, 8-line
// groups along K `sbo` bytes apart, 64-element column blocks `lbo` bytes apart.
__device__ __forceinline__ uint64_t smem_desc_sw128_mn(uint32_t saddr, uint32_t lbo,
                                                       uint32_t sbo) {
  uint64_t d = 0;
  d |= (uint64_t)((saddr & 0x3FFFFu) >> 4);
  d |= (uint64_t)((lbo >> 4) & 0x3FFFu) << 16;
  d |= (uint64_t)((sbo >> 4) & 0x3FFFu) << 32;
  d |= (uint64_t)1 << 46;
  d |= (uint64_t)2 << 61;
  return d;
}

__device__ __forceinline__ void tmem_st32(uint32_t taddr, const uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,"
      "%13,%14,%15,%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31,%32};" ::"r"(
          taddr),
      "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]),
      "r"(r[8]), "r"(r[9]), "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]),
      "r"(r[15]), "r"(r[16]), "r"(r[17]), "r"(r[18]), "r"(r[19]), "r"(r[20]), "r"(r[21]),
      "r"(r[22]), "r"(r[23]), "r"(r[24]), "r"(r[25]), "r"(r[26]), "r"(r[27]), "r"(r[28]),
      "r"(r[29]), "r"(r[30]), "r"(r[31])
      : "memory");
}
__device__ __forceinline__ void tmem_st_wait() {
  asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
}

__device__ __forceinline__ uint32_t cvt_bf2(float lo, float hi) {
  uint32_t r;
  asm("cvt.rn.bf16x2.f32 %0, %1, %2;" : "=r"(r) : "f"(hi), "f"(lo));
  return r;
}
// bf16 pair (128 + c0, 128 + c1) -> s * c + b for both, packed to bf16x2
// (bb = b - 128 s).
__device__ __forceinline__ uint32_t deq_pair(uint32_t pr, float s, float bb) {
  const float lo = __uint_as_float(pr << 16), hi = __uint_as_float(pr & 0xFFFF0000u);
  return cvt_bf2(fmaf(s, lo, bb), fmaf(s, hi, bb));
}
__device__ __forceinline__ float ex2(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

// K tile: thread -> key tid / 2, dims [128 h, 128 h + 128) (h = tid % 2).
__device__ __forceinline__ void pa_dequant_k(const PrefillAttnParams &p, size_t bh, int k0,
                                             uint8_t *sk, int tid) {
  const int key = tid >> 1, h = tid & 1;
  const int kidx = min(k0 + key, p.keys - 1);  // keys past the end are masked later
  const size_t row = bh * p.cap + kidx;
  const uint4 *src = reinterpret_cast<const uint4 *>(p.kc + row * 32 + h * 16);
  uint4 w4[4];
#pragma unroll
  for (int i = 0; i < 4; ++i) w4[i] = ldg_nc_v4(src + i);
  const uint2 sv = *reinterpret_cast<const uint2 *>(p.ks + row * 4);
  const uint2 bv = *reinterpret_cast<const uint2 *>(p.kb + row * 4);
  float s[2], bb[2];
#pragma unroll
  for (int g = 0; g < 2; ++g) {
    const uint32_t sw = h ? sv.y : sv.x, bw = h ? bv.y : bv.x;
    s[g] = bf2f(g ? (sw >> 16) : (sw & 0xFFFFu));
    bb[g] = fmaf(-128.f, s[g], bf2f(g ? (bw >> 16) : (bw & 0xFFFFu)));
  }
  const uint32_t w[16] = {w4[0].x, w4[0].y, w4[0].z, w4[0].w, w4[1].x, w4[1].y, w4[1].z, w4[1].w,
                          w4[2].x, w4[2].y, w4[2].z, w4[2].w, w4[3].x, w4[3].y, w4[3].z, w4[3].w};
#pragma unroll
  for (int c = 0; c < 16; ++c) {  // 8 dims per word and chunk
    const int g = c >> 3;
    uint32_t pr[4];
    nib_pairs4(w[c], pr);  // (d0,d4), (d1,d5), (d2,d6), (d3,d7)
    float v[8];
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      v[i] = fmaf(s[g], __uint_as_float(pr[i] << 16), bb[g]);
      v[i + 4] = fmaf(s[g], __uint_as_float(pr[i] & 0xFFFF0000u), bb[g]);
    }
    const uint4 o = make_uint4(cvt_bf2(v[0], v[1]), cvt_bf2(v[2], v[3]), cvt_bf2(v[4], v[5]),
                               cvt_bf2(v[6], v[7]));
    *reinterpret_cast<uint4 *>(sk + (2 * h + g) * PA_BLOCK + sw_off(key, c & 7)) = o;
  }
}

// V tile: thread -> key tid / 2, dims [128 h, 128 h + 128): 12 words of the
// 3-bit stream, 8 dims (24 bits) per chunk.
__device__ __forceinline__ void pa_dequant_v(const PrefillAttnParams &p, size_t bh, int k0,
                                             uint8_t *sv_, int tid) {
  const int key = tid >> 1, h = tid & 1;
  const int kidx = min(k0 + key, p.keys - 1);
  const size_t row = bh * p.cap + kidx;
  const uint4 *src = reinterpret_cast<const uint4 *>(p.vc + row * 24 + h * 12);
  uint4 w4[3];
#pragma unroll
  for (int i = 0; i < 3; ++i) w4[i] = ldg_nc_v4(src + i);
  const uint2 svv = *reinterpret_cast<const uint2 *>(p.vs + row * 4);
  const uint2 bvv = *reinterpret_cast<const uint2 *>(p.vb + row * 4);
  float s[2], bb[2];
#pragma unroll
  for (int g = 0; g < 2; ++g) {
    const uint32_t sw = h ? svv.y : svv.x, bw = h ? bvv.y : bvv.x;
    s[g] = bf2f(g ? (sw >> 16) : (sw & 0xFFFFu));
    bb[g] = fmaf(-128.f, s[g], bf2f(g ? (bw >> 16) : (bw & 0xFFFFu)));
  }
  const uint32_t w[12] = {w4[0].x, w4[0].y, w4[0].z, w4[0].w, w4[1].x, w4[1].y,
                          w4[1].z, w4[1].w, w4[2].x, w4[2].y, w4[2].z, w4[2].w};
#pragma unroll
  for (int c = 0; c < 16; ++c) {
    const int bit = 24 * c, wi = bit >> 5, off = bit & 31;
    const uint32_t win = (off + 24 <= 32) ? (w[wi] >> off) : __funnelshift_r(w[wi], w[wi + 1], off);
    const int g = c >> 3;
    uint32_t o[4];
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      const uint32_t a = win >> (6 * k);
      const uint32_t pr = lop_and_or(a << 13, 0x00070000u, lop_and_or(a, 0x7u, 0x43004300u));
      o[k] = deq_pair(pr, s[g], bb[g]);
    }
    *reinterpret_cast<uint4 *>(sv_ + (2 * h + g) * PA_BLOCK + sw_off(key, c & 7)) =
        make_uint4(o[0], o[1], o[2], o[3]);
  }
}

__global__ void __launch_bounds__(PA_THREADS, 1) kv_prefill_attn_kernel(PrefillAttnParams p) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t *smem = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                              ~uintptr_t(1023));
  __shared__ __align__(8) uint64_t bar_s, bar_o;
  __shared__ uint32_t s_tmem;
  __shared__ int s_abort;
  const int tid = threadIdx.x, warp = tid >> 5;
  const int tile = p.n_row_tiles - 1 - blockIdx.x;  // longest (causal) tiles first
  const int bh_i = blockIdx.y;
  const int b = bh_i / p.Hkv, hkv = bh_i % p.Hkv;
  const size_t bh = (size_t)b * p.Hkv + hkv;
  const int P = p.P, p0 = tile * P;
  const int off = p.keys - p.Lq;  // absolute position of query 0
  const int last_pos = min(p0 + P, p.Lq) - 1;
  const int kend = p.causal ? off + last_pos + 1 : p.keys;  // visible keys of this CTA
  const int n_kt = (kend + PA_KT - 1) / PA_KT;

  if (tid == 0) {
    tc::mbar_init(&bar_s, 1);
    tc::mbar_init(&bar_o, 1);
    s_abort = 0;
    tc::fence_mbar_init();
  }
  if (warp == 0) {
    tc::tmem_alloc(&s_tmem, 512);
    tc::tmem_relinquish();
  }
  // Q tile: row m = r * P + j (query head hkv * rep + r, position p0 + j),
  // bf16(q * scale) like the reference.
  {
    const int m = tid >> 1, h = tid & 1;
    const int r = m / P, j = m % P;
    const bool valid = r < p.rep && p0 + j < p.Lq;
    const uint4 *src = reinterpret_cast<const uint4 *>(
        p.q + (((size_t)b * p.Hq + hkv * p.rep + (valid ? r : 0)) * p.Lq + (valid ? p0 + j : 0)) *
                  256 + h * 128);
#pragma unroll 4
    for (int c = 0; c < 16; ++c) {
      uint4 o = make_uint4(0, 0, 0, 0);
      if (valid) {
        const uint4 v = ldg_nc_v4(src + c);
        const uint32_t u[4] = {v.x, v.y, v.z, v.w};
        uint32_t y[4];
#pragma unroll
        for (int i = 0; i < 4; ++i)
          y[i] = pack_bf2(__fmul_rn(bf2f(u[i] & 0xFFFFu), p.scale),
                          __fmul_rn(bf2f(u[i] >> 16), p.scale));
        o = make_uint4(y[0], y[1], y[2], y[3]);
      }
      *reinterpret_cast<uint4 *>(smem + PA_Q + (2 * h + (c >> 3)) * PA_BLOCK + sw_off(m, c & 7)) = o;
    }
  }
  tc::tc_fence_before();
  __syncthreads();
  tc::tc_fence_after();
  const uint32_t tmem = s_tmem;
  volatile int *abort = &s_abort;
  const uint32_t idesc_s = tc::idesc_bf16_f32(128, 128);
  const uint32_t idesc_o = tc::idesc_bf16_f32(128, 256) | (1u << 16);  // B MN-major
  const uint32_t sbase = tc::smem_u32(smem);

  // softmax state (threads 0..127: row = tid = TMEM lane)
  const int m = tid;
  const int r_row = m / P, j_row = m % P;
  const bool row_valid = tid < PA_ROWS && r_row < p.rep && p0 + j_row < p.Lq;
  const int kmax = row_valid ? (p.causal ? off + p0 + j_row : p.keys - 1) : -1;
  float m_ref = -INFINITY, lsum = 0.f;
  const uint32_t trow = tmem + (((uint32_t)(warp & 3) * 32u) << 16);
  int n_s = 0, n_o = 0, w_s = 0, w_o = 0;  // MMA batches issued / waited (S, O)
  // tcgen05.ld/st are warp-collective (.sync.aligned): every branch around
  // them below is uniform per warp; a failed wait is turned into a
  // CTA-uniform abort at the next barrier.

  for (int kt = 0; kt < n_kt; ++kt) {
    const int k0 = kt * PA_KT;
    pa_dequant_k(p, bh, k0, smem + PA_K, tid);
    tc::fence_proxy_async_smem();
    __syncthreads();
    if (tid == 0) {
      tc::tc_fence_after();
#pragma unroll
      for (int kk = 0; kk < 16; ++kk) {
        const uint32_t o = (kk >> 2) * PA_BLOCK + (kk & 3) * 32;
        tc::mma_bf16_ss(tmem + PA_TS, tc::smem_desc_sw128(sbase + PA_Q + o),
                        tc::smem_desc_sw128(sbase + PA_K + o), idesc_s, kk > 0 ? 1u : 0u);
      }
      tc::mma_commit(&bar_s);
    }
    ++n_s;
    // V and P buffers are free once the previous O MMAs are done.
    if (n_o > w_o) {
      if (!tc::mbar_wait(&bar_o, (uint32_t)(w_o & 1), abort, PA_WAIT_NS)) s_abort = 1;
      ++w_o;
    }
    tc::tc_fence_after();
    if (!*abort) pa_dequant_v(p, bh, k0, smem + PA_V, tid);
    if (!tc::mbar_wait(&bar_s, (uint32_t)(w_s & 1), abort, PA_WAIT_NS)) s_abort = 1;
    ++w_s;
    __syncthreads();
    if (*abort) break;
    tc::tc_fence_after();
    if (tid < PA_ROWS) {  // warps 0-3: one row per thread
      // scores of this row: bf16-rounded, masked, in log2 units
      float sc[PA_KT];
      float mt = -INFINITY;
#pragma unroll
      for (int c0 = 0; c0 < PA_KT; c0 += 32) {
        uint32_t v[32];
        tc::tmem_ld32(trow + PA_TS + c0, v);
        tc::tmem_ld_wait();
#pragma unroll
        for (int i = 0; i < 32; ++i) {
          const int key = k0 + c0 + i;
          const float sv = key <= kmax ? rbf(__uint_as_float(v[i])) * 1.4426950408889634f
                                       : -INFINITY;
          sc[c0 + i] = sv;
          mt = fmaxf(mt, sv);
        }
      }
      const bool move = mt > m_ref + PA_RESCALE;
      const float alpha = !move ? 1.f : (m_ref == -INFINITY ? 0.f : ex2(m_ref - mt));
      if (move) {
        lsum *= alpha;
        m_ref = mt;
      }
      if (kt > 0 && __any_sync(0xffffffffu, move)) {  // the whole warp rescales its O rows
#pragma unroll 1
        for (int c0 = 0; c0 < 256; c0 += 32) {
          uint32_t v[32];
          tc::tmem_ld32(trow + PA_TO + c0, v);
          tc::tmem_ld_wait();
#pragma unroll
          for (int i = 0; i < 32; ++i) v[i] = __float_as_uint(__uint_as_float(v[i]) * alpha);
          tmem_st32(trow + PA_TO + c0, v);
        }
        tmem_st_wait();
      }
      // P row -> shared memory (2 blocks of 64 keys)
#pragma unroll
      for (int c = 0; c < 16; ++c) {
        float e[8];
#pragma unroll
        for (int i = 0; i < 8; ++i) {
          const float x = sc[8 * c + i];
          e[i] = x == -INFINITY ? 0.f : ex2(x - m_ref);
          lsum += e[i];
        }
        const uint4 o = make_uint4(cvt_bf2(e[0], e[1]), cvt_bf2(e[2], e[3]), cvt_bf2(e[4], e[5]),
                                   cvt_bf2(e[6], e[7]));
        *reinterpret_cast<uint4 *>(smem + PA_P + (c >> 3) * PA_BLOCK + sw_off(m, c & 7)) = o;
      }
    }
    tc::tc_fence_before();
    tc::fence_proxy_async_smem();
    __syncthreads();
    if (tid == 0) {
      tc::tc_fence_after();
#pragma unroll
      for (int kk = 0; kk < 8; ++kk) {
        const uint32_t a = (kk >> 2) * PA_BLOCK + (kk & 3) * 32;
        tc::mma_bf16_ss(tmem + PA_TO, tc::smem_desc_sw128(sbase + PA_P + a),
                        smem_desc_sw128_mn(sbase + PA_V + kk * 2048, PA_BLOCK, 1024), idesc_o,
                        (kt > 0 || kk > 0) ? 1u : 0u);
      }
      tc::mma_commit(&bar_o);
    }
    ++n_o;
  }
  // Wait (bounded) for every MMA batch this CTA issued before reading O or
  // freeing TMEM.
  while (w_s < n_s) {
    if (!tc::mbar_wait(&bar_s, (uint32_t)(w_s & 1), nullptr, PA_WAIT_NS)) s_abort = 1;
    ++w_s;
  }
  while (w_o < n_o) {
    if (!tc::mbar_wait(&bar_o, (uint32_t)(w_o & 1), nullptr, PA_WAIT_NS)) s_abort = 1;
    ++w_o;
  }
  __syncthreads();
  tc::tc_fence_after();
  const bool failed = *abort != 0;
  if (failed && tid == 0) flag_status(p.status, VB_STATUS_TIMEOUT);
  if (!failed && tid < PA_ROWS) {  // warp-uniform: all lanes load, valid rows store
    const float inv = lsum > 0.f ? 1.f / lsum : 0.f;
    uint16_t *dst = p.out +
        (((size_t)b * p.Hq + hkv * p.rep + (row_valid ? r_row : 0)) * p.Lq + p0 +
         (row_valid ? j_row : 0)) * 256;
#pragma unroll 1
    for (int c0 = 0; c0 < 256; c0 += 32) {
      uint32_t v[32];
      tc::tmem_ld32(trow + PA_TO + c0, v);
      tc::tmem_ld_wait();
      float o[32];
#pragma unroll
      for (int i = 0; i < 32; ++i) o[i] = rbf(__uint_as_float(v[i]) * inv);
      if (p.rv) {
        float y[32];
#pragma unroll
        for (int blk = 0; blk < 8; ++blk) {
          const float *R = p.rv + (size_t)((c0 >> 2) + blk) * 16;
#pragma unroll
          for (int i = 0; i < 4; ++i) {
            float acc = 0.f;
#pragma unroll
            for (int kk = 0; kk < 4; ++kk)
              acc = __fadd_rn(acc, __fmul_rn(o[4 * blk + kk], rbf(__ldg(R + i * 4 + kk))));
            y[4 * blk + i] = rbf(acc);
          }
        }
#pragma unroll
        for (int i = 0; i < 32; ++i) o[i] = y[i];
      }
      if (row_valid) {
        uint4 *d4 = reinterpret_cast<uint4 *>(dst + c0);
#pragma unroll
        for (int q = 0; q < 4; ++q)
          d4[q] = make_uint4(pack_bf2(o[8 * q], o[8 * q + 1]), pack_bf2(o[8 * q + 2], o[8 * q + 3]),
                             pack_bf2(o[8 * q + 4], o[8 * q + 5]),
                             pack_bf2(o[8 * q + 6], o[8 * q + 7]));
      }
    }
  }
  tc::tc_fence_before();
  __syncthreads();
  tc::tc_fence_after();
  if (warp == 0) tc::tmem_dealloc(tmem, 512);
}

}  // namespace
}  // namespace vb

using namespace vb;

extern "C" {

int vb_kv_prefill_attn(const uint16_t *q, const uint32_t *k_codes, const uint16_t *k_scales,
                       const uint16_t *k_biases, const uint32_t *v_codes,
                       const uint16_t *v_scales, const uint16_t *v_biases,
                       const float *rv_blocks, int32_t batch, int32_t q_heads, int32_t kv_heads,
                       int32_t L, int32_t dim, int32_t keys, int32_t cap, int32_t group,
                       int32_t k_bits, int32_t v_bits, float scale, int32_t causal,
                       uint16_t *out, int32_t *status, vb_stream_t stream) {
  VB_REQUIRE(dim == 256 && group == 64 && k_bits == 4 && v_bits == 3,
             "vb_kv_prefill_attn: supports D=256, group 64, K4/V3 (got D=%d g=%d k%d v%d)",
             dim, group, k_bits, v_bits);
  VB_REQUIRE(batch > 0 && kv_heads > 0 && q_heads % kv_heads == 0,
             "vb_kv_prefill_attn: heads %d/%d", q_heads, kv_heads);
  const int rep = q_heads / kv_heads;
  VB_REQUIRE(rep <= PA_ROWS && PA_ROWS % rep == 0, "vb_kv_prefill_attn: %d query heads per kv head", rep);
  VB_REQUIRE(L >= 1 && keys >= L && keys <= cap, "vb_kv_prefill_attn: L=%d keys=%d cap=%d", L,
             keys, cap);
  VB_REQUIRE(q && k_codes && k_scales && k_biases && v_codes && v_scales && v_biases && out,
             "vb_kv_prefill_attn: null pointer");
  VB_REQUIRE(((uintptr_t)q % 16) == 0 && ((uintptr_t)out % 16) == 0 &&
                 ((uintptr_t)k_codes % 16) == 0 && ((uintptr_t)v_codes % 16) == 0 &&
                 ((uintptr_t)k_scales % 8) == 0 && ((uintptr_t)k_biases % 8) == 0 &&
                 ((uintptr_t)v_scales % 8) == 0 && ((uintptr_t)v_biases % 8) == 0,
             "vb_kv_prefill_attn: q/out/codes must be 16-byte and scales 8-byte aligned");
  PrefillAttnParams p;
  p.q = q; p.kc = k_codes; p.vc = v_codes; p.ks = k_scales; p.kb = k_biases;
  p.vs = v_scales; p.vb = v_biases; p.rv = rv_blocks;
  p.B = batch; p.Hq = q_heads; p.Hkv = kv_heads; p.Lq = L; p.keys = keys; p.cap = cap;
  p.rep = rep; p.P = PA_ROWS / rep; p.causal = causal ? 1 : 0; p.scale = scale;
  p.n_row_tiles = (L + p.P - 1) / p.P;
  p.out = out; p.status = status;
  VB_REQUIRE((long long)batch * kv_heads <= 65535, "vb_kv_prefill_attn: too many heads");
  static bool attr_done = false;
  if (!attr_done) {
    const cudaError_t e = cudaFuncSetAttribute(kv_prefill_attn_kernel,
                                               cudaFuncAttributeMaxDynamicSharedMemorySize, PA_SMEM);
    if (e != cudaSuccess) return set_error(VB_ERR_CUDA, "kv_prefill_attn_kernel attributes: %s", cudaGetErrorString(e));
    attr_done = true;
  }
  kv_prefill_attn_kernel<<<dim3(p.n_row_tiles, batch * kv_heads), PA_THREADS, PA_SMEM,
                           as_stream(stream)>>>(p);
  return check_launch("kv_prefill_attn_kernel");
}

}  // extern "C"
