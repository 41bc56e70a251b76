// Affine dequantization of packed rows (MLX affine format) and the
// one-launch seeded fill of a synthetic expert pool.
//
// vb_dequantize is the standalone form of the dequantization every fused
// kernel performs: w[r, c] = q[r, c] * scale[r, c / g] + bias[r, c / g] with
// q the c-th `bits`-wide field of row r's LSB-first uint32 bitstream
// (native/ext/compute/fused_moe.cpp:131-145 `qvalue`; MLX mx.dequantize).
// The 4-bit bf16 path calls dequant4_bf16x2, the helper that produces every
// bf16 weight operand of the prefill GEMMs, so its output pins those
// operands bit for bit.
#include <algorithm>

#include "common.cuh"

namespace vb {

// 4-bit codes, bf16 output: one thread per packed word (8 columns).
__global__ void dequant4_bf16_kernel(const uint32_t *__restrict__ words,
                                     const uint16_t *__restrict__ scales,
                                     const uint16_t *__restrict__ biases, int64_t rows,
                                     int cols, int gshift, uint16_t *__restrict__ out) {
  const int wpr = cols >> 3;
  const int64_t n = rows * wpr;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n;
       i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t r = i / wpr;
    const int wc = (int)(i - r * wpr);
    const int64_t gi = r * (cols >> gshift) + ((wc * 8) >> gshift);
    const uint32_t sc = scales[gi], bi = biases[gi];
    uint32_t o[4];
    dequant4_bf16x2(words[i], sc | (sc << 16), bi | (bi << 16), o);
    // pairs (0,4),(1,5),(2,6),(3,7) -> columns 0..7
    *reinterpret_cast<uint4 *>(out + r * cols + wc * 8) =
        make_uint4(__byte_perm(o[0], o[1], 0x5410), __byte_perm(o[2], o[3], 0x5410),
                   __byte_perm(o[0], o[1], 0x7632), __byte_perm(o[2], o[3], 0x7632));
  }
}

// Any width 2..8: one thread per output value; a field that straddles a
// word boundary takes its high bits from the next word.
__global__ void dequant_any_kernel(const uint32_t *__restrict__ words,
                                   const uint16_t *__restrict__ scales,
                                   const uint16_t *__restrict__ biases, int64_t rows, int cols,
                                   int group, int bits, int out_bf16, void *__restrict__ out) {
  const int wpr = cols * bits / 32;
  const uint32_t mask = (1u << bits) - 1u;
  const int64_t n = rows * cols;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n;
       i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t r = i / cols;
    const int c = (int)(i - r * cols);
    const int bit = c * bits, wi = bit >> 5, sh = bit & 31;
    const uint32_t *row = words + r * wpr;
    uint32_t q = row[wi] >> sh;
    if (sh + bits > 32) q |= row[wi + 1] << (32 - sh);
    q &= mask;
    const int64_t gi = r * (cols / group) + c / group;
    const float v = __fmaf_rn((float)q, bf2f(scales[gi]), bf2f(biases[gi]));
    if (out_bf16)
      reinterpret_cast<uint16_t *>(out)[i] = f2bf(v);
    else
      reinterpret_cast<float *>(out)[i] = v;
  }
}

// One launch fills the nine tensors of many synthetic experts: blockIdx.y
// is the expert, blockIdx.z the projection (gate, up, down). The values are
// those of vb_synth_fill_u32 / vb_synth_fill_scales called per tensor with
// the per-tensor seeds mix_seed(expert_seed, 3*proj) (codes) and
// mix_seed(expert_seed, 3*proj + 1) (scales, biases = bias_mul * scale).
__host__ __device__ inline uint64_t splitmix(uint64_t z) {
  z += 0x9E3779B97F4A7C15ull;
  z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
  z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
  return z ^ (z >> 31);
}
__host__ __device__ inline uint64_t mix_seed(uint64_t seed, uint64_t salt) {
  uint64_t z = seed * 0x9E3779B97F4A7C15ull + salt * 0xBF58476D1CE4E5B9ull + 0x94D049BB133111EBull;
  return z ^ (z >> 31);
}

constexpr int SYNTH_POOL_MAX = 1024;
struct SynthPoolList {
  int32_t slot[SYNTH_POOL_MAX];
  uint64_t seed[SYNTH_POOL_MAX];
};

__global__ void synth_pool_kernel(VbQuantPool pool, SynthPoolList list, int hidden, int inter,
                                  int bits, int group, float lo, float hi, float bias_mul) {
  const int e = blockIdx.y, proj = blockIdx.z;
  const int slot = list.slot[e];
  const uint64_t eseed = list.seed[e];
  const int out_d = proj < 2 ? inter : hidden, in_d = proj < 2 ? hidden : inter;
  const int64_t nw = (int64_t)out_d * (in_d * bits / 32);
  const int64_t ns = (int64_t)out_d * (in_d / group);
  uint32_t *w = (uint32_t *)pool_ptr(pool, 3 * proj, slot);
  uint16_t *s = (uint16_t *)pool_ptr(pool, 3 * proj + 1, slot);
  uint16_t *b = (uint16_t *)pool_ptr(pool, 3 * proj + 2, slot);
  const uint64_t kw = splitmix(mix_seed(eseed, 3 * proj));
  const uint64_t ks = splitmix(mix_seed(eseed, 3 * proj + 1) ^ 0x5CA1E5ull);
  const int64_t stride = (int64_t)gridDim.x * blockDim.x;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < nw; i += stride)
    w[i] = (uint32_t)(splitmix(kw ^ (uint64_t)i) >> 32);
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < ns; i += stride) {
    const uint32_t r = (uint32_t)(splitmix(ks ^ (uint64_t)i) >> 40);  // 24 bits
    const float u = (float)r * (1.0f / 16777216.0f);
    const uint16_t sv = f2bf(__fmaf_rn(__fsub_rn(hi, lo), u, lo));
    s[i] = sv;
    b[i] = f2bf(bf2f(sv) * bias_mul);
  }
}

}  // namespace vb

using namespace vb;

extern "C" {

int vb_dequantize(const uint32_t *words, const uint16_t *scales, const uint16_t *biases,
                  int64_t rows, int32_t cols, int32_t group, int32_t bits, int32_t out_bf16,
                  void *out, vb_stream_t stream) {
  VB_REQUIRE(rows >= 0 && cols > 0 && group > 0 && cols % group == 0,
             "vb_dequantize: rows=%lld cols=%d group=%d", (long long)rows, cols, group);
  VB_REQUIRE(bits >= 2 && bits <= 8 && (int64_t)cols * bits % 32 == 0,
             "vb_dequantize: bits=%d with cols=%d (cols*bits must fill whole words)", bits,
             cols);
  if (rows == 0) return VB_OK;
  VB_REQUIRE(words && scales && biases && out, "vb_dequantize: null pointer");
  const cudaStream_t s = as_stream(stream);
  const bool pow2_group = (group & (group - 1)) == 0 && group >= 8;
  if (bits == 4 && out_bf16 && pow2_group && ((uintptr_t)out & 15) == 0) {
    const int64_t n = rows * (cols / 8);
    const int64_t blocks = std::min<int64_t>((n + 255) / 256, 148 * 16);
    dequant4_bf16_kernel<<<(unsigned)blocks, 256, 0, s>>>(words, scales, biases, rows, cols,
                                                          __builtin_ctz(group), (uint16_t *)out);
  } else {
    const int64_t n = rows * cols;
    const int64_t blocks = std::min<int64_t>((n + 255) / 256, 148 * 16);
    dequant_any_kernel<<<(unsigned)blocks, 256, 0, s>>>(words, scales, biases, rows, cols, group,
                                                        bits, out_bf16, out);
  }
  return check_launch("vb_dequantize");
}

int vb_synth_fill_pool(const VbQuantPool *pool, const int32_t *slots, const uint64_t *seeds,
                       int32_t n, int32_t hidden, int32_t inter, int32_t bits, int32_t group,
                       float lo, float hi, float bias_mul, vb_stream_t stream) {
  VB_REQUIRE(pool && n >= 0 && hidden > 0 && inter > 0 && group > 0 && bits >= 2 && bits <= 8,
             "vb_synth_fill_pool: bad args");
  VB_REQUIRE(hidden % group == 0 && inter % group == 0 && hidden * bits % 32 == 0 &&
                 inter * bits % 32 == 0,
             "vb_synth_fill_pool: hidden=%d inter=%d group=%d bits=%d", hidden, inter, group,
             bits);
  if (n == 0) return VB_OK;
  VB_REQUIRE(slots && seeds, "vb_synth_fill_pool: null slots/seeds");
  for (int i = 0; i < 9; ++i) VB_REQUIRE(pool->ptr[i], "vb_synth_fill_pool: null pool tensor");
  for (int32_t first = 0; first < n; first += SYNTH_POOL_MAX) {
    const int32_t m = std::min<int32_t>(SYNTH_POOL_MAX, n - first);
    SynthPoolList list;
    for (int32_t i = 0; i < m; ++i) {
      VB_REQUIRE(slots[first + i] >= 0 && slots[first + i] < pool->cap,
                 "vb_synth_fill_pool: slot %d outside [0, %d)", slots[first + i], pool->cap);
      list.slot[i] = slots[first + i];
      list.seed[i] = seeds[first + i];
    }
    synth_pool_kernel<<<dim3(16, (unsigned)m, 3), 256, 0, as_stream(stream)>>>(
        *pool, list, hidden, inter, bits, group, lo, hi, bias_mul);
    const int rc = check_launch("vb_synth_fill_pool");
    if (rc != VB_OK) return rc;
  }
  return VB_OK;
}

}  // extern "C"
