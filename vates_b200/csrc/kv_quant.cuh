// MLX affine quantize + pack of one cache row held 8 values per lane: the
// shared tail of the IsoQuant KV append kernels (kv_quant.cu, and the fused
// attention input side in qwen_next.cu).
//
// Reference: AsymmetricQuantizedKVCache.update_and_fetch
// (mlx_streaming/core/cache/quant_kv.py:105-137): mx.quantize with group 64
// (K 4-bit, V 3-bit), codes slice-assigned at the row's position.
#pragma once

#include "common.cuh"

namespace vb {

// v: this lane's 8 consecutive dims (already SO(4)-rotated) of a row of
// D = 8 LPR dims spread over LPR lanes (lane sub of the row; rsub = the
// row's index inside the warp). A 64-dim group spans 8 lanes, so the group
// min/max are three xor-shuffles; the row's codes form one continuous
// LSB-first bitstream: each lane builds a 64-bit chunk of its 8 codes and
// words are assembled from at most two neighbouring lanes' chunks. Every lane
// of the warp must call this (shuffles); rows with !valid store nothing.
// crow: the cache row (head * cap + position).
template <int LPR>
__device__ __forceinline__ void kv_quant_store(float (&v)[8], int sub, int rsub, int bits,
                                               bool valid, int64_t crow, uint32_t *codes,
                                               uint16_t *scales, uint16_t *biases) {
  constexpr int D = LPR * 8;
  // MLX affine quantization of this lane's group (8 lanes = 64 dims).
  float mn = v[0], mx = v[0];
#pragma unroll
  for (int i = 1; i < 8; ++i) { mn = fminf(mn, v[i]); mx = fmaxf(mx, v[i]); }
#pragma unroll
  for (int o = 1; o < 8; o <<= 1) {
    mn = fminf(mn, __shfl_xor_sync(0xffffffffu, mn, o));
    mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
  }
  const float n_bins = (float)((1 << bits) - 1);
  float scale = fmaxf(__fdiv_rn(__fsub_rn(mx, mn), n_bins), 1e-7f);
  const bool side = fabsf(mn) > fabsf(mx);
  scale = side ? scale : -scale;
  const float edge = side ? mn : mx;
  const float q0 = rintf(__fdiv_rn(edge, scale));
  float bias = 0.f;
  if (q0 != 0.f) {
    scale = __fdiv_rn(edge, q0);
    bias = edge;
  }
  uint64_t chunk = 0;
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    float q = rintf(__fdiv_rn(__fsub_rn(v[i], bias), scale));
    q = fminf(fmaxf(q, 0.f), n_bins);
    chunk |= (uint64_t)(uint32_t)q << (bits * i);
  }

  const int words_per_row = D * bits / 32;
  const int cbits = 8 * bits;           // bits per lane chunk
  const int base_lane = rsub * LPR;
  const int iters = (words_per_row + LPR - 1) / LPR;
  for (int it = 0; it < iters; ++it) {
    const int w = sub + it * LPR;
    const int wq = w < words_per_row ? w : words_per_row - 1;
    const int l0 = (32 * wq) / cbits;
    const int o = 32 * wq - l0 * cbits;
    const int l1 = l0 + 1 < LPR ? l0 + 1 : l0;
    const uint32_t lo0 = __shfl_sync(0xffffffffu, (uint32_t)chunk, base_lane + l0);
    const uint32_t hi0 = __shfl_sync(0xffffffffu, (uint32_t)(chunk >> 32), base_lane + l0);
    const uint32_t lo1 = __shfl_sync(0xffffffffu, (uint32_t)chunk, base_lane + l1);
    const uint32_t hi1 = __shfl_sync(0xffffffffu, (uint32_t)(chunk >> 32), base_lane + l1);
    const uint64_t c0 = ((uint64_t)hi0 << 32) | lo0;
    const uint64_t c1 = ((uint64_t)hi1 << 32) | lo1;
    uint64_t word = c0 >> o;
    if (cbits - o < 32 && l1 != l0) word |= c1 << (cbits - o);
    if (valid && w < words_per_row) codes[crow * words_per_row + w] = (uint32_t)word;
  }
  if (valid && (sub & 7) == 0) {
    const int gi = sub >> 3;
    scales[crow * (D / 64) + gi] = f2bf(scale);
    biases[crow * (D / 64) + gi] = f2bf(bias);
  }
}

}  // namespace vb
