// IsoQuant KV append: SO(4) block rotation + MLX affine quantize + pack.
//
// Reference: rotate_last (mlx_streaming/core/cache/quant_kv.py:68-70) applied
// to k (R_k) and v (R_v) at kv_quant_patch.py:49-55, then
// AsymmetricQuantizedKVCache.update_and_fetch (quant_kv.py:105-137), which
// quantizes with mx.quantize(group 64, K 4-bit / V 3-bit) and slice-assigns
// the codes/scales/biases at [offset, offset+n).
//
// One row (batch, head, position) of D dims is handled by D/8 lanes, 8
// consecutive dims per lane (two 4x4 rotation blocks). A 64-dim group spans 8
// lanes, so group min/max are 3 xor-shuffles. The row's codes form one
// continuous LSB-first bitstream; each lane builds a 64-bit chunk of its 8
// codes and words are assembled from at most two neighbouring lanes' chunks.
#include "kv_quant.cuh"

namespace vb {

template <int LPR>  // lanes per row = D/8
__global__ void __launch_bounds__(256) kv_quant_kernel(
    const uint16_t *__restrict__ src, const float *__restrict__ blocks,
    int64_t rows, int n, int heads_total, int bits, int offset, int cap,
    uint32_t *__restrict__ codes, uint16_t *__restrict__ scales,
    uint16_t *__restrict__ biases, const int32_t *__restrict__ offset_dev,
    int32_t *status) {
  constexpr int D = LPR * 8;
  pdl_launch_dependents();
  pdl_wait();
  if (offset_dev) {  // position read on the device (the same for every thread)
    offset = *offset_dev;
    if (offset < 0 || offset + n > cap) {
      if (blockIdx.x == 0 && threadIdx.x == 0) flag_status(status, VB_STATUS_BOUNDS);
      return;
    }
  }
  const int lane = threadIdx.x & 31;
  const int sub = lane % LPR;           // lane within the row
  const int rsub = lane / LPR;          // row within the warp
  const int64_t row = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) / 32 * (32 / LPR) + rsub;
  const bool valid = row < rows;
  const int64_t r = valid ? row : rows - 1;

  float v[8];
  {
    const uint4 raw = *reinterpret_cast<const uint4 *>(src + r * D + sub * 8);
    const uint32_t w[4] = {raw.x, raw.y, raw.z, raw.w};
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      v[2 * i] = bf2f(w[i] & 0xFFFF);
      v[2 * i + 1] = bf2f(w[i] >> 16);
    }
  }
  if (blocks) rotate8(v, blocks, sub * 2, false);

  const int64_t bh = r / n, pos = offset + (r % n);
  kv_quant_store<LPR>(v, sub, rsub, bits, valid, bh * cap + pos, codes, scales, biases);
}

__global__ void so4_rotate_kernel(const uint16_t *__restrict__ src,
                                  const float *__restrict__ blocks, int64_t rows,
                                  int dim, int transpose, uint16_t *__restrict__ dst) {
  const int64_t idx = blockIdx.x * (int64_t)blockDim.x + threadIdx.x;  // one per 8 dims
  const int per_row = dim / 8;
  if (idx >= rows * per_row) return;
  const int64_t r = idx / per_row;
  const int sub = (int)(idx % per_row);
  float v[8];
  const uint4 raw = *reinterpret_cast<const uint4 *>(src + r * dim + sub * 8);
  const uint32_t w[4] = {raw.x, raw.y, raw.z, raw.w};
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    v[2 * i] = bf2f(w[i] & 0xFFFF);
    v[2 * i + 1] = bf2f(w[i] >> 16);
  }
  rotate8(v, blocks, sub * 2, transpose != 0);
  uint4 o;
  o.x = pack_bf2(v[0], v[1]);
  o.y = pack_bf2(v[2], v[3]);
  o.z = pack_bf2(v[4], v[5]);
  o.w = pack_bf2(v[6], v[7]);
  *reinterpret_cast<uint4 *>(dst + r * dim + sub * 8) = o;
}

}  // namespace vb

using namespace vb;

extern "C" {

static int kv_quant_append_impl(const uint16_t *src, const float *so4_blocks,
                                int32_t batch, int32_t heads, int32_t n, int32_t dim,
                                int32_t group, int32_t bits, int32_t offset,
                                const int32_t *offset_dev, int32_t cap, uint32_t *codes,
                                uint16_t *scales, uint16_t *biases, int32_t *status,
                                vb_stream_t stream) {
  VB_REQUIRE(dim == 64 || dim == 128 || dim == 256, "vb_kv_quant_append: dim=%d", dim);
  VB_REQUIRE(group == 64, "vb_kv_quant_append: group=%d (64 only)", group);
  VB_REQUIRE(bits == 2 || bits == 3 || bits == 4 || bits == 5 || bits == 6 || bits == 8,
             "vb_kv_quant_append: bits=%d", bits);
  VB_REQUIRE(batch > 0 && heads > 0 && n >= 0 && n <= cap &&
                 (offset_dev || (offset >= 0 && offset + n <= cap)),
             "vb_kv_quant_append: batch=%d heads=%d n=%d offset=%d cap=%d", batch,
             heads, n, offset, cap);
  if (n == 0) return VB_OK;
  VB_REQUIRE(src && codes && scales && biases, "vb_kv_quant_append: null pointer");
  const int64_t rows = (int64_t)batch * heads * n;
  const int lpr = dim / 8;
  const int64_t rows_per_block = 8 * (32 / lpr);  // 8 warps
  const unsigned blocks = (unsigned)((rows + rows_per_block - 1) / rows_per_block);
  cudaStream_t s = as_stream(stream);
  auto kern = lpr == 32 ? kv_quant_kernel<32> : (lpr == 16 ? kv_quant_kernel<16> : kv_quant_kernel<8>);
  vb_launch(kern, dim3(blocks), dim3(256), 0, s, false, src, so4_blocks, rows, (int)n,
            (int)(batch * heads), (int)bits, (int)offset, (int)cap, codes, scales, biases,
            offset_dev, status);
  return check_launch("kv_quant_kernel");
}

int vb_kv_quant_append(const uint16_t *src, const float *so4_blocks,
                       int32_t batch, int32_t heads, int32_t n, int32_t dim,
                       int32_t group, int32_t bits, int32_t offset,
                       int32_t cap, uint32_t *codes, uint16_t *scales,
                       uint16_t *biases, vb_stream_t stream) {
  return kv_quant_append_impl(src, so4_blocks, batch, heads, n, dim, group, bits, offset,
                              nullptr, cap, codes, scales, biases, nullptr, stream);
}

int vb_kv_quant_append_at(const uint16_t *src, const float *so4_blocks,
                          int32_t batch, int32_t heads, int32_t n, int32_t dim,
                          int32_t group, int32_t bits, const int32_t *offset,
                          int32_t cap, uint32_t *codes, uint16_t *scales,
                          uint16_t *biases, int32_t *status, vb_stream_t stream) {
  VB_REQUIRE(offset != nullptr, "vb_kv_quant_append_at: null position");
  return kv_quant_append_impl(src, so4_blocks, batch, heads, n, dim, group, bits, 0, offset,
                              cap, codes, scales, biases, status, stream);
}

int vb_so4_rotate(const uint16_t *src, const float *so4_blocks, int64_t rows,
                  int32_t dim, int32_t transpose, uint16_t *dst,
                  vb_stream_t stream) {
  VB_REQUIRE(dim % 8 == 0 && dim > 0, "vb_so4_rotate: dim=%d", dim);
  VB_REQUIRE(rows >= 0, "vb_so4_rotate: rows");
  if (rows == 0) return VB_OK;
  VB_REQUIRE(src && so4_blocks && dst, "vb_so4_rotate: null pointer");
  const int64_t total = rows * (dim / 8);
  so4_rotate_kernel<<<(unsigned)((total + 255) / 256), 256, 0, as_stream(stream)>>>(
      src, so4_blocks, rows, dim, transpose, dst);
  return check_launch("so4_rotate_kernel");
}

}  // extern "C"
