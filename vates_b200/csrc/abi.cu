// Error reporting, version, slot-table gather and seeded synthetic fills.
#include <cstdarg>
#include <cstdio>

#include "common.cuh"

namespace vb {

static thread_local char g_last_error[512] = "";

int set_error(int code, const char *fmt, ...) {
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(g_last_error, sizeof(g_last_error), fmt, ap);
  va_end(ap);
  return code;
}

int check_launch(const char *what) {
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess)
    return set_error(VB_ERR_CUDA, "%s: %s", what, cudaGetErrorString(e));
  return VB_OK;
}

// ----------------------------------------------------------------------------
// Slot-table gather (demand.cpp:1201-1232 without row leases: the table is
// read-only while a step runs).
// ----------------------------------------------------------------------------
__global__ void slot_remap_kernel(const uint32_t *__restrict__ ids,
                                  const int32_t *__restrict__ table,
                                  int32_t *__restrict__ local, int64_t n,
                                  int32_t table_size, int32_t *miss_count,
                                  int32_t *status) {
  int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x;
  if (i >= n) return;
  uint32_t id = ids[i];
  int32_t slot = -1;
  if (id < (uint32_t)table_size) {
    slot = table[id];
  } else {
    flag_status(status, VB_STATUS_BOUNDS);
  }
  local[i] = slot;
  if (slot < 0 && miss_count) atomicAdd(miss_count, 1);
}

// ----------------------------------------------------------------------------
// Counter-hash synthetic data (splitmix64 finaliser of seed ^ index).
// ----------------------------------------------------------------------------
__host__ __device__ inline uint64_t mix64(uint64_t z) {
  z += 0x9E3779B97F4A7C15ull;
  z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
  z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
  return z ^ (z >> 31);
}

__global__ void synth_u32_kernel(uint32_t *words, int64_t n, uint64_t seed) {
  int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x;
  int64_t stride = (int64_t)gridDim.x * blockDim.x;
  uint64_t key = mix64(seed);
  for (; i < n; i += stride) words[i] = (uint32_t)(mix64(key ^ (uint64_t)i) >> 32);
}

__global__ void synth_scales_kernel(uint16_t *scales, uint16_t *biases,
                                    int64_t n, uint64_t seed, float lo,
                                    float hi, float bias_mul) {
  int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x;
  int64_t stride = (int64_t)gridDim.x * blockDim.x;
  uint64_t key = mix64(seed ^ 0x5CA1E5ull);
  for (; i < n; i += stride) {
    uint32_t r = (uint32_t)(mix64(key ^ (uint64_t)i) >> 40);  // 24 bits
    float u = (float)r * (1.0f / 16777216.0f);
    uint16_t s = f2bf(__fmaf_rn(__fsub_rn(hi, lo), u, lo));
    scales[i] = s;
    if (biases) biases[i] = f2bf(bf2f(s) * bias_mul);
  }
}

}  // namespace vb

using namespace vb;

extern "C" {

int vb_version(void) { return 100; }

const char *vb_last_error(void) { return g_last_error; }

int vb_slot_remap(const uint32_t *ids, const int32_t *table, int32_t *local,
                  int64_t n, int32_t table_size, int32_t *miss_count,
                  int32_t *status, vb_stream_t stream) {
  VB_REQUIRE(n >= 0 && table_size > 0, "vb_slot_remap: n=%lld table_size=%d",
             (long long)n, table_size);
  if (n == 0) return VB_OK;
  VB_REQUIRE(ids && table && local, "vb_slot_remap: null pointer");
  int threads = 256;
  int64_t blocks = (n + threads - 1) / threads;
  slot_remap_kernel<<<(unsigned)blocks, threads, 0, as_stream(stream)>>>(
      ids, table, local, n, table_size, miss_count, status);
  return check_launch("vb_slot_remap");
}

int vb_synth_fill_u32(uint32_t *words, int64_t n, uint64_t seed,
                      vb_stream_t stream) {
  VB_REQUIRE(words && n >= 0, "vb_synth_fill_u32: bad args");
  if (n == 0) return VB_OK;
  int64_t blocks = (n + 255) / 256;
  if (blocks > 148 * 32) blocks = 148 * 32;
  synth_u32_kernel<<<(unsigned)blocks, 256, 0, as_stream(stream)>>>(words, n, seed);
  return check_launch("vb_synth_fill_u32");
}

int vb_synth_fill_scales(uint16_t *scales, uint16_t *biases, int64_t n,
                         uint64_t seed, float lo, float hi, float bias_mul,
                         vb_stream_t stream) {
  VB_REQUIRE(scales && n >= 0, "vb_synth_fill_scales: bad args");
  if (n == 0) return VB_OK;
  int64_t blocks = (n + 255) / 256;
  if (blocks > 148 * 32) blocks = 148 * 32;
  synth_scales_kernel<<<(unsigned)blocks, 256, 0, as_stream(stream)>>>(
      scales, biases, n, seed, lo, hi, bias_mul);
  return check_launch("vb_synth_fill_scales");
}

}  // extern "C"
