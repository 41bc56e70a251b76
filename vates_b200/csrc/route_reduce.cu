// Deterministic route reduce: deterministic_route_reduce
// (mlx_streaming/core/moe/custom_kernel.py:20-118).
//
// The reference sorts a group's flat route positions and lets one
// segment-start thread per (token, column) add the token's routes in rank
// order, rounding to the output dtype after each add (custom_kernel.py:63-77).
// Here the positions are scattered into a dense [tokens*k] inverse map (no
// sort needed: positions are unique), and one thread per (token, column pair)
// walks the k ranks in order. No atomics, so results are bit-reproducible.
#include "common.cuh"

namespace vb {

__global__ void rr_scatter_kernel(const int32_t *__restrict__ pos, int32_t G,
                                  int32_t *__restrict__ inv, int64_t limit,
                                  int32_t *status) {
  int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= G) return;
  int32_t q = pos[i];
  if (q < 0 || (int64_t)q >= limit) {
    flag_status(status, VB_STATUS_BOUNDS);
    return;
  }
  inv[q] = i;
}

template <bool BF16>
__global__ void rr_reduce_kernel(const void *__restrict__ previous,
                                 const void *__restrict__ weighted,
                                 const int32_t *__restrict__ inv, int tokens,
                                 int hidden, int k, void *out) {
  const int half = hidden / 2;
  int64_t idx = blockIdx.x * (int64_t)blockDim.x + threadIdx.x;
  if (idx >= (int64_t)tokens * half) return;
  const int t = (int)(idx / half);
  const int c2 = (int)(idx - (int64_t)t * half);
  const int32_t *inv_t = inv + (size_t)t * k;
  if (BF16) {
    const uint32_t *prev = (const uint32_t *)previous;
    const uint32_t *w = (const uint32_t *)weighted;
    uint32_t pv = prev[(size_t)t * half + c2];
    float a0 = bf2f(pv & 0xFFFF), a1 = bf2f(pv >> 16);
    for (int j = 0; j < k; ++j) {
      int i = inv_t[j];
      if (i < 0) continue;
      uint32_t wv = w[(size_t)i * half + c2];
      a0 = rbf(__fadd_rn(a0, bf2f(wv & 0xFFFF)));
      a1 = rbf(__fadd_rn(a1, bf2f(wv >> 16)));
    }
    ((uint32_t *)out)[(size_t)t * half + c2] = pack_bf2(a0, a1);
  } else {
    const float2 *prev = (const float2 *)previous;
    const float2 *w = (const float2 *)weighted;
    float2 a = prev[(size_t)t * half + c2];
    for (int j = 0; j < k; ++j) {
      int i = inv_t[j];
      if (i < 0) continue;
      float2 wv = w[(size_t)i * half + c2];
      a.x = __fadd_rn(a.x, wv.x);
      a.y = __fadd_rn(a.y, wv.y);
    }
    ((float2 *)out)[(size_t)t * half + c2] = a;
  }
}

}  // namespace vb

using namespace vb;

extern "C" {

size_t vb_route_reduce_workspace_size(int32_t tokens, int32_t k) {
  if (tokens <= 0 || k <= 0) return 0;
  return align_up((size_t)tokens * k * sizeof(int32_t), 256);
}

int vb_route_reduce(const void *previous, const void *weighted,
                    const int32_t *assignment_pos, int32_t groups,
                    int32_t tokens, int32_t hidden, int32_t k, int32_t dtype,
                    void *out, int32_t *status, void *workspace,
                    size_t workspace_bytes, vb_stream_t stream) {
  VB_REQUIRE(tokens > 0 && hidden > 0 && k > 0 && groups >= 0,
             "vb_route_reduce: tokens=%d hidden=%d k=%d groups=%d", tokens,
             hidden, k, groups);
  VB_REQUIRE(hidden % 2 == 0, "vb_route_reduce: hidden must be even");
  VB_REQUIRE(dtype == 0 || dtype == 1, "vb_route_reduce: dtype=%d", dtype);
  VB_REQUIRE(previous && out && (groups == 0 || (weighted && assignment_pos)),
             "vb_route_reduce: null pointer");
  VB_REQUIRE(workspace && workspace_bytes >= vb_route_reduce_workspace_size(tokens, k),
             "vb_route_reduce: workspace too small");
  cudaStream_t s = as_stream(stream);
  int32_t *inv = static_cast<int32_t *>(workspace);
  const int64_t limit = (int64_t)tokens * k;
  cudaError_t e = cudaMemsetAsync(inv, 0xFF, (size_t)limit * sizeof(int32_t), s);
  if (e != cudaSuccess) return set_error(VB_ERR_CUDA, "vb_route_reduce: %s", cudaGetErrorString(e));
  if (groups > 0) {
    rr_scatter_kernel<<<(groups + 255) / 256, 256, 0, s>>>(assignment_pos, groups, inv, limit, status);
    int rc = check_launch("rr_scatter_kernel");
    if (rc) return rc;
  }
  const int64_t n = (int64_t)tokens * (hidden / 2);
  const unsigned blocks = (unsigned)((n + 255) / 256);
  if (dtype == 1)
    rr_reduce_kernel<true><<<blocks, 256, 0, s>>>(previous, weighted, inv, tokens, hidden, k, out);
  else
    rr_reduce_kernel<false><<<blocks, 256, 0, s>>>(previous, weighted, inv, tokens, hidden, k, out);
  return check_launch("rr_reduce_kernel");
}

}  // extern "C"
