// Float32 fused MoE with the reference native extension's semantics, any bit
// width of the MLX affine format (2/3/4/5/6/8 bits, straddling fields).
//
// Reference: fused_moe_slots_pairs / fused_moe_pairs + reduce_pairs
// (native/ext/compute/fused_moe.cpp:160-298) and _custom_fused_moe_indexed
// (mlx_streaming/core/moe/custom_kernel.py:226-383).
//
//  C1: one warp per (pair, intermediate row): gate and up dot products over
//      the hidden dimension in float32, act = g*(1/(1+exp(-g)))*u.
//  C2: one warp per (token or pair, output row): down dot product over the
//      intermediate dimension; the slots/staged form adds the k routes of a
//      token in rank order weighted by their scores (reduce_pairs order).
#include "common.cuh"

namespace vb {

__device__ __forceinline__ uint32_t field(const uint32_t *__restrict__ row,
                                          int col, int bits, uint32_t mask) {
  const int bit = col * bits;
  const int wi = bit >> 5, sh = bit & 31;
  uint32_t q = __ldg(row + wi) >> sh;
  if (sh + bits > 32) q |= __ldg(row + wi + 1) << (32 - sh);
  return q & mask;
}

struct CompatParams {
  const float *x;              // [rows_x, H]
  const uint32_t *slots;       // [P] or null (pair p -> slot p)
  const uint8_t *active;       // [P] or null
  const float *scores;         // [P] (slots form)
  VbQuantPool pool;
  int P, T, k, H, I, group, bits;
  int x_per_pair;              // 1: x row = pair; 0: x row = pair / k
  float *act;                  // [P, I]
  float *out;                  // slots form: [T, H]; pairs form: [P, H]
  int32_t *status;
};

__device__ __forceinline__ int pair_slot(const CompatParams &p, int pair) {
  int slot = p.slots ? (int)p.slots[pair] : pair;
  if (slot < 0 || slot >= p.pool.cap) {
    flag_status(p.status, VB_STATUS_BOUNDS);
    return -1;
  }
  return slot;
}

__global__ void __launch_bounds__(256) compat_gateup_kernel(CompatParams p) {
  const int pair = blockIdx.x;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int row = blockIdx.y * 8 + warp;
  if (row >= p.I) return;
  float *act = p.act + (size_t)pair * p.I + row;
  if (p.active && !p.active[pair]) {
    if (lane == 0) *act = 0.f;
    return;
  }
  const int slot = pair_slot(p, pair);
  if (slot < 0) {
    if (lane == 0) *act = 0.f;
    return;
  }
  const int words = p.H * p.bits / 32, ngr = p.H / p.group;
  const uint32_t mask = (1u << p.bits) - 1u;
  const uint32_t *gw = (const uint32_t *)((const uint8_t *)p.pool.ptr[0] + (size_t)slot * p.pool.slot_stride[0]) + (size_t)row * words;
  const uint16_t *gs = (const uint16_t *)((const uint8_t *)p.pool.ptr[1] + (size_t)slot * p.pool.slot_stride[1]) + (size_t)row * ngr;
  const uint16_t *gb = (const uint16_t *)((const uint8_t *)p.pool.ptr[2] + (size_t)slot * p.pool.slot_stride[2]) + (size_t)row * ngr;
  const uint32_t *uw = (const uint32_t *)((const uint8_t *)p.pool.ptr[3] + (size_t)slot * p.pool.slot_stride[3]) + (size_t)row * words;
  const uint16_t *us = (const uint16_t *)((const uint8_t *)p.pool.ptr[4] + (size_t)slot * p.pool.slot_stride[4]) + (size_t)row * ngr;
  const uint16_t *ub = (const uint16_t *)((const uint8_t *)p.pool.ptr[5] + (size_t)slot * p.pool.slot_stride[5]) + (size_t)row * ngr;
  const float *x = p.x + (size_t)(p.x_per_pair ? pair : pair / p.k) * p.H;
  float ga = 0.f, ua = 0.f;
  for (int col = lane; col < p.H; col += 32) {
    const int gi = col / p.group;
    const float xv = x[col];
    const float wgv = fmaf((float)field(gw, col, p.bits, mask), bf2f(__ldg(gs + gi)), bf2f(__ldg(gb + gi)));
    const float wuv = fmaf((float)field(uw, col, p.bits, mask), bf2f(__ldg(us + gi)), bf2f(__ldg(ub + gi)));
    ga = fmaf(wgv, xv, ga);
    ua = fmaf(wuv, xv, ua);
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    ga += __shfl_xor_sync(0xffffffffu, ga, o);
    ua += __shfl_xor_sync(0xffffffffu, ua, o);
  }
  if (lane == 0) *act = ga * (1.0f / (1.0f + expf(-ga))) * ua;
}

__device__ __forceinline__ float down_dot(const CompatParams &p, int slot,
                                          int row, const float *act, int lane) {
  const int words = p.I * p.bits / 32, ngr = p.I / p.group;
  const uint32_t mask = (1u << p.bits) - 1u;
  const uint32_t *dw = (const uint32_t *)((const uint8_t *)p.pool.ptr[6] + (size_t)slot * p.pool.slot_stride[6]) + (size_t)row * words;
  const uint16_t *ds = (const uint16_t *)((const uint8_t *)p.pool.ptr[7] + (size_t)slot * p.pool.slot_stride[7]) + (size_t)row * ngr;
  const uint16_t *db = (const uint16_t *)((const uint8_t *)p.pool.ptr[8] + (size_t)slot * p.pool.slot_stride[8]) + (size_t)row * ngr;
  float a = 0.f;
  for (int col = lane; col < p.I; col += 32) {
    const int gi = col / p.group;
    const float w = fmaf((float)field(dw, col, p.bits, mask), bf2f(__ldg(ds + gi)), bf2f(__ldg(db + gi)));
    a = fmaf(w, __ldcg(act + col), a);
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) a += __shfl_xor_sync(0xffffffffu, a, o);
  return a;
}

// Slots/staged form: out[t, row] = sum_j y[t*k+j, row] * scores[t*k+j].
__global__ void __launch_bounds__(256) compat_down_reduce_kernel(CompatParams p) {
  const int t = blockIdx.x;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int row = blockIdx.y * 8 + warp;
  if (row >= p.H) return;
  float acc = 0.f;
  for (int j = 0; j < p.k; ++j) {
    const int pair = t * p.k + j;
    const int slot = pair_slot(p, pair);
    float y = 0.f;
    if (slot >= 0) y = down_dot(p, slot, row, p.act + (size_t)pair * p.I, lane);
    acc = fmaf(y, p.scores[pair], acc);
  }
  if (lane == 0) p.out[(size_t)t * p.H + row] = acc;
}

// Pairs form: y[pair, row] (zero rows for inactive pairs).
__global__ void __launch_bounds__(256) compat_down_pairs_kernel(CompatParams p) {
  const int pair = blockIdx.x;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int row = blockIdx.y * 8 + warp;
  if (row >= p.H) return;
  float y = 0.f;
  if (!(p.active && !p.active[pair])) {
    const int slot = pair_slot(p, pair);
    if (slot >= 0) y = down_dot(p, slot, row, p.act + (size_t)pair * p.I, lane);
  }
  if (lane == 0) p.out[(size_t)pair * p.H + row] = y;
}

static int check_dims(int H, int I, int group, int bits) {
  VB_REQUIRE(bits == 2 || bits == 3 || bits == 4 || bits == 5 || bits == 6 || bits == 8,
             "fused_moe: bits=%d unsupported", bits);
  VB_REQUIRE(group == 32 || group == 64 || group == 128, "fused_moe: group=%d", group);
  VB_REQUIRE(H > 0 && I > 0 && H % group == 0 && I % group == 0,
             "fused_moe: hidden=%d inter=%d not multiples of group %d", H, I, group);
  VB_REQUIRE((H * bits) % 32 == 0 && (I * bits) % 32 == 0,
             "fused_moe: (hidden*bits)%%32 and (inter*bits)%%32 must be 0");
  return VB_OK;
}

}  // namespace vb

using namespace vb;

extern "C" {

size_t vb_fused_moe_workspace_size(int32_t pairs, int32_t inter) {
  if (pairs <= 0 || inter <= 0) return 0;
  return align_up((size_t)pairs * inter * sizeof(float), 256);
}

int vb_fused_moe_slots(const float *x, const uint32_t *local_slots,
                       const float *scores, const VbQuantPool *pool,
                       int32_t tokens, int32_t k, int32_t hidden,
                       int32_t inter, int32_t group, int32_t bits, float *out,
                       int32_t *status, void *workspace, size_t workspace_bytes,
                       vb_stream_t stream) {
  int rc = check_dims(hidden, inter, group, bits);
  if (rc) return rc;
  VB_REQUIRE(tokens > 0 && k > 0, "vb_fused_moe_slots: tokens=%d k=%d", tokens, k);
  VB_REQUIRE(x && scores && pool && out, "vb_fused_moe_slots: null pointer");
  const int P = tokens * k;
  VB_REQUIRE(workspace && workspace_bytes >= vb_fused_moe_workspace_size(P, inter),
             "vb_fused_moe_slots: workspace too small");
  CompatParams p;
  p.x = x; p.slots = local_slots; p.active = nullptr; p.scores = scores;
  p.pool = *pool; p.P = P; p.T = tokens; p.k = k; p.H = hidden; p.I = inter;
  p.group = group; p.bits = bits; p.x_per_pair = 0;
  p.act = static_cast<float *>(workspace); p.out = out; p.status = status;
  cudaStream_t s = as_stream(stream);
  compat_gateup_kernel<<<dim3(P, (inter + 7) / 8), 256, 0, s>>>(p);
  rc = check_launch("compat_gateup_kernel");
  if (rc) return rc;
  compat_down_reduce_kernel<<<dim3(tokens, (hidden + 7) / 8), 256, 0, s>>>(p);
  return check_launch("compat_down_reduce_kernel");
}

int vb_fused_moe_pairs(const float *x, const uint32_t *indices,
                       const uint8_t *active_mask, const VbQuantPool *pool,
                       int32_t pairs, int32_t hidden, int32_t inter,
                       int32_t group, int32_t bits, float *y, int32_t *status,
                       void *workspace, size_t workspace_bytes,
                       vb_stream_t stream) {
  int rc = check_dims(hidden, inter, group, bits);
  if (rc) return rc;
  VB_REQUIRE(pairs > 0 && x && indices && pool && y, "vb_fused_moe_pairs: bad args");
  VB_REQUIRE(workspace && workspace_bytes >= vb_fused_moe_workspace_size(pairs, inter),
             "vb_fused_moe_pairs: workspace too small");
  CompatParams p;
  p.x = x; p.slots = indices; p.active = active_mask; p.scores = nullptr;
  p.pool = *pool; p.P = pairs; p.T = pairs; p.k = 1; p.H = hidden; p.I = inter;
  p.group = group; p.bits = bits; p.x_per_pair = 1;
  p.act = static_cast<float *>(workspace); p.out = y; p.status = status;
  cudaStream_t s = as_stream(stream);
  compat_gateup_kernel<<<dim3(pairs, (inter + 7) / 8), 256, 0, s>>>(p);
  rc = check_launch("compat_gateup_kernel");
  if (rc) return rc;
  compat_down_pairs_kernel<<<dim3(pairs, (hidden + 7) / 8), 256, 0, s>>>(p);
  return check_launch("compat_down_pairs_kernel");
}

}  // extern "C"
