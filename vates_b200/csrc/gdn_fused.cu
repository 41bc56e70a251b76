// Gated-DeltaNet layer core in one launch: conv1d + SiLU + q/k RMS scaling +
// beta/g (vb_gdn_prepare), the recurrence with per-row state checkpoints
// (vb_gated_delta_step_at) and the gated RMSNorm (vb_gdn_gated_norm).
//
// Reference: the verify-mode GDN layer, mlx_streaming/mtp/kv_cache.py:34-103
// (conv window checkpoints, q = Dk^-1 rms_norm(q), k = Dk^-0.5 rms_norm(k),
// gated_delta_update_multistate, norm(out, z)); gated_delta_multistate.py:
// 28-130 for the recurrence.
//
// One thread-block cluster per key head: its 8 CTAs are the r = Hv/Hk value
// heads x 4 blocks of 32 state rows (r = 2, Dv = 128). Every CTA recomputes
// the head's q/k conv outputs and norms (256 channels, T <= 8 rows) and its
// own 32 v channels, so the recurrence needs nothing from the others. Two
// cluster barriers replace the kernel boundaries:
// - after every CTA has read the conv window, the owners move it (q/k
//   channels: cluster rank 0; v channels: their CTA) - the window is read by
//   eight CTAs and rewritten in place;
// - the gated RMSNorm of a value head needs all 128 dims of y: each CTA
//   publishes its 32 y values per row in shared memory and reads its head's
//   four blocks through distributed shared memory, summing the squares in
//   the same lane order as the one-kernel-per-step path (dims l, l+32, l+64,
//   l+96), so the output is bit-identical to the three-kernel sequence.
#include <cooperative_groups.h>

#include "common.cuh"

namespace cg = cooperative_groups;

namespace vb {

constexpr int GF_T = 8;        // max rows (tokens) per call
constexpr int GF_R = 32;       // state rows per CTA
constexpr int GF_DK = 128;
constexpr int GF_THREADS = 256;

__device__ __forceinline__ float gf_silu_bf16(float x) {
  return rbf(__fmul_rn(x, rbf(mlx_sigmoid(x))));
}

__device__ __forceinline__ float gf_softplus(float x) {
  return fmaxf(x, 0.f) + log1pf(expf(-fabsf(x)));
}

struct GdnFusedParams {
  const uint16_t *proj;
  int stride, T, Hk, Hv, Dv, max_t, slots;
  uint16_t *conv;              // [3 + max_t, C]
  const int32_t *conv_off;     // accepted rows of the previous step
  const int32_t *in_slot;      // accepted rows - 1
  const uint16_t *conv_w;      // [C, 4]
  const float *a_log;
  const uint16_t *dt_bias;
  float *states;               // [slots, Hv, Dv, Dk]
  const uint16_t *norm_w;      // [Dv]
  float eps;
  uint16_t *out;               // [T, Hv * Dv]
  int32_t *status;
};

__global__ void __launch_bounds__(GF_THREADS) gdn_fused_kernel(GdnFusedParams p) {
  __shared__ float s_q[GF_T][GF_DK];
  __shared__ float s_k[GF_T][GF_DK];
  __shared__ float s_v[GF_T][GF_R];
  __shared__ float s_y[GF_T][GF_R];
  __shared__ float s_g[GF_T], s_b[GF_T];
  __shared__ float red[GF_T][8];
  cg::cluster_group cluster = cg::this_cluster();
  const int rank = (int)cluster.block_rank();
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int r = p.Hv / p.Hk, blocks_per_head = p.Dv / GF_R;
  const int hk = blockIdx.x / (r * blocks_per_head);
  const int j = rank / blocks_per_head, rb = rank % blocks_per_head;
  const int hv = hk * r + j, row0 = rb * GF_R;
  const int T = p.T, Dk = GF_DK;
  const int W = 2 * Dk + 2 * r * p.Dv;
  const int C = 2 * p.Hk * Dk + p.Hv * p.Dv;

  // 0. this thread's 16 floats of the start state (rows row0..row0+31 of
  //    value head hv, 8 threads per row), in flight during the conv work
  const int rr = tid >> 3, seg = tid & 7, d0 = seg * 16;
  const int dv = row0 + rr;
  const size_t slot_stride = (size_t)p.Hv * p.Dv * Dk;
  const size_t srow = ((size_t)hv * p.Dv + dv) * Dk + d0;
  const int slot = p.in_slot ? min(max(*p.in_slot, 0), p.slots - 1) : 0;
  float4 st[4];
  {
    const float4 *sin = reinterpret_cast<const float4 *>(p.states + slot * slot_stride + srow);
#pragma unroll
    for (int i = 0; i < 4; ++i) st[i] = sin[i];
  }

  // 1. channels: thread tid -> q (tid < 128) or k channel of key head hk;
  //    threads < 32 also the v channel row0 + tid of value head hv
  const int kind = tid < Dk ? 0 : 1, d = tid & (Dk - 1);
  const int ch = kind == 0 ? hk * Dk + d : p.Hk * Dk + hk * Dk + d;
  const int col = hk * W + kind * Dk + d;
  const bool has_v = tid < GF_R;
  const int vch = 2 * p.Hk * Dk + hv * p.Dv + row0 + tid;
  const int vcol = hk * W + 2 * Dk + j * p.Dv + row0 + tid;
  float cw[4], vw[4];
#pragma unroll
  for (int q = 0; q < 4; ++q) {
    cw[q] = bf2f(p.conv_w[(size_t)ch * 4 + q]);
    vw[q] = has_v ? bf2f(p.conv_w[(size_t)vch * 4 + q]) : 0.f;
  }
  int off = p.conv_off ? *p.conv_off : 0;
  if (off < 0 || off > p.max_t) {
    if (tid == 0 && rank == 0) flag_status(p.status, VB_STATUS_BOUNDS);
    off = 0;
  }
  float win[3 + GF_T], vwin[3 + GF_T];
#pragma unroll
  for (int i = 0; i < 3; ++i) {
    win[i] = bf2f(p.conv[(size_t)(off + i) * C + ch]);
    vwin[i] = has_v ? bf2f(p.conv[(size_t)(off + i) * C + vch]) : 0.f;
  }
#pragma unroll
  for (int t = 0; t < GF_T; ++t) {
    win[3 + t] = t < T ? bf2f(p.proj[(size_t)t * p.stride + col]) : 0.f;
    vwin[3 + t] = (t < T && has_v) ? bf2f(p.proj[(size_t)t * p.stride + vcol]) : 0.f;
  }
  // 2. conv + SiLU (fp32 fma in tap order, bf16 at the conv output and in SiLU)
  float y[GF_T], yv[GF_T];
#pragma unroll
  for (int t = 0; t < GF_T; ++t) {
    float acc = 0.f, av = 0.f;
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      acc = fmaf(cw[q], win[t + q], acc);
      av = fmaf(vw[q], vwin[t + q], av);
    }
    y[t] = t < T ? gf_silu_bf16(rbf(acc)) : 0.f;
    yv[t] = (t < T && has_v) ? gf_silu_bf16(rbf(av)) : 0.f;
  }
  // 3. q/k RMS scaling (warps 0-3: q, 4-7: k; sums added in warp order)
#pragma unroll
  for (int t = 0; t < GF_T; ++t) {
    float ss = y[t] * y[t];
#pragma unroll
    for (int o = 16; o; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
    if (lane == 0) red[t][warp] = ss;
  }
  if (tid < T) {   // beta and g of value head hv
    const int t = tid;
    const size_t base = (size_t)t * p.stride + (size_t)p.Hk * W + hk * 2 * r;
    const float b = bf2f(p.proj[base + j]);
    const float a = bf2f(p.proj[base + r + j]);
    s_b[t] = rbf(mlx_sigmoid(b));
    const float ad = rbf(a + bf2f(p.dt_bias[hv]));
    const float sp = rbf(gf_softplus(ad));
    s_g[t] = expf(-expf(p.a_log[hv]) * sp);
  }
  __syncthreads();
  {
    const int w0 = kind * (Dk / 32), nw = Dk / 32;
    const float k_scale = rbf(rsqrtf((float)Dk));
    const float q_scale = rbf(1.f / (float)Dk);
    // (loops over the fixed row bound, so y and yv stay in registers)
#pragma unroll
    for (int t = 0; t < GF_T; ++t) {
      if (t < T) {
        float tot = 0.f;
        for (int w = 0; w < nw; ++w) tot += red[t][w0 + w];
        const float inv = rsqrtf(tot / (float)Dk + 1e-6f);
        const float nv = rbf(y[t] * inv);
        if (kind == 0)
          s_q[t][d] = rbf(nv * q_scale);
        else
          s_k[t][d] = rbf(nv * k_scale);
        if (has_v) s_v[t][tid] = yv[t];
      }
    }
  }
  // 4. every CTA has read the window: move it (owners only)
  cluster.sync();
#pragma unroll
  for (int i = 0; i < 3 + GF_T; ++i) {
    if (i < 3 + T) {
      if (rank == 0) p.conv[(size_t)i * C + ch] = f2bf(win[i]);
      if (has_v) p.conv[(size_t)i * C + vch] = f2bf(vwin[i]);
    }
  }

  // 5. recurrence on rows row0..row0+31 of value head hv (8 threads per row,
  //    16 key dims each; start state loaded at entry), the state after row t
  //    checkpointed in slot t
  for (int t = 0; t < T; ++t) {
    const float4 *k4 = reinterpret_cast<const float4 *>(&s_k[t][d0]);
    const float4 *q4 = reinterpret_cast<const float4 *>(&s_q[t][d0]);
    const float g = s_g[t];
    float mem = 0.f;
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const float4 kf = k4[i];
      st[i].x *= g; st[i].y *= g; st[i].z *= g; st[i].w *= g;
      mem = fmaf(st[i].x, kf.x, mem);
      mem = fmaf(st[i].y, kf.y, mem);
      mem = fmaf(st[i].z, kf.z, mem);
      mem = fmaf(st[i].w, kf.w, mem);
    }
    mem += __shfl_xor_sync(0xffffffffu, mem, 4);
    mem += __shfl_xor_sync(0xffffffffu, mem, 2);
    mem += __shfl_xor_sync(0xffffffffu, mem, 1);
    const float delta = (s_v[t][rr] - mem) * s_b[t];
    float out = 0.f;
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const float4 kf = k4[i], qf = q4[i];
      st[i].x = fmaf(kf.x, delta, st[i].x);
      st[i].y = fmaf(kf.y, delta, st[i].y);
      st[i].z = fmaf(kf.z, delta, st[i].z);
      st[i].w = fmaf(kf.w, delta, st[i].w);
      out = fmaf(st[i].x, qf.x, out);
      out = fmaf(st[i].y, qf.y, out);
      out = fmaf(st[i].z, qf.z, out);
      out = fmaf(st[i].w, qf.w, out);
    }
    out += __shfl_xor_sync(0xffffffffu, out, 4);
    out += __shfl_xor_sync(0xffffffffu, out, 2);
    out += __shfl_xor_sync(0xffffffffu, out, 1);
    if (seg == 0) s_y[t][rr] = rbf(out);
    float4 *so = reinterpret_cast<float4 *>(p.states + (size_t)t * slot_stride + srow);
#pragma unroll
    for (int i = 0; i < 4; ++i) so[i] = st[i];
  }
  // 6. gated RMSNorm: the head's four row blocks through distributed shared
  //    memory, squares summed in the lane order of the per-row kernel
  cluster.sync();
  if (warp < T) {
    const int t = warp;
    float ss = 0.f;
    for (int q = 0; q < blocks_per_head; ++q) {
      const float *yq = cluster.map_shared_rank(&s_y[t][lane], j * blocks_per_head + q);
      const float v = *yq;
      ss = fmaf(v, v, ss);
    }
#pragma unroll
    for (int o = 16; o; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
    const float inv = rsqrtf(ss / (float)p.Dv + p.eps);
    const int dd = row0 + lane;
    const float nv = rbf(rbf(s_y[t][lane] * inv) * bf2f(p.norm_w[dd]));
    const float z = bf2f(p.proj[(size_t)t * p.stride + hk * W + 2 * Dk + r * p.Dv + j * p.Dv + dd]);
    p.out[((size_t)t * p.Hv + hv) * p.Dv + dd] = f2bf(swiglu_bf16(z, nv));
  }
  cluster.sync();  // no CTA leaves while another reads its shared memory
}

}  // namespace vb

using namespace vb;

extern "C" {

int vb_gdn_fused(const uint16_t *proj, int32_t proj_stride, int32_t tokens, int32_t k_heads,
                 int32_t v_heads, int32_t head_k, int32_t head_v, uint16_t *conv_buf,
                 int32_t max_tokens, const int32_t *conv_off, const uint16_t *conv_w,
                 const float *a_log, const uint16_t *dt_bias, float *states, int32_t slots,
                 const int32_t *in_slot, const uint16_t *norm_w, float eps, uint16_t *out,
                 int32_t *status, vb_stream_t stream) {
  VB_REQUIRE(tokens >= 1 && tokens <= GF_T && tokens <= max_tokens && max_tokens <= GF_T &&
                 tokens <= slots,
             "vb_gdn_fused: tokens=%d max_tokens=%d slots=%d", tokens, max_tokens, slots);
  VB_REQUIRE(head_k == GF_DK && head_v % GF_R == 0, "vb_gdn_fused: head dims %d/%d", head_k,
             head_v);
  VB_REQUIRE(k_heads >= 1 && v_heads % k_heads == 0, "vb_gdn_fused: heads %d/%d", k_heads,
             v_heads);
  const int r = v_heads / k_heads, bph = head_v / GF_R;
  VB_REQUIRE(r * bph <= 8, "vb_gdn_fused: %d CTAs per key head (cluster of at most 8)", r * bph);
  VB_REQUIRE(proj_stride >= k_heads * (2 * head_k + 2 * r * head_v) + 2 * v_heads,
             "vb_gdn_fused: projection row of %d elements", proj_stride);
  VB_REQUIRE(proj && conv_buf && conv_w && a_log && dt_bias && states && norm_w && out && eps > 0.f,
             "vb_gdn_fused: null tensor");
  VB_REQUIRE(((uintptr_t)states % 16) == 0, "vb_gdn_fused: states 16-byte aligned");
  GdnFusedParams p;
  p.proj = proj; p.stride = proj_stride; p.T = tokens; p.Hk = k_heads; p.Hv = v_heads;
  p.Dv = head_v; p.max_t = max_tokens; p.slots = slots; p.conv = conv_buf;
  p.conv_off = conv_off; p.in_slot = in_slot; p.conv_w = conv_w; p.a_log = a_log;
  p.dt_bias = dt_bias; p.states = states; p.norm_w = norm_w; p.eps = eps; p.out = out;
  p.status = status;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(k_heads * r * bph);
  cfg.blockDim = dim3(GF_THREADS);
  cfg.stream = as_stream(stream);
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = r * bph;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  cudaLaunchKernelEx(&cfg, gdn_fused_kernel, p);
  return check_launch("gdn_fused_kernel");
}

}  // extern "C"
