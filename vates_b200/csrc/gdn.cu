// Gated-DeltaNet recurrent step for decode / MTP verify (T tokens through the
// linear-attention state of one layer).
//
// Reference: the gated-delta kernel of mlx_streaming/core/linear_attn/
// gated_delta_multistate.py:28-130 (vendored from mlx-lm, with a per-step
// state output) and the blocked scan of mlx_streaming/core/attention/
// gdn_fused.py:13-97. Per value head hv (key head hv / (Hv / Hk)), state
// S[dv][dk] in float32, for t = 0..T-1 (a masked step leaves S unchanged and
// writes y = 0):
//   S        = S * g_t                (g per head, or per head and key dim)
//   kv[dv]   = sum_dk S[dv][dk] k_t[dk]
//   delta    = (v_t[dv] - kv[dv]) * beta_t
//   S[dv][:] += k_t[:] * delta
//   y_t[dv]  = bf16(sum_dk S[dv][dk] q_t[dk])
// One CTA of 128 threads owns 16 state rows of one head: 8 threads per row,
// 16 key dims (4 float4) each, reductions over the 8 threads by shuffles.
// The state stays in registers across the T steps; q/k/v/g/beta of all
// steps are staged in shared memory once.
#include "common.cuh"

namespace vb {

constexpr int GDN_DK = 128;
constexpr int GDN_ROWS = 16;          // state rows per CTA
constexpr int GDN_THREADS = GDN_ROWS * 8;
constexpr int GDN_MAX_T = 16;

struct GdnParams {
  const uint16_t *q, *k, *v;
  const float *g, *beta;
  const float *state_in;
  float *state_out, *states_out;
  const uint8_t *mask;
  uint16_t *y;
  const int32_t *in_slot;  // nullable: state_in = state_in + *in_slot * slot_stride
  size_t slot_stride;
  int B, T, Hk, Hv, Dv, g_per_key, slots;
};

__global__ void __launch_bounds__(GDN_THREADS) gdn_step_kernel(GdnParams p) {
  __shared__ float s_k[GDN_MAX_T][GDN_DK];
  __shared__ float s_q[GDN_MAX_T][GDN_DK];
  __shared__ float s_g[GDN_MAX_T][GDN_DK];
  __shared__ float s_v[GDN_MAX_T][GDN_ROWS];
  __shared__ float s_b[GDN_MAX_T];
  __shared__ int s_m[GDN_MAX_T];
  const int tid = threadIdx.x;
  pdl_launch_dependents();
  pdl_wait();
  const int row0 = blockIdx.x * GDN_ROWS, hv = blockIdx.y, b = blockIdx.z;
  const int hk = hv / (p.Hv / p.Hk);
  const int T = p.T;
  for (int i = tid; i < T * GDN_DK; i += GDN_THREADS) {
    const int t = i / GDN_DK, d = i % GDN_DK;
    const size_t kq = (((size_t)b * T + t) * p.Hk + hk) * GDN_DK + d;
    s_k[t][d] = bf2f(p.k[kq]);
    s_q[t][d] = bf2f(p.q[kq]);
    const size_t gi = ((size_t)b * T + t) * p.Hv + hv;
    s_g[t][d] = p.g_per_key ? p.g[gi * GDN_DK + d] : p.g[gi];
  }
  for (int i = tid; i < T * GDN_ROWS; i += GDN_THREADS) {
    const int t = i / GDN_ROWS, r = i % GDN_ROWS;
    s_v[t][r] = bf2f(p.v[(((size_t)b * T + t) * p.Hv + hv) * p.Dv + row0 + r]);
  }
  for (int t = tid; t < T; t += GDN_THREADS) {
    s_b[t] = p.beta[((size_t)b * T + t) * p.Hv + hv];
    s_m[t] = p.mask ? p.mask[(size_t)b * T + t] : 1;
  }
  const int r = tid >> 3, seg = tid & 7, d0 = seg * 16;
  const int dv = row0 + r;
  const size_t srow = (((size_t)b * p.Hv + hv) * p.Dv + dv) * GDN_DK + d0;
  float4 st[4];
  const float *state_in = p.state_in;
  if (p.in_slot) state_in += (size_t)min(max(*p.in_slot, 0), p.slots - 1) * p.slot_stride;
  const float4 *sin = reinterpret_cast<const float4 *>(state_in + srow);
#pragma unroll
  for (int i = 0; i < 4; ++i) st[i] = sin[i];
  __syncthreads();
  for (int t = 0; t < T; ++t) {
    float out = 0.f;
    if (s_m[t]) {
      const float4 *k4 = reinterpret_cast<const float4 *>(&s_k[t][d0]);
      const float4 *q4 = reinterpret_cast<const float4 *>(&s_q[t][d0]);
      const float4 *g4 = reinterpret_cast<const float4 *>(&s_g[t][d0]);
      float mem = 0.f;
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const float4 kf = k4[i], gf = g4[i];
        st[i].x *= gf.x; st[i].y *= gf.y; st[i].z *= gf.z; st[i].w *= gf.w;
        mem = fmaf(st[i].x, kf.x, mem);
        mem = fmaf(st[i].y, kf.y, mem);
        mem = fmaf(st[i].z, kf.z, mem);
        mem = fmaf(st[i].w, kf.w, mem);
      }
      mem += __shfl_xor_sync(0xffffffffu, mem, 4);
      mem += __shfl_xor_sync(0xffffffffu, mem, 2);
      mem += __shfl_xor_sync(0xffffffffu, mem, 1);
      const float delta = (s_v[t][r] - mem) * s_b[t];
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
    }
    if (seg == 0) p.y[(((size_t)b * T + t) * p.Hv + hv) * p.Dv + dv] = f2bf(out);
    if (p.states_out) {
      float4 *so = reinterpret_cast<float4 *>(
          p.states_out + ((((size_t)b * T + t) * p.Hv + hv) * p.Dv + dv) * GDN_DK + d0);
#pragma unroll
      for (int i = 0; i < 4; ++i) so[i] = st[i];
    }
  }
  if (p.state_out) {
    float4 *sout = reinterpret_cast<float4 *>(p.state_out + srow);
#pragma unroll
    for (int i = 0; i < 4; ++i) sout[i] = st[i];
  }
}

}  // namespace vb

using namespace vb;

extern "C" {

int vb_gated_delta_step(const uint16_t *q, const uint16_t *k, const uint16_t *v, const float *g,
                        int32_t g_per_key, const float *beta, const float *state_in,
                        float *state_out, float *states_out, const uint8_t *mask, uint16_t *y,
                        int32_t batch, int32_t tokens, int32_t k_heads, int32_t v_heads,
                        int32_t k_dim, int32_t v_dim, vb_stream_t stream) {
  VB_REQUIRE(batch >= 1 && tokens >= 1 && tokens <= GDN_MAX_T,
             "vb_gated_delta_step: batch=%d tokens=%d (1..%d)", batch, tokens, GDN_MAX_T);
  VB_REQUIRE(k_dim == GDN_DK, "vb_gated_delta_step: key dim %d (128 only)", k_dim);
  VB_REQUIRE(v_dim >= GDN_ROWS && v_dim % GDN_ROWS == 0, "vb_gated_delta_step: value dim %d",
             v_dim);
  VB_REQUIRE(k_heads >= 1 && v_heads >= k_heads && v_heads % k_heads == 0,
             "vb_gated_delta_step: heads k=%d v=%d", k_heads, v_heads);
  VB_REQUIRE(q && k && v && g && beta && state_in && state_out && y,
             "vb_gated_delta_step: null tensor");
  VB_REQUIRE(((uintptr_t)state_in % 16) == 0 && ((uintptr_t)state_out % 16) == 0 &&
                 ((uintptr_t)states_out % 16) == 0,
             "vb_gated_delta_step: state tensors must be 16-byte aligned");
  GdnParams p;
  p.q = q; p.k = k; p.v = v; p.g = g; p.beta = beta;
  p.state_in = state_in; p.state_out = state_out; p.states_out = states_out;
  p.mask = mask; p.y = y;
  p.B = batch; p.T = tokens; p.Hk = k_heads; p.Hv = v_heads; p.Dv = v_dim;
  p.g_per_key = g_per_key ? 1 : 0;
  p.in_slot = nullptr; p.slot_stride = 0; p.slots = 1;
  gdn_step_kernel<<<dim3(v_dim / GDN_ROWS, v_heads, batch), GDN_THREADS, 0, as_stream(stream)>>>(p);
  return check_launch("gdn_step_kernel");
}

int vb_gated_delta_step_at(const uint16_t *q, const uint16_t *k, const uint16_t *v,
                           const float *g, int32_t g_per_key, const float *beta, float *states,
                           int32_t slots, const int32_t *in_slot, const uint8_t *mask,
                           uint16_t *y, int32_t batch, int32_t tokens, int32_t k_heads,
                           int32_t v_heads, int32_t k_dim, int32_t v_dim, vb_stream_t stream) {
  VB_REQUIRE(batch == 1 && tokens >= 1 && tokens <= GDN_MAX_T && tokens <= slots,
             "vb_gated_delta_step_at: batch=%d (1 only) tokens=%d slots=%d", batch, tokens, slots);
  VB_REQUIRE(k_dim == GDN_DK, "vb_gated_delta_step_at: key dim %d (128 only)", k_dim);
  VB_REQUIRE(v_dim >= GDN_ROWS && v_dim % GDN_ROWS == 0, "vb_gated_delta_step_at: value dim %d",
             v_dim);
  VB_REQUIRE(k_heads >= 1 && v_heads >= k_heads && v_heads % k_heads == 0,
             "vb_gated_delta_step_at: heads k=%d v=%d", k_heads, v_heads);
  VB_REQUIRE(q && k && v && g && beta && states && in_slot && y,
             "vb_gated_delta_step_at: null tensor");
  VB_REQUIRE(((uintptr_t)states % 16) == 0, "vb_gated_delta_step_at: states 16-byte aligned");
  GdnParams p;
  p.q = q; p.k = k; p.v = v; p.g = g; p.beta = beta;
  p.state_in = states; p.state_out = nullptr; p.states_out = states;
  p.mask = mask; p.y = y;
  p.B = batch; p.T = tokens; p.Hk = k_heads; p.Hv = v_heads; p.Dv = v_dim;
  p.g_per_key = g_per_key ? 1 : 0;
  p.in_slot = in_slot; p.slot_stride = (size_t)batch * v_heads * v_dim * GDN_DK; p.slots = slots;
  vb_launch(gdn_step_kernel, dim3(v_dim / GDN_ROWS, v_heads, batch), dim3(GDN_THREADS), 0,
            as_stream(stream), false, p);
  return check_launch("gdn_step_kernel");
}

}  // extern "C"
