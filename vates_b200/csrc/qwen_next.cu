// Qwen3-Next decoder pieces around the MoE block and the IsoQuant attention,
// for decode and speculative (MTP) verify at T <= 8 tokens, and the device
// side of the speculative loop.
//
// References (the model is mlx-lm 0.31.3 models/qwen3_next.py, which the
// reference patches):
// - Gated-DeltaNet input side in verify mode, mtp/kv_cache.py:34-91: the
//   fused projection split per key head (fix_query_key_value_ordering), the
//   depthwise causal conv1d (kernel 4) over [conv state; new rows] with its
//   window after every token kept for the commit, SiLU, q = 128^-1 *
//   rms_norm(q), k = 128^-0.5 * rms_norm(k), beta = sigmoid(b),
//   g = exp(-exp(A_log) * softplus(a + dt_bias)) (gated_delta_multistate.py:
//   201-226 with mlx-lm gated_delta.compute_g); output side: the gated
//   RMSNorm rms_norm(y) * w * silu(z) (kv_cache.py:102).
// - Full attention, core/cache/kv_quant_patch.py:26-71: q_proj split into
//   queries and gate, q_norm / k_norm, RoPE at the cache offset (partial
//   rotary dims, non-traditional), the SO(4) rotation of q, and
//   output * sigmoid(gate) before o_proj; the MTP layer's plain attention
//   (mtp/qwen3_next_mtp.py:40-56) writes k/v into a bf16 cache instead.
// - The speculative loop, mtp/generate.py:338-352 (accept_prefix),
//   818-853 (accepted length, emitted tokens, pending token) and
//   drafter.py:178-186 (MTP cache sync over the accepted pairs).
// Every sequence position (cache offset, accepted count) is read from device
// memory, so a whole decode / verify step is one CUDA graph.
#include "kv_quant.cuh"

namespace vb {

constexpr int QN_MAX_T = 8;

__device__ __forceinline__ float silu_bf16(float x) {
  return rbf(__fmul_rn(x, rbf(mlx_sigmoid(x))));
}

// mx.logaddexp(x, 0) in float32.
__device__ __forceinline__ float softplus_f(float x) {
  return fmaxf(x, 0.f) + log1pf(expf(-fabsf(x)));
}

// ---------------------------------------------------------------------------
// Gated-DeltaNet input side. One CTA per key head, one thread per conv
// channel of the head: q (Dk), k (Dk), then the r = Hv/Hk value heads (r Dv).
// The thread owns its channel's conv rows, so the window can be moved in
// place: it reads rows [off, off+3) of the previous step's buffer (off = the
// accepted count), then writes the window to rows 0..2 and the new inputs to
// rows 3..3+T-1.
// ---------------------------------------------------------------------------
struct GdnPrepParams {
  const uint16_t *proj;
  int stride;
  int T, Hk, Hv, Dk, Dv, max_t;
  uint16_t *conv;
  const int32_t *conv_off;
  const uint16_t *conv_w;
  const float *a_log;
  const uint16_t *dt_bias;
  uint16_t *q, *k, *v;
  float *g, *beta;
  int32_t *status;
};

__global__ void __launch_bounds__(1024) gdn_prepare_kernel(GdnPrepParams p) {
  __shared__ float red[QN_MAX_T][32];
  const int hk = blockIdx.x, tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int r = p.Hv / p.Hk;
  const int W = 2 * p.Dk + 2 * r * p.Dv;
  const int C = 2 * p.Hk * p.Dk + p.Hv * p.Dv;
  const int T = p.T;
  int kind, ch, col, d;
  if (tid < p.Dk) {
    kind = 0; d = tid; ch = hk * p.Dk + d; col = hk * W + d;
  } else if (tid < 2 * p.Dk) {
    kind = 1; d = tid - p.Dk; ch = p.Hk * p.Dk + hk * p.Dk + d; col = hk * W + p.Dk + d;
  } else {
    kind = 2; d = tid - 2 * p.Dk;
    ch = 2 * p.Hk * p.Dk + hk * r * p.Dv + d;
    col = hk * W + 2 * p.Dk + d;
  }
  float cw[4];
#pragma unroll
  for (int j = 0; j < 4; ++j) cw[j] = bf2f(p.conv_w[(size_t)ch * 4 + j]);
  pdl_launch_dependents();
  pdl_wait();
  int off = p.conv_off ? *p.conv_off : 0;
  if (off < 0 || off > p.max_t) {
    if (tid == 0) flag_status(p.status, VB_STATUS_BOUNDS);
    off = 0;
  }
  float win[3 + QN_MAX_T];
#pragma unroll
  for (int i = 0; i < 3; ++i) win[i] = bf2f(p.conv[(size_t)(off + i) * C + ch]);
#pragma unroll
  for (int t = 0; t < QN_MAX_T; ++t)
    win[3 + t] = t < T ? bf2f(p.proj[(size_t)t * p.stride + col]) : 0.f;
#pragma unroll
  for (int i = 0; i < 3 + QN_MAX_T; ++i)
    if (i < 3 + T) p.conv[(size_t)i * C + ch] = f2bf(win[i]);
  float y[QN_MAX_T];
#pragma unroll
  for (int t = 0; t < QN_MAX_T; ++t) {
    float acc = 0.f;
#pragma unroll
    for (int j = 0; j < 4; ++j) acc = fmaf(cw[j], win[t + j], acc);
    y[t] = t < T ? silu_bf16(rbf(acc)) : 0.f;
  }
  // sums of squares of the q and k heads (warps of one kind never mix: Dk is
  // a multiple of 32)
#pragma unroll
  for (int t = 0; t < QN_MAX_T; ++t) {
    float ss = y[t] * y[t];
#pragma unroll
    for (int o = 16; o; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
    if (lane == 0) red[t][warp] = ss;
  }
  __syncthreads();
  if (kind < 2) {
    const int w0 = kind * (p.Dk / 32), nw = p.Dk / 32;
    const float k_scale = rbf(rsqrtf((float)p.Dk));           // bf16(Dk^-0.5)
    const float q_scale = rbf(1.f / (float)p.Dk);              // bf16(Dk^-1)
#pragma unroll
    for (int t = 0; t < QN_MAX_T; ++t) {
      if (t >= T) break;
      float tot = 0.f;
      for (int w = 0; w < nw; ++w) tot += red[t][w0 + w];
      const float inv = rsqrtf(tot / (float)p.Dk + 1e-6f);
      const float nv = rbf(y[t] * inv);
      const size_t o = ((size_t)t * p.Hk + hk) * p.Dk + d;
      if (kind == 0)
        p.q[o] = f2bf(nv * q_scale);
      else
        p.k[o] = f2bf(nv * k_scale);
    }
  } else {
    const int j = d / p.Dv, dd = d % p.Dv, hv = hk * r + j;
#pragma unroll
    for (int t = 0; t < QN_MAX_T; ++t)
      if (t < T) p.v[((size_t)t * p.Hv + hv) * p.Dv + dd] = f2bf(y[t]);
  }
  if (tid < r * T) {
    const int t = tid / r, j = tid % r, hv = hk * r + j;
    const size_t base = (size_t)t * p.stride + (size_t)p.Hk * W + hk * 2 * r;
    const float b = bf2f(p.proj[base + j]);
    const float a = bf2f(p.proj[base + r + j]);
    p.beta[t * p.Hv + hv] = rbf(mlx_sigmoid(b));
    const float ad = rbf(a + bf2f(p.dt_bias[hv]));
    const float sp = rbf(softplus_f(ad));
    p.g[t * p.Hv + hv] = expf(-expf(p.a_log[hv]) * sp);
  }
}

// Gated RMSNorm of the recurrence output: out = silu(z) * (w * rms_norm(y)),
// bf16 at each MLX op. One warp per (token, value head).
__global__ void __launch_bounds__(256) gdn_gated_norm_kernel(
    const uint16_t *__restrict__ y, const uint16_t *__restrict__ proj, int stride, int T,
    int Hk, int Hv, int Dk, int Dv, const uint16_t *__restrict__ w, float eps,
    uint16_t *__restrict__ out) {
  const int row = blockIdx.x * 8 + (threadIdx.x >> 5), lane = threadIdx.x & 31;
  pdl_launch_dependents();
  pdl_wait();
  if (row >= T * Hv) return;
  const int t = row / Hv, hv = row % Hv;
  const int r = Hv / Hk, hk = hv / r, j = hv % r;
  const int W = 2 * Dk + 2 * r * Dv;
  const uint16_t *yr = y + (size_t)row * Dv;
  const uint16_t *zr = proj + (size_t)t * stride + hk * W + 2 * Dk + r * Dv + j * Dv;
  float ss = 0.f;
  for (int d = lane; d < Dv; d += 32) {
    const float v = bf2f(yr[d]);
    ss = fmaf(v, v, ss);
  }
#pragma unroll
  for (int o = 16; o; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
  const float inv = rsqrtf(ss / (float)Dv + eps);
  for (int d = lane; d < Dv; d += 32) {
    const float nv = rbf(rbf(bf2f(yr[d]) * inv) * bf2f(w[d]));
    out[(size_t)row * Dv + d] = f2bf(swiglu_bf16(bf2f(zr[d]), nv));
  }
}

// ---------------------------------------------------------------------------
// Attention input side. One warp per (token, head row) of D = 256 (8 dims per
// lane): rows 0..Hq-1 queries (q_norm, RoPE, optional SO(4) rotation),
// Hq..Hq+Hkv-1 keys (k_norm, RoPE), then values. Queries go to q_out
// [Hq, T, D]; keys and values to [Hkv, T, D] rows (kv_cap = 0) or into bf16
// caches [Hkv, kv_cap, D] at position pos + pos_add + t.
// ---------------------------------------------------------------------------
struct AttnPrepParams {
  const uint16_t *proj;
  int stride, T, Hq, Hkv;
  const uint16_t *qw, *kw;
  float eps;
  int rope_dims;
  float rope_log2_base;
  const int32_t *pos;
  int pos_add;
  const float *rk;
  uint16_t *q_out, *k_out, *v_out;
  int kv_cap;
  int32_t *status;
  // Quantized caches (kc non-null): keys and values are rotated by rk / rv
  // and quantized straight into [Hkv, qcap, ...] at their positions.
  const float *rv;
  uint32_t *kc, *vc;
  uint16_t *ks, *kb, *vs, *vb;
  int kbits, vbits, qcap;
};

__global__ void __launch_bounds__(256) attn_prepare_kernel(AttnPrepParams p) {
  const int wid = blockIdx.x * 8 + (threadIdx.x >> 5), lane = threadIdx.x & 31;
  const int rows = p.Hq + 2 * p.Hkv;
  pdl_launch_dependents();
  pdl_wait();
  if (wid >= p.T * rows) return;
  const int t = wid / rows, h = wid % rows;
  const int kind = h < p.Hq ? 0 : (h < p.Hq + p.Hkv ? 1 : 2);
  const int hh = kind == 0 ? h : (kind == 1 ? h - p.Hq : h - p.Hq - p.Hkv);
  size_t col;
  if (kind == 0) col = (size_t)hh * 512;
  else if (kind == 1) col = (size_t)p.Hq * 512 + hh * 256;
  else col = (size_t)p.Hq * 512 + (size_t)p.Hkv * 256 + hh * 256;
  const uint16_t *src = p.proj + (size_t)t * p.stride + col + lane * 8;
  float v[8];
  {
    const uint4 raw = *reinterpret_cast<const uint4 *>(src);
    const uint32_t w[4] = {raw.x, raw.y, raw.z, raw.w};
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      v[2 * i] = __uint_as_float(w[i] << 16);
      v[2 * i + 1] = __uint_as_float(w[i] & 0xFFFF0000u);
    }
  }
  const int p0 = (p.pos ? *p.pos : 0) + p.pos_add;
  if (kind < 2) {
    float ss = 0.f;
#pragma unroll
    for (int i = 0; i < 8; ++i) ss = fmaf(v[i], v[i], ss);
#pragma unroll
    for (int o = 16; o; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
    const float inv = rsqrtf(ss / 256.f + p.eps);
    const uint16_t *nw = (kind == 0 ? p.qw : p.kw) + lane * 8;
#pragma unroll
    for (int i = 0; i < 8; ++i) v[i] = rbf(rbf(v[i] * inv) * bf2f(nw[i]));
    // RoPE over dims [0, rope_dims): pairs (i, i + rope_dims/2), partner lane
    // lane ^ (rope_dims / 16).
    const int half = p.rope_dims >> 1;
    float pv[8];
#pragma unroll
    for (int i = 0; i < 8; ++i) pv[i] = __shfl_xor_sync(0xffffffffu, v[i], half >> 3);
    const int d0 = lane * 8;
    if (d0 < p.rope_dims) {
      const bool first = d0 < half;
      const float posf = (float)(p0 + t);
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        const int fi = (first ? d0 : d0 - half) + i;
        const float inv_freq = exp2f(-((float)fi / (float)half) * p.rope_log2_base);
        float sn, cs;
        sincosf(posf * inv_freq, &sn, &cs);
        const float x1 = first ? v[i] : pv[i], x2 = first ? pv[i] : v[i];
        v[i] = rbf(first ? (x1 * cs - x2 * sn) : (x1 * sn + x2 * cs));
      }
    }
    if (kind == 0 && p.rk) rotate8(v, p.rk, lane * 2, false);
  }
  if (kind != 0 && p.kc) {
    // IsoQuant append of this key / value row: the bf16 row the unfused path
    // would write (v holds bf16 values), SO(4)-rotated, quantized and packed
    // exactly as vb_kv_quant_append_at does with it.
    const int at = p0 + t;
    if (at < 0 || at >= p.qcap) {
      if (lane == 0) flag_status(p.status, VB_STATUS_BOUNDS);
      return;
    }
    const bool key = kind == 1;
    rotate8(v, key ? p.rk : p.rv, lane * 2, false);
    kv_quant_store<32>(v, lane, 0, key ? p.kbits : p.vbits, true, (int64_t)hh * p.qcap + at,
                       key ? p.kc : p.vc, key ? p.ks : p.vs, key ? p.kb : p.vb);
    return;
  }
  uint4 o;
  o.x = pack_bf2(v[0], v[1]);
  o.y = pack_bf2(v[2], v[3]);
  o.z = pack_bf2(v[4], v[5]);
  o.w = pack_bf2(v[6], v[7]);
  if (kind == 0) {
    *reinterpret_cast<uint4 *>(p.q_out + ((size_t)hh * p.T + t) * 256 + lane * 8) = o;
    return;
  }
  uint16_t *dst = kind == 1 ? p.k_out : p.v_out;
  size_t row;
  if (p.kv_cap > 0) {
    const int at = p0 + t;
    if (at < 0 || at >= p.kv_cap) {
      if (lane == 0) flag_status(p.status, VB_STATUS_BOUNDS);
      return;
    }
    row = (size_t)hh * p.kv_cap + at;
  } else {
    row = (size_t)hh * p.T + t;
  }
  *reinterpret_cast<uint4 *>(dst + row * 256 + lane * 8) = o;
}

// output * sigmoid(gate): o [Hq, T, D] (attention output) -> [T, Hq * D].
__global__ void __launch_bounds__(256) attn_gate_kernel(const uint16_t *__restrict__ o,
                                                        const uint16_t *__restrict__ proj,
                                                        int stride, int T, int Hq,
                                                        uint16_t *__restrict__ out) {
  const int i = blockIdx.x * 256 + threadIdx.x;
  pdl_launch_dependents();
  pdl_wait();
  if (i >= T * Hq * 256) return;
  const int t = i / (Hq * 256), rem = i % (Hq * 256), h = rem >> 8, d = rem & 255;
  const float gv = bf2f(proj[(size_t)t * stride + h * 512 + 256 + d]);
  const float ov = bf2f(o[((size_t)h * T + t) * 256 + d]);
  out[i] = f2bf(ov * rbf(mlx_sigmoid(gv)));
}

// ---------------------------------------------------------------------------
// Speculative loop, device side. State words (int32): [0] pos (main cache
// length), [1] mtp_pos, [2] accepted count of the last verify / prefill
// chunk, [3] accepted - 1 (recurrent state slot), [4] pending token, [5]
// emitted tokens so far, [6] verify steps, [7..7+V] histogram of matched
// drafts. ids[0] is the pending token, ids[1..K] the drafts.
// ---------------------------------------------------------------------------
enum { SP_POS = 0, SP_MTP_POS, SP_ACC, SP_SLOT, SP_PENDING, SP_NOUT, SP_STEPS, SP_HIST };

__global__ void __launch_bounds__(256) spec_accept_kernel(
    int32_t *state, int32_t *ids, const int32_t *preds, int V, int K, int mode,
    const uint16_t *__restrict__ vh, uint16_t *h_last, uint16_t *prev_h, int H,
    int32_t *out_tokens, int out_cap) {
  __shared__ int s_a;
  pdl_launch_dependents();
  pdl_wait();
  if (threadIdx.x == 0) {
    int a, pending;
    if (mode == 1) {  // prefill chunk: every row is committed
      a = V;
      pending = preds[V - 1];
    } else {
      const int n = min(K, V);
      int matched = 0;
      while (matched < n && preds[matched] == ids[1 + matched]) ++matched;
      a = min(matched + 1, V);
      int nout = state[SP_NOUT];
      const int emit = matched < V ? matched + 1 : V;
      for (int i = 0; i < emit; ++i) {
        const int tok = i < matched ? ids[1 + i] : preds[matched];
        if (nout < out_cap) out_tokens[nout] = tok;
        ++nout;
      }
      state[SP_NOUT] = nout;
      pending = matched < V ? preds[matched] : ids[V];
      state[SP_STEPS] += 1;
      state[SP_HIST + min(matched, 7)] += 1;
    }
    state[SP_POS] += a;
    state[SP_ACC] = a;
    state[SP_SLOT] = a - 1;
    state[SP_PENDING] = pending;
    if (mode == 1) ids[0] = pending;
    s_a = a;
  }
  __syncthreads();
  const int a = s_a;
  for (int i = threadIdx.x; i < H; i += 256) {
    prev_h[i] = h_last[i];
    h_last[i] = vh[(size_t)(a - 1) * H + i];
  }
}

// Inputs of the MTP cache sync over the accepted pairs (drafter.py:178-186):
// slot i < a takes token ids[i] and hidden i == 0 ? prev_h : vh[i - 1]; slots
// past a repeat slot a - 1 (their cache rows lie past the new MTP position).
// Then ids[0] = the pending token, the first input of the next drafts.
__global__ void __launch_bounds__(256) spec_sync_inputs_kernel(
    const int32_t *state, int32_t *ids, const uint16_t *__restrict__ vh,
    const uint16_t *__restrict__ prev_h, int V, int H, int32_t *sync_ids,
    uint16_t *sync_h) {
  pdl_launch_dependents();
  pdl_wait();
  const int a = max(1, min(state[SP_ACC], V));
  for (int i = 0; i < V; ++i) {
    const int j = min(i, a - 1);
    if (threadIdx.x == 0) sync_ids[i] = ids[j];
    const uint16_t *src = j == 0 ? prev_h : vh + (size_t)(j - 1) * H;
    for (int e = threadIdx.x; e < H; e += 256) sync_h[(size_t)i * H + e] = src[e];
  }
  __syncthreads();
  if (threadIdx.x == 0) ids[0] = state[SP_PENDING];
}

__global__ void spec_advance_mtp_kernel(int32_t *state) {
  pdl_launch_dependents();
  pdl_wait();
  state[SP_MTP_POS] += state[SP_ACC];
}

// Prompt chunk ids: ids[i] = prompt[pos + i] (i < T).
__global__ void spec_prompt_ids_kernel(const int32_t *state, const int32_t *prompt,
                                       int prompt_len, int T, int32_t *ids) {
  const int i = threadIdx.x;
  pdl_launch_dependents();
  pdl_wait();
  if (i < T) {
    const int at = state[SP_POS] + i;
    ids[i] = at < prompt_len ? prompt[at] : 0;
  }
}

}  // namespace vb

using namespace vb;

extern "C" {

int vb_gdn_prepare(const uint16_t *proj, int32_t proj_stride, int32_t tokens, int32_t k_heads,
                   int32_t v_heads, int32_t head_k, int32_t head_v, uint16_t *conv_buf,
                   int32_t max_tokens, const int32_t *conv_off, const uint16_t *conv_w,
                   const float *a_log, const uint16_t *dt_bias, uint16_t *q, uint16_t *k,
                   uint16_t *v, float *g, float *beta, int32_t *status, vb_stream_t stream) {
  VB_REQUIRE(tokens >= 1 && tokens <= QN_MAX_T && tokens <= max_tokens &&
                 max_tokens <= QN_MAX_T,
             "vb_gdn_prepare: tokens=%d max_tokens=%d (<= %d)", tokens, max_tokens, QN_MAX_T);
  VB_REQUIRE(k_heads >= 1 && v_heads % k_heads == 0 && head_k % 32 == 0 && head_v % 32 == 0,
             "vb_gdn_prepare: heads k=%d v=%d dims %d/%d", k_heads, v_heads, head_k, head_v);
  const int r = v_heads / k_heads;
  const int threads = 2 * head_k + r * head_v;
  VB_REQUIRE(threads <= 1024, "vb_gdn_prepare: %d channels per key head (<= 1024)", threads);
  VB_REQUIRE(proj_stride >= k_heads * (2 * head_k + 2 * r * head_v) + 2 * v_heads,
             "vb_gdn_prepare: projection row of %d elements", proj_stride);
  VB_REQUIRE(proj && conv_buf && conv_w && a_log && dt_bias && q && k && v && g && beta,
             "vb_gdn_prepare: null tensor");
  GdnPrepParams p;
  p.proj = proj; p.stride = proj_stride; p.T = tokens; p.Hk = k_heads; p.Hv = v_heads;
  p.Dk = head_k; p.Dv = head_v; p.max_t = max_tokens; p.conv = conv_buf; p.conv_off = conv_off;
  p.conv_w = conv_w; p.a_log = a_log; p.dt_bias = dt_bias; p.q = q; p.k = k; p.v = v;
  p.g = g; p.beta = beta; p.status = status;
  vb_launch(gdn_prepare_kernel, dim3(k_heads), dim3(threads), 0, as_stream(stream), false, p);
  return check_launch("gdn_prepare_kernel");
}

int vb_gdn_gated_norm(const uint16_t *y, const uint16_t *proj, int32_t proj_stride,
                      int32_t tokens, int32_t k_heads, int32_t v_heads, int32_t head_k,
                      int32_t head_v, const uint16_t *weight, float eps, uint16_t *out,
                      vb_stream_t stream) {
  VB_REQUIRE(tokens >= 1 && k_heads >= 1 && v_heads % k_heads == 0 && eps > 0.f,
             "vb_gdn_gated_norm: tokens=%d heads %d/%d", tokens, k_heads, v_heads);
  VB_REQUIRE(y && proj && weight && out, "vb_gdn_gated_norm: null tensor");
  const int rows = tokens * v_heads;
  vb_launch(gdn_gated_norm_kernel, dim3((rows + 7) / 8), dim3(256), 0, as_stream(stream), false, y,
            proj, (int)proj_stride, (int)tokens, (int)k_heads, (int)v_heads, (int)head_k,
            (int)head_v, weight, eps, out);
  return check_launch("gdn_gated_norm_kernel");
}

int vb_attn_prepare(const uint16_t *proj, int32_t proj_stride, int32_t tokens, int32_t q_heads,
                    int32_t kv_heads, int32_t head_dim, const uint16_t *q_norm_w,
                    const uint16_t *k_norm_w, float eps, int32_t rope_dims, float rope_base,
                    const int32_t *pos, int32_t pos_add, const float *rk_blocks,
                    uint16_t *q_out, uint16_t *k_out, uint16_t *v_out, int32_t kv_cap,
                    int32_t *status, vb_stream_t stream) {
  VB_REQUIRE(head_dim == 256, "vb_attn_prepare: head_dim %d (256 only)", head_dim);
  VB_REQUIRE(tokens >= 1 && q_heads >= 1 && kv_heads >= 1,
             "vb_attn_prepare: tokens=%d heads %d/%d", tokens, q_heads, kv_heads);
  VB_REQUIRE(rope_dims >= 16 && rope_dims <= head_dim && rope_dims % 16 == 0 &&
                 ((rope_dims / 16) & (rope_dims / 16 - 1)) == 0,
             "vb_attn_prepare: rope_dims %d (16 x a power of two)", rope_dims);
  VB_REQUIRE(proj_stride % 8 == 0 && proj_stride >= q_heads * 512 + 2 * kv_heads * 256,
             "vb_attn_prepare: projection row of %d elements", proj_stride);
  VB_REQUIRE(proj && q_norm_w && k_norm_w && q_out && k_out && v_out && eps > 0.f &&
                 rope_base > 1.f,
             "vb_attn_prepare: bad arguments");
  AttnPrepParams p = {};
  p.proj = proj; p.stride = proj_stride; p.T = tokens; p.Hq = q_heads; p.Hkv = kv_heads;
  p.qw = q_norm_w; p.kw = k_norm_w; p.eps = eps; p.rope_dims = rope_dims;
  p.rope_log2_base = log2f(rope_base); p.pos = pos; p.pos_add = pos_add; p.rk = rk_blocks;
  p.q_out = q_out; p.k_out = k_out; p.v_out = v_out; p.kv_cap = kv_cap; p.status = status;
  const int warps = tokens * (q_heads + 2 * kv_heads);
  vb_launch(attn_prepare_kernel, dim3((warps + 7) / 8), dim3(256), 0, as_stream(stream), false, p);
  return check_launch("attn_prepare_kernel");
}

int vb_attn_prepare_quant(const uint16_t *proj, int32_t proj_stride, int32_t tokens,
                          int32_t q_heads, int32_t kv_heads, int32_t head_dim,
                          const uint16_t *q_norm_w, const uint16_t *k_norm_w, float eps,
                          int32_t rope_dims, float rope_base, const int32_t *pos,
                          const float *rk_blocks, const float *rv_blocks, uint16_t *q_out,
                          int32_t cap, int32_t k_bits, uint32_t *k_codes, uint16_t *k_scales,
                          uint16_t *k_biases, int32_t v_bits, uint32_t *v_codes,
                          uint16_t *v_scales, uint16_t *v_biases, int32_t *status,
                          vb_stream_t stream) {
  VB_REQUIRE(head_dim == 256, "vb_attn_prepare_quant: head_dim %d (256 only)", head_dim);
  VB_REQUIRE(tokens >= 1 && q_heads >= 1 && kv_heads >= 1,
             "vb_attn_prepare_quant: tokens=%d heads %d/%d", tokens, q_heads, kv_heads);
  VB_REQUIRE(rope_dims >= 16 && rope_dims <= head_dim && rope_dims % 16 == 0 &&
                 ((rope_dims / 16) & (rope_dims / 16 - 1)) == 0,
             "vb_attn_prepare_quant: rope_dims %d (16 x a power of two)", rope_dims);
  VB_REQUIRE(proj_stride % 8 == 0 && proj_stride >= q_heads * 512 + 2 * kv_heads * 256,
             "vb_attn_prepare_quant: projection row of %d elements", proj_stride);
  auto bits_ok = [](int b) { return b == 2 || b == 3 || b == 4 || b == 5 || b == 6 || b == 8; };
  VB_REQUIRE(bits_ok(k_bits) && bits_ok(v_bits), "vb_attn_prepare_quant: bits %d/%d", k_bits,
             v_bits);
  VB_REQUIRE(proj && q_norm_w && k_norm_w && q_out && pos && rk_blocks && rv_blocks && k_codes &&
                 k_scales && k_biases && v_codes && v_scales && v_biases && cap >= 1 &&
                 eps > 0.f && rope_base > 1.f,
             "vb_attn_prepare_quant: bad arguments");
  AttnPrepParams p = {};
  p.proj = proj; p.stride = proj_stride; p.T = tokens; p.Hq = q_heads; p.Hkv = kv_heads;
  p.qw = q_norm_w; p.kw = k_norm_w; p.eps = eps; p.rope_dims = rope_dims;
  p.rope_log2_base = log2f(rope_base); p.pos = pos; p.pos_add = 0; p.rk = rk_blocks;
  p.q_out = q_out; p.kv_cap = 0; p.status = status;
  p.rv = rv_blocks; p.kc = k_codes; p.ks = k_scales; p.kb = k_biases; p.vc = v_codes;
  p.vs = v_scales; p.vb = v_biases; p.kbits = k_bits; p.vbits = v_bits; p.qcap = cap;
  const int warps = tokens * (q_heads + 2 * kv_heads);
  vb_launch(attn_prepare_kernel, dim3((warps + 7) / 8), dim3(256), 0, as_stream(stream), false, p);
  return check_launch("attn_prepare_kernel");
}

int vb_attn_gate(const uint16_t *attn_out, const uint16_t *proj, int32_t proj_stride,
                 int32_t tokens, int32_t q_heads, uint16_t *out, vb_stream_t stream) {
  VB_REQUIRE(tokens >= 1 && q_heads >= 1, "vb_attn_gate: tokens=%d heads=%d", tokens, q_heads);
  VB_REQUIRE(attn_out && proj && out, "vb_attn_gate: null tensor");
  const int n = tokens * q_heads * 256;
  vb_launch(attn_gate_kernel, dim3((n + 255) / 256), dim3(256), 0, as_stream(stream), false,
            attn_out, proj, (int)proj_stride, (int)tokens, (int)q_heads, out);
  return check_launch("attn_gate_kernel");
}

int vb_spec_accept(int32_t *state, int32_t *ids, const int32_t *preds, int32_t verify_len,
                   int32_t drafts, int32_t mode, const uint16_t *verify_hidden,
                   uint16_t *h_last, uint16_t *prev_h, int32_t hidden, int32_t *out_tokens,
                   int32_t out_cap, vb_stream_t stream) {
  VB_REQUIRE(verify_len >= 1 && verify_len <= QN_MAX_T && drafts >= 0 && (mode == 0 || mode == 1),
             "vb_spec_accept: verify_len=%d drafts=%d mode=%d", verify_len, drafts, mode);
  VB_REQUIRE(mode == 1 || verify_len <= drafts + 1,
             "vb_spec_accept: verify_len %d > drafts + 1", verify_len);
  VB_REQUIRE(state && ids && preds && verify_hidden && h_last && prev_h && hidden > 0,
             "vb_spec_accept: null tensor");
  vb_launch(spec_accept_kernel, dim3(1), dim3(256), 0, as_stream(stream), false, state, ids, preds,
            (int)verify_len, (int)drafts, (int)mode, verify_hidden, h_last, prev_h, (int)hidden,
            out_tokens, (int)out_cap);
  return check_launch("spec_accept_kernel");
}

int vb_spec_sync_inputs(const int32_t *state, int32_t *ids, const uint16_t *verify_hidden,
                        const uint16_t *prev_h, int32_t verify_len, int32_t hidden,
                        int32_t *sync_ids, uint16_t *sync_hidden, vb_stream_t stream) {
  VB_REQUIRE(verify_len >= 1 && verify_len <= QN_MAX_T && hidden > 0,
             "vb_spec_sync_inputs: verify_len=%d", verify_len);
  VB_REQUIRE(state && ids && verify_hidden && prev_h && sync_ids && sync_hidden,
             "vb_spec_sync_inputs: null tensor");
  vb_launch(spec_sync_inputs_kernel, dim3(1), dim3(256), 0, as_stream(stream), false,
            (const int32_t *)state, ids, verify_hidden, prev_h, (int)verify_len, (int)hidden,
            sync_ids, sync_hidden);
  return check_launch("spec_sync_inputs_kernel");
}

int vb_spec_advance_mtp(int32_t *state, vb_stream_t stream) {
  VB_REQUIRE(state, "vb_spec_advance_mtp: null state");
  vb_launch(spec_advance_mtp_kernel, dim3(1), dim3(1), 0, as_stream(stream), false, state);
  return check_launch("spec_advance_mtp_kernel");
}

int vb_spec_prompt_ids(const int32_t *state, const int32_t *prompt, int32_t prompt_len,
                       int32_t tokens, int32_t *ids, vb_stream_t stream) {
  VB_REQUIRE(tokens >= 1 && tokens <= QN_MAX_T && prompt_len >= 0,
             "vb_spec_prompt_ids: tokens=%d", tokens);
  VB_REQUIRE(state && prompt && ids, "vb_spec_prompt_ids: null tensor");
  vb_launch(spec_prompt_ids_kernel, dim3(1), dim3(32), 0, as_stream(stream), false, state, prompt,
            (int)prompt_len, (int)tokens, ids);
  return check_launch("spec_prompt_ids_kernel");
}

}  // extern "C"
