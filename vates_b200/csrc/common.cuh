// Shared device helpers for the vates_b200 sm_100a kernels.
#pragma once

#include <cuda_runtime.h>
#include <cuda_bf16.h>
#include <stdint.h>

#include <utility>

#include "../../include/vates_b200.h"

namespace vb {

// ----------------------------------------------------------------------------
// Host-side error reporting (abi.cu)
// ----------------------------------------------------------------------------
int set_error(int code, const char *fmt, ...);
int check_launch(const char *what);

#define VB_REQUIRE(cond, ...)                                   \
  do {                                                          \
    if (!(cond)) return ::vb::set_error(VB_ERR_INVALID, __VA_ARGS__); \
  } while (0)

static inline cudaStream_t as_stream(vb_stream_t s) {
  return reinterpret_cast<cudaStream_t>(s);
}

static inline size_t align_up(size_t v, size_t a) { return (v + a - 1) / a * a; }

// ----------------------------------------------------------------------------
// bf16 helpers
// ----------------------------------------------------------------------------
__device__ __forceinline__ float bf2f(uint16_t b) {
  return __uint_as_float(static_cast<uint32_t>(b) << 16);
}
// Round-to-nearest-even float -> bf16 bits (hardware cvt.rn).
__device__ __forceinline__ uint16_t f2bf(float f) {
  return __bfloat16_as_ushort(__float2bfloat16_rn(f));
}
__device__ __forceinline__ float rbf(float f) { return bf2f(f2bf(f)); }

// Pack two floats into a bf16x2 word (lo in bits 0-15), round to nearest
// even: one cvt.rn.bf16x2.f32.
__device__ __forceinline__ uint32_t pack_bf2(float lo, float hi) {
  uint32_t r;
  asm("cvt.rn.bf16x2.f32 %0, %1, %2;" : "=r"(r) : "f"(hi), "f"(lo));
  return r;
}

// MLX sigmoid: y = 1/(1+exp(-|x|)), x<0 -> 1-y (float32).
__device__ __forceinline__ float mlx_sigmoid(float x) {
  float y = 1.0f / (1.0f + expf(-fabsf(x)));
  return x < 0.0f ? 1.0f - y : y;
}

// mlx-lm SwiGLU on bf16 values: bf16(bf16(g*bf16(sigmoid(g)))*u).
__device__ __forceinline__ float swiglu_bf16(float g, float u) {
  float s = rbf(mlx_sigmoid(g));
  float a = rbf(__fmul_rn(g, s));
  return rbf(__fmul_rn(a, u));
}

// ----------------------------------------------------------------------------
// Status word
// ----------------------------------------------------------------------------
__device__ __forceinline__ void flag_status(int32_t *status, int32_t bits) {
  if (status) atomicOr(status, bits);
}

// ----------------------------------------------------------------------------
// Loads
// ----------------------------------------------------------------------------
__device__ __forceinline__ uint2 ldg_nc_v2(const void *p) {
  uint2 r;
  asm volatile("ld.global.nc.L1::no_allocate.v2.u32 {%0,%1}, [%2];"
               : "=r"(r.x), "=r"(r.y) : "l"(p));
  return r;
}
__device__ __forceinline__ uint4 ldg_nc_v4(const void *p) {
  uint4 r;
  asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0,%1,%2,%3}, [%4];"
               : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w) : "l"(p));
  return r;
}
__device__ __forceinline__ uint4 ldg_v4(const void *p) {
  return *reinterpret_cast<const uint4 *>(p);
}
// Asynchronous bulk prefetch of [p, p + bytes) into L2 (TMA unit; p and
// bytes multiples of 16). A hint: it neither blocks nor completes anything.
__device__ __forceinline__ void prefetch_l2_bulk(const void *p, uint32_t bytes) {
  asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(p), "r"(bytes) : "memory");
}
__device__ __forceinline__ void prefetch_l2(const void *p) {
  asm volatile("prefetch.global.L2 [%0];" ::"l"(p));
}

// ----------------------------------------------------------------------------
// Warp-level MMA: D[16x8] += A[16x16] * B[16x8], bf16 in, f32 accumulate.
// Fragment layout (PTX ISA, mma.m16n8k16, g = lane/4, c = lane%4):
//   a[0] = A[g][2c..2c+1]   a[1] = A[g+8][2c..2c+1]
//   a[2] = A[g][2c+8..+9]   a[3] = A[g+8][2c+8..+9]
//   b[0] = B[2c..2c+1][g]   b[1] = B[2c+8..+9][g]
//   d[0..1] = D[g][2c..2c+1]  d[2..3] = D[g+8][2c..2c+1]
// ----------------------------------------------------------------------------
__device__ __forceinline__ void mma_bf16(float (&d)[4], uint32_t a0, uint32_t a1,
                                         uint32_t a2, uint32_t a3, uint32_t b0,
                                         uint32_t b1) {
  asm(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 "
      "{%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};\n"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

// 4-bit code pairs as exact bf16 values (128 + q): nibble i (low half) and
// nibble i+4 (high half) of `w`.
__device__ __forceinline__ uint32_t nib_pair(uint32_t w, int i) {
  return ((w >> (4 * i)) & 0x000F000Fu) | 0x43004300u;
}

// Start of tensor t (gate w,s,b, up w,s,b, down w,s,b) of a pool slot.
__device__ __forceinline__ const uint8_t *pool_ptr(const VbQuantPool &pool, int t, int slot) {
  return (const uint8_t *)pool.ptr[t] + (size_t)slot * pool.slot_stride[t];
}

// (a & m) | o in one LOP3.
__device__ __forceinline__ uint32_t lop_and_or(uint32_t a, uint32_t m, uint32_t o) {
  uint32_t r;
  asm("lop3.b32 %0, %1, %2, %3, 0xEA;" : "=r"(r) : "r"(a), "r"(m), "r"(o));
  return r;
}
// The four code pairs of a 32-bit word of 4-bit codes as exact bf16 pairs
// (128 + q): p[i] holds nibble i (low half) and nibble i+4 (high half).
__device__ __forceinline__ void nib_pairs4(uint32_t w, uint32_t (&p)[4]) {
  constexpr uint32_t M = 0x000F000Fu, O = 0x43004300u;
  p[0] = lop_and_or(w, M, O);
  p[1] = lop_and_or(w >> 4, M, O);
  p[2] = lop_and_or(w >> 8, M, O);
  p[3] = lop_and_or(w >> 12, M, O);
}

__device__ __forceinline__ uint32_t bf16x2_fma(uint32_t a, uint32_t b, uint32_t c) {
  uint32_t d;
  asm("fma.rn.bf16x2 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(c));
  return d;
}

// Dequantized bf16 weights of one word of 4-bit codes (MLX affine format,
// fused_moe.cpp:131-145 qvalue): o[i] holds columns i (low half) and i+4
// (high half) as bf16(q*s + b). (128 + q) - 128 is exact and q*s is exact, so
// the one rounding of fma.rn.bf16x2 gives the float32 value q*s + b rounded
// to bf16 whenever that float32 sum is exact (always for the bias range of a
// quantized group). s2/b2 hold the group's bf16 scale/bias in both halves.
// Every bf16 weight operand of the prefill GEMMs comes from here.
__device__ __forceinline__ void dequant4_bf16x2(uint32_t w, uint32_t s2, uint32_t b2,
                                                uint32_t (&o)[4]) {
  uint32_t pr[4];
  nib_pairs4(w, pr);
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    uint32_t q;
    asm("sub.rn.bf16x2 %0, %1, %2;" : "=r"(q) : "r"(pr[i]), "r"(0x43004300u));
    o[i] = bf16x2_fma(q, s2, b2);
  }
}

// Rotate 8 consecutive dims (two 4x4 blocks) held by one lane.
// out[4b+i] = sum_k x[4b+k] * R[b][k][i] (R rounded to bf16), products and
// sums in float32 in ascending k, then rounded to bf16.
__device__ __forceinline__ void rotate8(float (&v)[8], const float *__restrict__ blocks,
                                        int blk0, bool transpose) {
#pragma unroll
  for (int h = 0; h < 2; ++h) {
    const float *R = blocks + (size_t)(blk0 + h) * 16;
    float x[4] = {v[4 * h], v[4 * h + 1], v[4 * h + 2], v[4 * h + 3]};
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      float acc = 0.f;
#pragma unroll
      for (int kk = 0; kk < 4; ++kk) {
        const float r = rbf(transpose ? __ldg(R + i * 4 + kk) : __ldg(R + kk * 4 + i));
        acc = __fadd_rn(acc, __fmul_rn(x[kk], r));
      }
      v[4 * h + i] = rbf(acc);
    }
  }
}

// Programmatic dependent launch controls (no-ops without the launch
// attribute).
__device__ __forceinline__ void pdl_wait() {
  asm volatile("griddepcontrol.wait;" ::: "memory");
}
__device__ __forceinline__ void pdl_launch_dependents() {
  asm volatile("griddepcontrol.launch_dependents;");
}

// Ampere-style asynchronous 16-byte global -> shared copies.
__device__ __forceinline__ void cp_async16(void *smem, const void *gmem) {
  const uint32_t s = (uint32_t)__cvta_generic_to_shared(smem);
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(s), "l"(gmem) : "memory");
}
__device__ __forceinline__ void cp_async8(void *smem, const void *gmem) {
  const uint32_t s = (uint32_t)__cvta_generic_to_shared(smem);
  asm volatile("cp.async.ca.shared.global [%0], [%1], 8;" ::"r"(s), "l"(gmem) : "memory");
}
__device__ __forceinline__ void cp_async4(void *smem, const void *gmem) {
  const uint32_t s = (uint32_t)__cvta_generic_to_shared(smem);
  asm volatile("cp.async.ca.shared.global [%0], [%1], 4;" ::"r"(s), "l"(gmem) : "memory");
}
__device__ __forceinline__ void cp_async_commit() {
  asm volatile("cp.async.commit_group;" ::: "memory");
}
template <int N>
__device__ __forceinline__ void cp_async_wait() {
  asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}

}  // namespace vb

// Kernel launch with an optional programmatic-dependent-launch attribute.
template <typename... KArgs, typename... Args>
static inline cudaError_t vb_launch(void (*kern)(KArgs...), dim3 grid, dim3 block,
                                    size_t smem, cudaStream_t s, bool pdl, Args &&...args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = pdl ? attr : nullptr;
  cfg.numAttrs = pdl ? 1 : 0;
  return cudaLaunchKernelEx(&cfg, kern, std::forward<Args>(args)...);
}
