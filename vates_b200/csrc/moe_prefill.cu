// Expert-major prefill of one sparse-MoE block on the 5th-generation tensor
// cores (tcgen05), MLX bf16 dtype chain.
//
// Reference: FileStreamingMoeBlock.__call__ prefill branch (mlx_streaming/
// core/moe/block.py:318-347) -> _expert_major_forward (block.py:111-243):
// histogram of routes, expert-ordered assignment list, groups of <= 128
// experts and <= 32768 assignments, per group gather -> gate/up -> SwiGLU ->
// down (gather_qmm, compute.py:156-199) -> y * score -> canonical route-rank
// reduce (deterministic_route_reduce, custom_kernel.py:20-118); then
// + sigmoid(x.w_sg) * shared_expert(x) (block.py:102-109, 345-346).
//
// B200 design (one call, all on the device, no host round trip):
//  P1 router GEMM (tcgen05, bf16 operands by TMA): logits of the E router
//     rows plus the shared-expert gate row, + bias, rounded to bf16.
//  P2 softmax (precise) + top-k + renormalisation per token (one warp per
//     token), route histogram, shared gate sigmoid.
//  P3 plan (one CTA): expert offsets, the reference's group of every expert
//     (the add order of the final reduce), and the list of 128-row tiles.
//     The shared expert is expert E and takes every token.
//  P4 sort: every route gets a row of the expert-sorted order (its token
//     row, its score, route <-> row maps); no rows are copied.
//  P5 grouped GEMM gate/up: dequantized 4-bit tiles (bf16, exact q*s+b
//     rounded once) x the routes' token rows, which two warps of the GEMM
//     copy straight from x into the swizzled A tiles (cp.async); fp32
//     accumulation in TMEM; epilogue bf16(gate), bf16(up), SwiGLU (bf16 per
//     op) -> h rows.
//  P6 grouped GEMM down: h rows x dequantized down tiles; epilogue
//     bf16(bf16(y) * score).
//  P7 combine: per token, the routed rows are added starting from zero in
//     the reference's order (group of the expert, then route rank) with a
//     bf16 rounding after every add, then + bf16(bf16(sigmoid) * shared).
//
// Code permutation: a packed 32-bit word holds codes 8w..8w+7 (LSB first).
// One LOP3 turns nibbles (i, i+4) into the bf16 pair (128+q_i, 128+q_{i+4}).
// Gate/up B tiles are put back into column order (their A rows are x rows
// as stored); down B tiles keep, inside every 8-column block, the order
// (0,4,1,5,2,6,3,7), and the gate/up epilogue writes the h rows (the down A
// operand) in that order too, which leaves every dot product unchanged.
//
// GEMM kernel (one persistent CTA per SM, 20 warps): warp 0 issues TMA loads
// (A tile 128x64 bf16 with the 128-byte swizzle, packed B 256 rows x 32 B),
// warps 2-3 (gate/up) copy the A rows from x instead, warp 1 issues
// tcgen05.mma (M=128, N=256, K=16 steps) into one of two TMEM accumulators,
// warps 4-11 dequantize B into the swizzled bf16 layout, and warps 12-19
// drain TMEM through the epilogue. Every mbarrier wait is
// bounded; on a timeout the kernel raises VB_STATUS_TIMEOUT, winds down and
// frees its TMEM.
#include <algorithm>
#include <mutex>
#include <vector>

#include "common.cuh"
#include "tc100.cuh"

namespace vb {

constexpr int PF_BM = 128;
constexpr int PF_BN = 256;
constexpr int PF_BK = 64;
constexpr int PF_STAGES_MAX = 4;
constexpr int PF_THREADS = 640;  // 20 warps
constexpr int PF_A_BYTES = PF_BM * PF_BK * 2;        // 16 KB
constexpr int PF_B_BYTES = PF_BN * PF_BK * 2;        // 32 KB
constexpr int PF_P_BYTES = PF_BN * PF_BK / 2;        // 8 KB packed codes
constexpr int PF_STAGE_BYTES = PF_A_BYTES + PF_B_BYTES + PF_P_BYTES;
// Epilogue staging for TMA stores (down): per epilogue warp one 32-row x 32-column
// bf16 chunks (64-byte rows, 64-byte swizzle).
constexpr int PF_OUT_CHUNK = 32 * 64;
constexpr uint64_t PF_WAIT_NS = 2000000000ull;       // 2 s per wait

enum PfMode : int { PF_GATEUP = 0, PF_DOWN = 1, PF_ROUTER = 2 };

// Shared memory per mode:
//  gate/up: 4 stages of (A, B, packed codes); h rows stored directly;
//  down:    4 stages of (A, B), the packed codes of dequantized tiles in a
//           2-slot ring of their own, one 32x32 output staging chunk per
//           epilogue warp (TMA stores);
//  router:  4 stages of (A, B); its rows are stored directly (no packed
//           codes, no staging).
constexpr int pf_stages(int mode) { return 4; }
constexpr bool pf_pring(int mode) { return mode == PF_DOWN; }
constexpr int pf_stage_bytes(int mode) {
  return pf_pring(mode) || mode == PF_ROUTER ? PF_A_BYTES + PF_B_BYTES : PF_STAGE_BYTES;
}
constexpr int pf_out_bufs(int mode) { return mode == PF_DOWN ? 1 : 0; }
constexpr int pf_smem(int mode) {
  return pf_stages(mode) * pf_stage_bytes(mode) + (pf_pring(mode) ? 2 * PF_P_BYTES : 0) +
         8 * pf_out_bufs(mode) * PF_OUT_CHUNK + 1024;  // + alignment slack
}
static_assert(pf_smem(PF_GATEUP) <= 232448 - 256 && pf_smem(PF_DOWN) <= 232448 - 256 &&
                  pf_smem(PF_ROUTER) <= 232448 - 256,
              "pf_gemm_kernel shared memory");

struct PfGemmParams {
  int mode;
  int K;            // reduction length
  int nt;           // N tiles
  int gshift;       // log2(group / 64)
  int shared_e;     // expert index of the shared expert (-1: none)
  int n_valid;      // router: valid output columns
  int tail_n;       // router: columns of the last N tile when narrower than PF_BN (0: none)
  const int32_t *mtiles;   // [n] (expert, row0, rows)
  const int32_t *n_mtiles;
  const int32_t *slot_of;  // expert -> pool slot
  const int32_t *heavy_of; // expert -> index of its pre-dequantized bf16 copy, or -1
  VbQuantPool pool, shared;
  uint16_t *out;    // output rows (bf16)
  int out_ld;
  const float *row_score;  // down: per sorted row
  const uint16_t *x;       // gate/up: token rows [*, K]
  const int32_t *tok_of;   // gate/up: row of x behind each sorted row
  const float *bias;       // router: per column (nullable)
  int32_t *status;
};

// Swizzled byte offset of 16-byte chunk `c` of row `r` in a K-major
// 128-byte-swizzled tile.
__device__ __forceinline__ uint32_t sw128(int r, int c) {
  return (uint32_t)((r >> 3) * 1024 + (r & 7) * 128 + ((c ^ (r & 7)) << 4));
}

// (bf16(hi) << 16) | bf16(lo), round to nearest even.
__device__ __forceinline__ uint32_t cvt_bf16x2(float lo, float hi) {
  uint32_t r;
  asm("cvt.rn.bf16x2.f32 %0, %1, %2;" : "=r"(r) : "f"(hi), "f"(lo));
  return r;
}
// Elementwise bf16 product, rounded once (the product of two bf16 values is
// exact in fp32, so this equals bf16(float(a) * float(b))).
__device__ __forceinline__ uint32_t mul_bf16x2(uint32_t a, uint32_t b) {
  uint32_t r;
  asm("mul.rn.bf16x2 %0, %1, %2;" : "=r"(r) : "r"(a), "r"(b));
  return r;
}


template <int MODE>
__global__ void __launch_bounds__(PF_THREADS, 1)
pf_gemm_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB0,
               const __grid_constant__ CUtensorMap tmB1, const __grid_constant__ CUtensorMap tmS0,
               const __grid_constant__ CUtensorMap tmS1, const __grid_constant__ CUtensorMap tmHv,
               const __grid_constant__ CUtensorMap tmOut, PfGemmParams p) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t *smem = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                              ~uintptr_t(1023));
  constexpr int NS = pf_stages(MODE);
  constexpr int SB = pf_stage_bytes(MODE);
  constexpr bool PRING = pf_pring(MODE);
  constexpr int NOUT = pf_out_bufs(MODE);
  __shared__ __align__(8) uint64_t bar_pempty[2];  // down: code ring slots free
  __shared__ __align__(8) uint64_t bar_tma[PF_STAGES_MAX], bar_deq[PF_STAGES_MAX],
      bar_empty[PF_STAGES_MAX];
  __shared__ __align__(8) uint64_t bar_acc_full[2], bar_acc_empty[2], bar_final;
  __shared__ uint32_t s_tmem;
  __shared__ int s_abort;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int n_mt = *p.n_mtiles;
  const int n_tiles = n_mt * p.nt;
  const int ksteps = p.K / PF_BK;
  constexpr bool DEQ = MODE != PF_ROUTER;

  if (tid == 0) {
    for (int s = 0; s < NS; ++s) {
      // gate/up: the TMA producer + the 64 threads of the A-gather warps
      tc::mbar_init(&bar_tma[s], MODE == PF_GATEUP ? 1 + 64 : 1);
      tc::mbar_init(&bar_deq[s], 8);
      tc::mbar_init(&bar_empty[s], 1);
    }
    for (int a = 0; a < 2; ++a) {
      tc::mbar_init(&bar_acc_full[a], 1);
      tc::mbar_init(&bar_acc_empty[a], 8);
    }
    tc::mbar_init(&bar_final, 1);
    tc::mbar_init(&bar_pempty[0], 8);
    tc::mbar_init(&bar_pempty[1], 8);
    s_abort = 0;
    tc::fence_mbar_init();
  }
  if (warp == 1) {
    tc::tmem_alloc(&s_tmem, 512);
    tc::tmem_relinquish();
  }
  if (warp == 0 && lane == 0) {
    if (MODE != PF_GATEUP) tc::prefetch_tmap(&tmA);
    tc::prefetch_tmap(&tmB0);
    if (MODE == PF_GATEUP) tc::prefetch_tmap(&tmB1);
  }
  if (warp == 12 && lane == 0 && MODE != PF_ROUTER) tc::prefetch_tmap(&tmOut);
  tc::tc_fence_before();
  __syncthreads();
  tc::tc_fence_after();
  const uint32_t tmem = s_tmem;
  volatile int32_t *abort = &s_abort;
  auto fail = [&]() {
    s_abort = 1;
    flag_status(p.status, VB_STATUS_TIMEOUT);
  };
  auto stage_a = [&](int s) { return smem + s * SB; };
  auto stage_b = [&](int s) { return smem + s * SB + PF_A_BYTES; };
  // Packed codes of stage s (down: slot `slot` of the code ring).
  auto stage_p = [&](int s, int slot) {
    return PRING ? smem + NS * SB + slot * PF_P_BYTES : smem + s * SB + PF_A_BYTES + PF_B_BYTES;
  };

  if (warp == 0) {
    // ---------------- TMA producer ----------------
    if (lane == 0) {
      int it = 0, pq = 0;  // pq: dequantized down stages issued (code ring)
      for (int t = blockIdx.x; t < n_tiles && !*abort; t += gridDim.x) {
        const int mt = t / p.nt, nt = t % p.nt;
        const int e = p.mtiles[3 * mt], row0 = p.mtiles[3 * mt + 1];
        const bool sh = e == p.shared_e;
        const int slot = sh ? 0 : (MODE == PF_ROUTER ? 0 : p.slot_of[e]);
        const int hv = MODE == PF_ROUTER ? -1 : p.heavy_of[e];
        for (int ks = 0; ks < ksteps; ++ks, ++it) {
          const int s = it % NS;
          const uint32_t ph = (it / NS) & 1;
          if (!tc::mbar_wait(&bar_empty[s], ph ^ 1, abort, PF_WAIT_NS)) { fail(); break; }
          if (hv >= 0) {
            // pre-dequantized bf16 weights: straight into the B tile
            tc::mbar_arrive_expect_tx(&bar_tma[s], (MODE == PF_GATEUP ? 0 : PF_A_BYTES) + PF_B_BYTES);
            if (MODE != PF_GATEUP) tc::tma_load_2d(stage_a(s), &tmA, &bar_tma[s], ks * PF_BK, row0);
            tc::tma_load_3d(stage_b(s), &tmHv, &bar_tma[s], ks * PF_BK, nt * PF_BN, hv);
          } else if (MODE == PF_ROUTER) {
            // The last N tile may be narrow (tmB1: box of tail_n rows).
            const bool narrow = p.tail_n > 0 && nt == p.nt - 1;
            tc::mbar_arrive_expect_tx(&bar_tma[s],
                                      PF_A_BYTES + (narrow ? p.tail_n * PF_BK * 2 : PF_B_BYTES));
            tc::tma_load_2d(stage_a(s), &tmA, &bar_tma[s], ks * PF_BK, row0);
            tc::tma_load_2d(stage_b(s), narrow ? &tmB1 : &tmB0, &bar_tma[s], ks * PF_BK,
                            nt * PF_BN);
          } else if (MODE == PF_GATEUP) {
            tc::mbar_arrive_expect_tx(&bar_tma[s], PF_P_BYTES);  // A: the gather warps
            const CUtensorMap *g = sh ? &tmS0 : &tmB0;
            const CUtensorMap *u = sh ? &tmS1 : &tmB1;
            tc::tma_load_3d(stage_p(s, 0), g, &bar_tma[s], ks * (PF_BK / 2), nt * 128, slot);
            tc::tma_load_3d(stage_p(s, 0) + PF_P_BYTES / 2, u, &bar_tma[s], ks * (PF_BK / 2),
                            nt * 128, slot);
          } else {
            // Down, dequantized tile: the codes go to the next ring slot once
            // the dequantizing warps have read what it held.
            int ps = 0;
            if (PRING) {
              ps = pq & 1;
              if (!tc::mbar_wait(&bar_pempty[ps], ((pq >> 1) & 1) ^ 1, abort, PF_WAIT_NS)) {
                fail();
                break;
              }
              ++pq;
            }
            tc::mbar_arrive_expect_tx(&bar_tma[s], PF_A_BYTES + PF_P_BYTES);
            tc::tma_load_2d(stage_a(s), &tmA, &bar_tma[s], ks * PF_BK, row0);
            const CUtensorMap *d = sh ? &tmS0 : &tmB0;
            tc::tma_load_3d(stage_p(s, ps), d, &bar_tma[s], ks * (PF_BK / 2), nt * PF_BN, slot);
          }
        }
      }
      // Wind down: let the copies already issued land before the CTA ends.
      for (int k = 0; k < NS && it - 1 - k >= 0; ++k) {
        const int j = it - 1 - k;
        tc::mbar_wait(&bar_tma[j % NS], (j / NS) & 1, nullptr, PF_WAIT_NS);
      }
    }
  } else if (MODE == PF_GATEUP && (warp == 2 || warp == 3)) {
    // ---------------- A gather (gate/up) ----------------
    // Warp gw copies tile rows 64 gw .. 64 gw + 63 of every k-step: lane l
    // moves 16-byte chunk l % 8 of rows 64 gw + 4 j + l / 8, j < 16 (rows
    // past the tile's end repeat its first row), into the swizzled A tile.
    // Every thread's arrival on the stage barrier fires when its copies
    // have landed (cp.async.mbarrier.arrive), so the warps never wait for
    // data, only for free stages.
    const int gw = warp - 2, c = lane & 7;
    int it = 0;
    bool ok = true;
    for (int t = blockIdx.x; t < n_tiles; t += gridDim.x) {
      if (__shfl_sync(0xffffffffu, (!ok || *abort) ? 1 : 0, 0)) break;  // warp-uniform
      const int mt = t / p.nt;
      const int row0 = p.mtiles[3 * mt + 1], rows = p.mtiles[3 * mt + 2];
      const int tok0 = p.tok_of[row0];
      const uint16_t *src[16];
#pragma unroll
      for (int j = 0; j < 16; ++j) {
        const int r = 64 * gw + 4 * j + (lane >> 3);
        src[j] = p.x + (size_t)(r < rows ? p.tok_of[row0 + r] : tok0) * p.K + c * 8;
      }
      for (int ks = 0; ks < ksteps; ++ks, ++it) {
        const int s = it % NS;
        const uint32_t ph = (it / NS) & 1;
        bool got = true;
        if (lane == 0) got = tc::mbar_wait(&bar_empty[s], ph ^ 1, abort, PF_WAIT_NS);
        if (!__shfl_sync(0xffffffffu, got ? 1 : 0, 0)) {
          if (lane == 0) fail();
          ok = false;
          break;
        }
        uint8_t *a = stage_a(s);
#pragma unroll
        for (int j = 0; j < 16; ++j)
          cp_async16(a + sw128(64 * gw + 4 * j + (lane >> 3), c), src[j] + ks * PF_BK);
        tc::cp_async_mbar_arrive_noinc(&bar_tma[s]);
      }
    }
    cp_async_wait<0>();
  } else if (warp == 1) {
    // ---------------- MMA issuer ----------------
    if (lane == 0) {
      const uint32_t idesc_full = tc::idesc_bf16_f32(PF_BM, PF_BN);
      const uint32_t idesc_tail =
          MODE == PF_ROUTER && p.tail_n > 0 ? tc::idesc_bf16_f32(PF_BM, p.tail_n) : idesc_full;
      int it = 0, tcount = 0;
      uint32_t deq_par = 0;  // per stage: parity of the next dequant phase
      bool issued = false;
      for (int t = blockIdx.x; t < n_tiles && !*abort; t += gridDim.x, ++tcount) {
        const int acc = tcount & 1;
        const bool deq = DEQ && p.heavy_of[p.mtiles[3 * (t / p.nt)]] < 0;
        const uint32_t idesc = (t % p.nt == p.nt - 1) ? idesc_tail : idesc_full;
        if (!tc::mbar_wait(&bar_acc_empty[acc], ((tcount >> 1) & 1) ^ 1, abort, PF_WAIT_NS)) {
          fail();
          break;
        }
        tc::tc_fence_after();
        const uint32_t d = tmem + acc * PF_BN;
        bool ok = true;
        for (int ks = 0; ks < ksteps; ++ks, ++it) {
          const int s = it % NS;
          const uint32_t ph = (it / NS) & 1;
          // The dequant barrier of a stage only advances on dequantized
          // steps, so its parity is tracked separately.
          uint64_t *ready = deq ? &bar_deq[s] : &bar_tma[s];
          const uint32_t rph = deq ? ((deq_par >> s) & 1u) : ph;
          if (deq) deq_par ^= 1u << s;
          if (!tc::mbar_wait(ready, rph, abort, PF_WAIT_NS)) { fail(); ok = false; break; }
          tc::tc_fence_after();
          const uint32_t a0 = tc::smem_u32(stage_a(s)), b0 = tc::smem_u32(stage_b(s));
#pragma unroll
          for (int k = 0; k < PF_BK / 16; ++k)
            tc::mma_bf16_ss(d, tc::smem_desc_sw128(a0 + 32 * k), tc::smem_desc_sw128(b0 + 32 * k),
                            idesc, (ks | k) != 0);
          tc::mma_commit(&bar_empty[s]);
          issued = true;
        }
        if (!ok) break;
        tc::mma_commit(&bar_acc_full[acc]);
      }
      // All issued MMAs complete before TMEM is released.
      if (issued) {
        tc::mma_commit(&bar_final);
        tc::mbar_wait(&bar_final, 0, nullptr, PF_WAIT_NS);
      }
    }
  } else if (DEQ && warp >= 4 && warp < 12) {
    // ---------------- dequantize B ----------------
    // Thread r owns B row r: gate rows 0..127 and up rows 128..255 of the
    // N tile (gate/up), or down rows (down).
    const int r = tid - 128;
    int it = 0, pq = 0;  // pq: dequantized down stages consumed (code ring)
    for (int t = blockIdx.x; t < n_tiles && !*abort; t += gridDim.x) {
      const int mt = t / p.nt, nt = t % p.nt;
      const int e = p.mtiles[3 * mt];
      if (p.heavy_of[e] >= 0) {
        // Pre-dequantized: B arrives by TMA. Still follow every phase of the
        // TMA barriers so that no later parity wait can match a stale phase.
        bool ok = true;
        for (int ks = 0; ks < ksteps; ++ks, ++it) {
          if (!tc::mbar_wait_sleep(&bar_tma[it % NS], (it / NS) & 1, abort,
                                   PF_WAIT_NS)) {
            fail();
            ok = false;
            break;
          }
        }
        if (!ok) break;
        continue;
      }
      const bool sh = e == p.shared_e;
      const VbQuantPool &pool = sh ? p.shared : p.pool;
      const int slot = sh ? 0 : p.slot_of[e];
      int tsc, row;
      if (MODE == PF_GATEUP) {
        tsc = r < 128 ? 1 : 4;
        row = nt * 128 + (r & 127);
      } else {
        tsc = 7;
        row = nt * PF_BN + r;
      }
      const int ng = (p.K >> 6) >> p.gshift;  // scale groups per row
      const uint16_t *sp =
          reinterpret_cast<const uint16_t *>(pool_ptr(pool, tsc, slot)) + (size_t)row * ng;
      const uint16_t *bp =
          reinterpret_cast<const uint16_t *>(pool_ptr(pool, tsc + 1, slot)) + (size_t)row * ng;
      bool ok = true;
      for (int ks = 0; ks < ksteps; ++ks, ++it) {
        const int s = it % NS;
        const uint32_t ph = (it / NS) & 1;
        const int gi = ks >> p.gshift;
        const uint32_t sc = __ldg(sp + gi), bi = __ldg(bp + gi);
        if (!tc::mbar_wait(&bar_tma[s], ph, abort, PF_WAIT_NS)) { fail(); ok = false; break; }
        const int ps = PRING ? (pq++ & 1) : 0;
        const uint4 *src = reinterpret_cast<const uint4 *>(stage_p(s, ps) + r * 32);
        const uint4 w0 = src[0], w1 = src[1];
        if (PRING) {  // the ring slot may be refilled once every warp has its codes
          __syncwarp();
          if (lane == 0) tc::mbar_arrive(&bar_pempty[ps]);
        }
        const uint32_t words[8] = {w0.x, w0.y, w0.z, w0.w, w1.x, w1.y, w1.z, w1.w};
        const uint32_t s2 = sc | (sc << 16), b2 = bi | (bi << 16);
        uint8_t *dst = stage_b(s);
#pragma unroll
        for (int w = 0; w < 8; ++w) {
          uint32_t o[4];
          dequant4_bf16x2(words[w], s2, b2, o);
          uint4 chunk;
          if (MODE == PF_GATEUP)  // pairs (0,4),(1,5),(2,6),(3,7) -> columns 0..7
            chunk = make_uint4(__byte_perm(o[0], o[1], 0x5410), __byte_perm(o[2], o[3], 0x5410),
                               __byte_perm(o[0], o[1], 0x7632), __byte_perm(o[2], o[3], 0x7632));
          else
            chunk = make_uint4(o[0], o[1], o[2], o[3]);
          *reinterpret_cast<uint4 *>(dst + sw128(r, w)) = chunk;
        }
        tc::fence_proxy_async_smem();
        __syncwarp();
        if (lane == 0) tc::mbar_arrive(&bar_deq[s]);
      }
      if (!ok) break;
    }
  } else if (warp >= 12) {
    // ---------------- epilogue ----------------
    // 8 warps: lane quarter q = warp % 4 (TMEM lanes 32q..32q+31), column
    // half hf = (warp - 12) / 4.
    const int q = warp & 3, hf = (warp - 12) >> 2;
    const int m = q * 32 + lane;  // tile row = TMEM lane
    int tcount = 0;
    // Chunks of 32 rows x 32 columns whose rows are all valid go out as one
    // TMA store from a swizzled staging buffer (two per warp, alternating);
    // the rows of a partial chunk are stored by their threads.
    uint8_t *obuf = smem + NS * SB + (PRING ? 2 * PF_P_BYTES : 0) +
                    (warp - 12) * NOUT * PF_OUT_CHUNK;  // not gate/up
    int nst = 0;
    auto store_chunk = [&](const uint32_t (&o)[16], bool full, bool valid, size_t orow,
                           int col) {
      if (full) {
        uint8_t *b = obuf + (NOUT == 2 ? (nst & 1) : 0) * PF_OUT_CHUNK;
        if (lane == 0 && nst >= NOUT) {
          if (NOUT == 2) tc::bulk_wait_read<1>();
          else tc::bulk_wait_read<0>();
        }
        __syncwarp();
        const int sw = (lane >> 1) & 3;  // 64-byte swizzle: chunk c ^ ((row >> 1) & 3)
#pragma unroll
        for (int c = 0; c < 4; ++c)
          *reinterpret_cast<uint4 *>(b + lane * 64 + ((c ^ sw) << 4)) =
              make_uint4(o[4 * c], o[4 * c + 1], o[4 * c + 2], o[4 * c + 3]);
        tc::fence_proxy_async_smem();
        __syncwarp();
        if (lane == 0) {
          tc::tma_store_2d(&tmOut, b, col, (int)(orow - lane));
          tc::bulk_commit();
        }
        ++nst;
      } else if (valid) {
        uint4 *dst = reinterpret_cast<uint4 *>(p.out + orow * p.out_ld + col);
#pragma unroll
        for (int v = 0; v < 4; ++v)
          dst[v] = make_uint4(o[4 * v], o[4 * v + 1], o[4 * v + 2], o[4 * v + 3]);
      }
    };
    for (int t = blockIdx.x; t < n_tiles && !*abort; t += gridDim.x, ++tcount) {
      const int mt = t / p.nt, nt = t % p.nt;
      const int row0 = p.mtiles[3 * mt + 1], rows = p.mtiles[3 * mt + 2];
      const int acc = tcount & 1;
      if (!tc::mbar_wait_sleep(&bar_acc_full[acc], (tcount >> 1) & 1, abort, PF_WAIT_NS)) {
        fail();
        break;
      }
      tc::tc_fence_after();
      const uint32_t tb = tmem + ((uint32_t)(q * 32) << 16) + acc * PF_BN;
      const bool valid = m < rows;
      const bool full = MODE != PF_GATEUP && q * 32 + 32 <= rows;  // warp-uniform
      const size_t orow = (size_t)(row0 + m);
      if (MODE == PF_GATEUP) {
        // Columns [0,128) gate, [128,256) up of intermediate rows nt*128 + c;
        // this warp takes c in [64 hf, 64 hf + 64).
#pragma unroll 1
        for (int c0 = 64 * hf; c0 < 64 * hf + 64; c0 += 32) {
          uint32_t g[32], u[32];
          tc::tmem_ld32(tb + c0, g);
          tc::tmem_ld32(tb + 128 + c0, u);
          tc::tmem_ld_wait();
          uint32_t o[16];
#pragma unroll
          for (int b = 0; b < 4; ++b) {
            float h[8];
#pragma unroll
            for (int j = 0; j < 8; ++j)
              h[j] = swiglu_bf16(rbf(__uint_as_float(g[8 * b + j])),
                                 rbf(__uint_as_float(u[8 * b + j])));
            // 8-column block in the (0,4,1,5,2,6,3,7) code order
#pragma unroll
            for (int i = 0; i < 4; ++i) o[4 * b + i] = pack_bf2(h[i], h[i + 4]);
          }
          store_chunk(o, full, valid, orow, nt * 128 + c0);
        }
      } else if (MODE == PF_DOWN) {
        // bf16(bf16(y) * score): the score is a bf16 value.
        const uint32_t s16 = valid ? (uint32_t)f2bf(p.row_score[orow]) : 0x3F80u;
        const uint32_t sc2 = s16 | (s16 << 16);
#pragma unroll 1
        for (int c0 = 128 * hf; c0 < 128 * hf + 128; c0 += 32) {
          uint32_t v[32];
          tc::tmem_ld32(tb + c0, v);
          tc::tmem_ld_wait();
          uint32_t o[16];
#pragma unroll
          for (int j = 0; j < 16; ++j)
            o[j] = mul_bf16x2(cvt_bf16x2(__uint_as_float(v[2 * j]), __uint_as_float(v[2 * j + 1])),
                              sc2);
          store_chunk(o, full, valid, orow, nt * PF_BN + c0);
        }
      } else {
        const float sc = 1.f;
        const int ncols = (p.tail_n > 0 && nt == p.nt - 1) ? p.tail_n : PF_BN;
#pragma unroll 1
        for (int c0 = 128 * hf; c0 < 128 * hf + 128 && c0 < ncols; c0 += 32) {
          uint32_t v[32];
          tc::tmem_ld32(tb + c0, v);
          tc::tmem_ld_wait();
          uint32_t o[16];
#pragma unroll
          for (int j = 0; j < 16; ++j) {
            float y0 = __uint_as_float(v[2 * j]), y1 = __uint_as_float(v[2 * j + 1]);
            if (MODE == PF_DOWN) {
              y0 = rbf(__fmul_rn(rbf(y0), sc));
              y1 = rbf(__fmul_rn(rbf(y1), sc));
            } else {
              const int col = nt * PF_BN + c0 + 2 * j;
              const float b0 = (p.bias && col < p.n_valid) ? p.bias[col] : 0.f;
              const float b1 = (p.bias && col + 1 < p.n_valid) ? p.bias[col + 1] : 0.f;
              y0 = rbf(y0 + b0);
              y1 = rbf(y1 + b1);
            }
            o[j] = pack_bf2(y0, y1);
          }
          if (valid) {
            uint4 *dst = reinterpret_cast<uint4 *>(p.out + orow * p.out_ld + nt * PF_BN + c0);
            const int nw = ncols - c0 >= 32 ? 4 : (ncols - c0) / 8;  // tail_n % 16 == 0
#pragma unroll
            for (int w = 0; w < 4; ++w)
              if (w < nw) dst[w] = make_uint4(o[4 * w], o[4 * w + 1], o[4 * w + 2], o[4 * w + 3]);
          }
        }
      }
      tc::tc_fence_before();
      __syncwarp();
      if (lane == 0) tc::mbar_arrive(&bar_acc_empty[acc]);
    }
    if (lane == 0) tc::bulk_wait<0>();  // stores complete before the CTA ends
  }
  tc::tc_fence_before();
  __syncthreads();
  tc::tc_fence_after();
  if (warp == 1) tc::tmem_dealloc(tmem, 512);
}

// ----------------------------------------------------------------------------
// P0: router rows (E experts + the shared gate) into a zero-padded bf16
// matrix of NRP rows.
// ----------------------------------------------------------------------------
__global__ void pf_router_rows_kernel(const uint16_t *__restrict__ wr,
                                      const uint16_t *__restrict__ wsg, int E, int H, int NRP,
                                      uint16_t *__restrict__ dst) {
  const size_t n = (size_t)NRP * H / 8;
  for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < n;
       i += (size_t)gridDim.x * blockDim.x) {
    const size_t row = i / (H / 8), c = i % (H / 8);
    uint4 v = make_uint4(0, 0, 0, 0);
    if (row < (size_t)E) v = reinterpret_cast<const uint4 *>(wr + row * H)[c];
    else if (row == (size_t)E && wsg) v = reinterpret_cast<const uint4 *>(wsg)[c];
    reinterpret_cast<uint4 *>(dst)[i] = v;
  }
}

// Tile list (0, row0, rows) covering T rows.
__global__ void pf_row_tiles_kernel(int T, int32_t *__restrict__ mtiles,
                                    int32_t *__restrict__ n_mtiles) {
  const int nm = (T + PF_BM - 1) / PF_BM;
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i < nm) {
    mtiles[3 * i] = 0;
    mtiles[3 * i + 1] = i * PF_BM;
    mtiles[3 * i + 2] = min(PF_BM, T - i * PF_BM);
  }
  if (i == 0) *n_mtiles = nm;
}

// ----------------------------------------------------------------------------
// P2: per token softmax + top-k + renormalisation (one warp per token).
// ----------------------------------------------------------------------------
template <int PER>
__global__ void pf_topk_kernel(const uint16_t *__restrict__ logits, int ld, int T, int E, int k,
                               int norm_topk, int has_shared, const int32_t *__restrict__ table,
                               int cap, int32_t *__restrict__ inds, float *__restrict__ scores,
                               int32_t *__restrict__ counts, float *__restrict__ sgate,
                               int32_t *__restrict__ out_inds, uint16_t *__restrict__ out_scores,
                               uint16_t *__restrict__ out_logits, int32_t *__restrict__ status) {
  // Route counts go to a shared-memory histogram first (the hot experts of
  // skewed routing would serialise global atomics on a few addresses).
  extern __shared__ int32_t s_hist[];  // [E]
  for (int i = threadIdx.x; i < E; i += blockDim.x) s_hist[i] = 0;
  __syncthreads();
  const int lane = threadIdx.x & 31;
  const int nw = blockDim.x >> 5;
  for (int t = blockIdx.x * nw + (threadIdx.x >> 5); t < T; t += gridDim.x * nw) {
  const uint16_t *lr = logits + (size_t)t * ld;
  float v[PER];
#pragma unroll
  for (int i = 0; i < PER; ++i) {
    const int idx = lane + 32 * i;
    v[i] = idx < E ? bf2f(lr[idx]) : -INFINITY;
    if (out_logits && idx < E) out_logits[(size_t)t * E + idx] = lr[idx];
  }
  float m = -INFINITY;
#pragma unroll
  for (int i = 0; i < PER; ++i) m = fmaxf(m, v[i]);
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
  double sd[PER];
#pragma unroll
  for (int i = 0; i < PER; ++i) {
    const int idx = lane + 32 * i;
    const float ex = idx < E ? expf(__fsub_rn(v[i], m)) : 0.f;
    v[i] = ex;
    sd[i] = (double)ex;
  }
#pragma unroll
  for (int w = 1; w < PER; w *= 2)
#pragma unroll
    for (int i = 0; i + w < PER; i += 2 * w) sd[i] += sd[i + w];
  double s = sd[0];
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
  const float inv = __frcp_rn((float)s);
  uint32_t key[PER];
  uint32_t lb = 0;
#pragma unroll
  for (int i = 0; i < PER; ++i) {
    const int idx = lane + 32 * i;
    key[i] = idx < E ? ((uint32_t)f2bf(__fmul_rn(v[i], inv)) << 16) | (0xFFFFu - idx) : 0u;
    lb = max(lb, key[i]);
  }
  double ssum = 0.0;
  uint32_t sel = 0;
  for (int r = 0; r < k; ++r) {
    const uint32_t best = __reduce_max_sync(0xffffffffu, lb);
    if (lb == best) {
      lb = 0;
#pragma unroll
      for (int i = 0; i < PER; ++i) {
        if (key[i] == best) key[i] = 0u;
        lb = max(lb, key[i]);
      }
    }
    if (lane == r) sel = best;
    ssum += (double)bf2f(best >> 16);
  }
  const float sel_p = bf2f(sel >> 16);
  float score = sel_p;
  if (norm_topk) score = rbf(__fdiv_rn(sel_p, rbf((float)ssum)));
  if (lane < k) {
    const int ex = 0xFFFF - (int)(sel & 0xFFFFu);
    if (table) {
      const int slot = table[ex];
      if (slot < 0 || slot >= cap) flag_status(status, slot < 0 ? VB_STATUS_MISS : VB_STATUS_BOUNDS);
    }
    inds[t * k + lane] = ex;
    scores[t * k + lane] = score;
    atomicAdd(s_hist + ex, 1);
    if (out_inds) out_inds[t * k + lane] = ex;
    if (out_scores) out_scores[t * k + lane] = f2bf(score);
  }
  if (lane == 0 && has_shared) sgate[t] = rbf(mlx_sigmoid(bf2f(lr[E])));
  }
  __syncthreads();
  for (int i = threadIdx.x; i < E; i += blockDim.x)
    if (s_hist[i]) atomicAdd(counts + i, s_hist[i]);
}

// ----------------------------------------------------------------------------
// P3: plan (one CTA of 1024 threads). Routed experts whose slot is not
// resident get no rows. Experts (and the shared expert) with at least
// PF_HEAVY_ROWS rows get a pre-dequantized bf16 copy (up to PF_HEAVY_MAX).
// ----------------------------------------------------------------------------
constexpr int PF_PLAN_THREADS = 1024;
constexpr int PF_HEAVY_ROWS = 3 * PF_BM;
constexpr int PF_HEAVY_MAX = 48;

__device__ __forceinline__ int block_excl_scan(int v, int *tmp) {
  // inclusive scan over the CTA via shared memory (Hillis-Steele), returns exclusive
  const int tid = threadIdx.x;
  tmp[tid] = v;
  __syncthreads();
  for (int o = 1; o < PF_PLAN_THREADS; o <<= 1) {
    const int add = tid >= o ? tmp[tid - o] : 0;
    __syncthreads();
    tmp[tid] += add;
    __syncthreads();
  }
  const int incl = tmp[tid];
  __syncthreads();
  return incl - v;
}

__global__ void __launch_bounds__(PF_PLAN_THREADS)
pf_plan_kernel(int32_t *__restrict__ counts, const int32_t *__restrict__ table, int E, int cap,
               int has_shared, int32_t *__restrict__ offsets, int32_t *__restrict__ slot_of,
               int32_t *__restrict__ heavy_of, int32_t *__restrict__ heavy_e,
               int32_t *__restrict__ n_heavy, int32_t *__restrict__ cursor,
               int32_t *__restrict__ mtiles, int32_t *__restrict__ n_mtiles) {
  __shared__ int s_tmp[PF_PLAN_THREADS];
  const int tid = threadIdx.x;
  const int ne = E + 1;  // expert E = the shared expert
  int c = tid < ne ? counts[tid] : 0;
  // Rows only for resident experts.
  int slot = -1;
  if (tid < E) {
    const int sl = table[tid];
    slot = (sl >= 0 && sl < cap) ? sl : -1;
  } else if (tid == E && has_shared) {
    slot = 0;
  }
  if (slot < 0) c = 0;
  if (tid < ne) {
    counts[tid] = c;
    slot_of[tid] = slot;
    cursor[tid] = 0;
  }
  const int off = block_excl_scan(c, s_tmp);
  const int nt = (c + PF_BM - 1) / PF_BM;
  const int toff = block_excl_scan(nt, s_tmp);
  const int hflag = (tid < ne && c >= PF_HEAVY_ROWS) ? 1 : 0;
  const int hidx = block_excl_scan(hflag, s_tmp);
  if (tid < ne) {
    offsets[tid] = off;
    const int h = (hflag && hidx < PF_HEAVY_MAX) ? hidx : -1;
    heavy_of[tid] = h;
    if (h >= 0) heavy_e[h] = tid;
    for (int m = 0; m < nt; ++m) {
      mtiles[3 * (toff + m)] = tid;
      mtiles[3 * (toff + m) + 1] = off + m * PF_BM;
      mtiles[3 * (toff + m) + 2] = min(PF_BM, c - m * PF_BM);
    }
  }
  if (tid == ne - 1) {
    offsets[ne] = off + c;
    *n_mtiles = toff + nt;
    *n_heavy = min(hidx + hflag, PF_HEAVY_MAX);
  }
}

// The reference's reduce groups (block.py:154-172): experts in id order,
// skipping empty ones; a group closes at min(layer_cap, 128) experts or
// before exceeding max_assign routes. `counts` covers every routed expert of
// the whole prefill batch (all ranks).
__global__ void __launch_bounds__(PF_PLAN_THREADS)
pf_groups_kernel(const int32_t *__restrict__ counts, int E, int layer_cap, int max_assign,
                 int32_t *__restrict__ group_of) {
  __shared__ int s_cnt[PF_PLAN_THREADS];
  const int tid = threadIdx.x;
  if (tid < E) s_cnt[tid] = counts[tid];
  __syncthreads();
  if (tid == 0) {
    const int gcap = min(layer_cap, 128);
    int gid = 0, in_group = 0, sum = 0;
    for (int e = 0; e < E; ++e) {
      const int ce = s_cnt[e];
      if (ce == 0) {
        s_cnt[e] = -1;
        continue;
      }
      if (in_group && (in_group >= gcap || sum + ce > max_assign)) {
        ++gid;
        in_group = 0;
        sum = 0;
      }
      s_cnt[e] = gid;
      ++in_group;
      sum += ce;
    }
  }
  __syncthreads();
  if (tid < E) group_of[tid] = s_cnt[tid];
}

// Route list of a single-GPU prefill: routes t*k+j, then one shared-expert
// route per token (expert E, score 1).
__global__ void pf_routes_kernel(int T, int k, int E, int has_shared,
                                 const int32_t *__restrict__ inds,
                                 const float *__restrict__ scores, int32_t *__restrict__ r_row,
                                 int32_t *__restrict__ r_exp, float *__restrict__ r_score) {
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  const int R = T * k;
  if (i < R) {
    r_row[i] = i / k;
    r_exp[i] = inds[i];
    r_score[i] = scores[i];
  } else if (i < R + T && has_shared) {
    r_row[i] = i - R;
    r_exp[i] = E;
    r_score[i] = 1.f;
  }
}

__global__ void pf_set_kernel(int32_t *p, int32_t v) { *p = v; }

// Route histogram over experts 0..E (E = shared); negative ids are skipped.
__global__ void pf_hist_kernel(const int32_t *__restrict__ r_exp, int n, int E,
                               int32_t *__restrict__ counts) {
  extern __shared__ int32_t s_hist[];  // [E + 1]: per-CTA counts, then one flush
  for (int i = threadIdx.x; i <= E; i += blockDim.x) s_hist[i] = 0;
  __syncthreads();
  for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < n; i += gridDim.x * blockDim.x) {
    const int e = r_exp[i];
    if (e >= 0 && e <= E) atomicAdd(s_hist + e, 1);
  }
  __syncthreads();
  for (int i = threadIdx.x; i <= E; i += blockDim.x)
    if (s_hist[i]) atomicAdd(counts + i, s_hist[i]);
}

// ----------------------------------------------------------------------------
// Pre-dequantization of the heavy experts into bf16 (the same values and
// 8-column code order as the GEMM's own dequantization). Gate/up rows are
// stored in 256-row blocks [gate rows 128j..128j+127 | up rows 128j..],
// down rows as they are. One thread per packed word.
// ----------------------------------------------------------------------------
__global__ void __launch_bounds__(256)
pf_predequant_kernel(VbQuantPool pool, VbQuantPool shared, int shared_e,
                     const int32_t *__restrict__ heavy_e, const int32_t *__restrict__ n_heavy,
                     const int32_t *__restrict__ slot_of, int H, int I, int gshift,
                     uint16_t *__restrict__ wgu, uint16_t *__restrict__ wd) {
  const int h = blockIdx.y;
  if (h >= *n_heavy) return;
  const int e = heavy_e[h];
  const bool sh = e == shared_e;
  const VbQuantPool &pl = sh ? shared : pool;
  const int slot = sh ? 0 : slot_of[e];
  // One thread per 32 consecutive codes of a row (four packed words, one
  // scale group): gate/up rows first, then down rows.
  const size_t wgu_q = (size_t)2 * I * (H / 32), wd_q = (size_t)H * (I / 32);
  for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < wgu_q + wd_q;
       i += (size_t)gridDim.x * blockDim.x) {
    int row, qc, K, tw, tsc;
    uint16_t *dst;
    const bool gu = i < wgu_q;
    if (gu) {
      K = H;
      const int r = (int)(i / (H / 32));  // destination row
      qc = (int)(i % (H / 32));
      const int blk = r >> 8, within = r & 255;
      const bool up = within >= 128;
      row = blk * 128 + (within & 127);
      tw = up ? 3 : 0;
      tsc = up ? 4 : 1;
      dst = wgu + ((size_t)h * 2 * I + r) * H + qc * 32;
    } else {
      K = I;
      const size_t j = i - wgu_q;
      row = (int)(j / (I / 32));
      qc = (int)(j % (I / 32));
      tw = 6;
      tsc = 7;
      dst = wd + ((size_t)h * H + row) * I + qc * 32;
    }
    const uint4 w4 = ldg_nc_v4(pool_ptr(pl, tw, slot) + ((size_t)row * (K / 8) + 4 * qc) * 4);
    const int ng = (K >> 6) >> gshift, gi = (qc >> 1) >> gshift;
    const uint32_t sc = reinterpret_cast<const uint16_t *>(pool_ptr(pl, tsc, slot))[(size_t)row * ng + gi];
    const uint32_t bi = reinterpret_cast<const uint16_t *>(pool_ptr(pl, tsc + 1, slot))[(size_t)row * ng + gi];
    const uint32_t s2 = sc | (sc << 16), b2 = bi | (bi << 16);
    const uint32_t words[4] = {w4.x, w4.y, w4.z, w4.w};
#pragma unroll
    for (int wi = 0; wi < 4; ++wi) {
      uint32_t o[4];
      dequant4_bf16x2(words[wi], s2, b2, o);
      uint4 *d = reinterpret_cast<uint4 *>(dst + 8 * wi);
      if (gu)  // gate/up rows in column order
        *d = make_uint4(__byte_perm(o[0], o[1], 0x5410), __byte_perm(o[2], o[3], 0x5410),
                        __byte_perm(o[0], o[1], 0x7632), __byte_perm(o[2], o[3], 0x7632));
      else  // down rows in the code order of the h rows
        *d = make_uint4(o[0], o[1], o[2], o[3]);
    }
  }
}

// ----------------------------------------------------------------------------
// P4: sort. Every routed (resident) route gets a row of the expert-sorted
// order: one CTA per PF_SORT_ROUTES routes counts them per expert in shared
// memory, reserves each expert's rows with one global add, then hands them
// out. The order inside an expert is arbitrary (rows are independent).
// ----------------------------------------------------------------------------
constexpr int PF_SORT_PER_THREAD = 8;
constexpr int PF_SORT_ROUTES = 256 * PF_SORT_PER_THREAD;
__global__ void __launch_bounds__(256) pf_sort_kernel(
    int n, int E, const int32_t *__restrict__ r_row, const int32_t *__restrict__ r_exp,
    const float *__restrict__ r_score, const int32_t *__restrict__ slot_of,
    const int32_t *__restrict__ offsets, int32_t *__restrict__ cursor,
    int32_t *__restrict__ tok_of, float *__restrict__ row_score, int32_t *__restrict__ pos_of) {
  extern __shared__ int32_t s_sort[];  // count[E + 1], base[E + 1]
  int32_t *cnt = s_sort, *base = s_sort + E + 1;
  for (int i = threadIdx.x; i <= E; i += blockDim.x) cnt[i] = 0;
  __syncthreads();
  const int w0 = blockIdx.x * PF_SORT_ROUTES;
  int ex[PF_SORT_PER_THREAD], loc[PF_SORT_PER_THREAD];
#pragma unroll
  for (int j = 0; j < PF_SORT_PER_THREAD; ++j) {
    const int w = w0 + threadIdx.x + 256 * j;
    ex[j] = w < n ? r_exp[w] : -1;
    loc[j] = -1;
    if (ex[j] >= 0 && ex[j] <= E && slot_of[ex[j]] >= 0) loc[j] = atomicAdd(cnt + ex[j], 1);
  }
  __syncthreads();
  for (int i = threadIdx.x; i <= E; i += blockDim.x)
    if (cnt[i]) base[i] = offsets[i] + atomicAdd(cursor + i, cnt[i]);
  __syncthreads();
#pragma unroll
  for (int j = 0; j < PF_SORT_PER_THREAD; ++j) {
    const int w = w0 + threadIdx.x + 256 * j;
    if (w >= n) continue;
    const int pos = loc[j] >= 0 ? base[ex[j]] + loc[j] : -1;
    pos_of[w] = pos;
    if (pos >= 0) {
      tok_of[pos] = r_row[w];
      row_score[pos] = r_score[w];
    }
  }
}

// Rows of the expert-sorted output back into route order (skipped routes
// become zero rows).
__global__ void pf_unsort_kernel(const uint16_t *__restrict__ ys, int H, int n,
                                 const int32_t *__restrict__ pos_of, uint16_t *__restrict__ out) {
  const int lane = threadIdx.x & 31;
  const int w = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  if (w >= n) return;
  const int pos = pos_of[w];
  uint4 *dst = reinterpret_cast<uint4 *>(out + (size_t)w * H);
  const uint4 *src = reinterpret_cast<const uint4 *>(ys + (size_t)(pos < 0 ? 0 : pos) * H);
  for (int c = lane; c < H / 8; c += 32) dst[c] = pos < 0 ? make_uint4(0, 0, 0, 0) : src[c];
}

// ----------------------------------------------------------------------------
// P7: combine. One warp per token; routes are ordered by (group of the
// expert, route rank); lanes own 8 columns at a time.
// ----------------------------------------------------------------------------
__global__ void __launch_bounds__(256, 4) pf_combine_kernel(const uint16_t *__restrict__ y, int T, int H, int k,
                                  const int32_t *__restrict__ inds,
                                  const int32_t *__restrict__ group_of,
                                  const int32_t *__restrict__ route_row,
                                  const uint16_t *__restrict__ y_shared,
                                  const int32_t *__restrict__ shared_row,
                                  const float *__restrict__ sgate, uint16_t *__restrict__ out) {
  const int lane = threadIdx.x & 31;
  const int t = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  if (t >= T) return;
  // Order of this token's routes: key = group * 32 + rank (lanes < k).
  int key = 0x7fffffff, pos = -1;
  if (lane < k) {
    pos = route_row[t * k + lane];
    const int g = group_of[inds[t * k + lane]];
    key = pos >= 0 ? g * 32 + lane : 0x7fffffff;
  }
  int order[16];
  int n = 0;
#pragma unroll
  for (int j = 0; j < 16; ++j) {
    if (j >= k) break;
    // j-th smallest key
    int kmin = key;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) kmin = min(kmin, __shfl_xor_sync(0xffffffffu, kmin, o));
    if (kmin == 0x7fffffff) break;
    const int src = __ffs(__ballot_sync(0xffffffffu, key == kmin)) - 1;
    order[j] = __shfl_sync(0xffffffffu, pos, src);
    if (lane == src) key = 0x7fffffff;
    n = j + 1;
  }
  const bool has_shared = y_shared != nullptr;
  const float g = has_shared ? sgate[t] : 0.f;
  const uint16_t *shr =
      has_shared ? y_shared + (size_t)(shared_row ? shared_row[t] : t) * H : nullptr;
  for (int c = lane * 8; c < H; c += 256) {
    float acc[8];
#pragma unroll
    for (int i = 0; i < 8; ++i) acc[i] = 0.f;
    // the chunk's route rows four at a time in flight, added in the
    // canonical order
    uint4 sv = make_uint4(0, 0, 0, 0);
    if (has_shared) sv = ldg_nc_v4(shr + c);
    for (int j0 = 0; j0 < n; j0 += 4) {
      uint4 rv[4];
#pragma unroll
      for (int q = 0; q < 4; ++q)
        if (j0 + q < n) rv[q] = ldg_nc_v4(y + (size_t)order[j0 + q] * H + c);
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        if (j0 + q >= n) break;
        const uint32_t w[4] = {rv[q].x, rv[q].y, rv[q].z, rv[q].w};
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          acc[2 * i] = rbf(acc[2 * i] + bf2f(w[i] & 0xFFFF));
          acc[2 * i + 1] = rbf(acc[2 * i + 1] + bf2f(w[i] >> 16));
        }
      }
    }
    if (has_shared) {
      const uint4 v = sv;
      const uint32_t w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        acc[2 * i] = rbf(acc[2 * i] + rbf(__fmul_rn(g, bf2f(w[i] & 0xFFFF))));
        acc[2 * i + 1] = rbf(acc[2 * i + 1] + rbf(__fmul_rn(g, bf2f(w[i] >> 16))));
      }
    }
    uint4 o;
    o.x = pack_bf2(acc[0], acc[1]);
    o.y = pack_bf2(acc[2], acc[3]);
    o.z = pack_bf2(acc[4], acc[5]);
    o.w = pack_bf2(acc[6], acc[7]);
    *reinterpret_cast<uint4 *>(out + (size_t)t * H + c) = o;
  }
}

// ----------------------------------------------------------------------------
// Expert-parallel dispatch: pack the rows and routes a rank sends to every
// destination rank (token rows deduplicated per destination; destination-
// major, tokens ascending, routes (t, j) ascending), and unpack the routes a
// rank received.
// ----------------------------------------------------------------------------
constexpr int EP_MAX_WORLD = 8;

__global__ void ep_count_kernel(const int32_t *__restrict__ inds, const int32_t *__restrict__ owner,
                                int T, int k, int world, int32_t *__restrict__ tok_cnt) {
  const int t = blockIdx.x * blockDim.x + threadIdx.x;
  if (t >= T) return;
  int cnt[EP_MAX_WORLD];
#pragma unroll
  for (int d = 0; d < EP_MAX_WORLD; ++d) cnt[d] = 0;
  for (int j = 0; j < k; ++j) {
    const int d = owner[inds[t * k + j]];
#pragma unroll
    for (int q = 0; q < EP_MAX_WORLD; ++q) cnt[q] += (q == d) ? 1 : 0;
  }
  for (int d = 0; d < world; ++d) tok_cnt[(size_t)t * world + d] = cnt[d];
}

// One CTA per destination: exclusive scans over tokens of (token goes to d)
// and (routes of the token to d).
__global__ void __launch_bounds__(1024)
ep_scan_kernel(const int32_t *__restrict__ tok_cnt, int T, int world, int32_t *__restrict__ row_idx,
               int32_t *__restrict__ route_base, int32_t *__restrict__ dest_rows,
               int32_t *__restrict__ dest_routes) {
  __shared__ int s_tmp[1024];
  const int d = blockIdx.x, tid = threadIdx.x;
  const int per = (T + 1023) / 1024;
  const int t0 = tid * per, t1 = min(T, t0 + per);
  int rows = 0, routes = 0;
  for (int t = t0; t < t1; ++t) {
    const int c = tok_cnt[(size_t)t * world + d];
    rows += c > 0 ? 1 : 0;
    routes += c;
  }
  // two block scans
  s_tmp[tid] = rows;
  __syncthreads();
  for (int o = 1; o < 1024; o <<= 1) {
    const int add = tid >= o ? s_tmp[tid - o] : 0;
    __syncthreads();
    s_tmp[tid] += add;
    __syncthreads();
  }
  int rbase = s_tmp[tid] - rows;
  const int rtot = s_tmp[1023];
  __syncthreads();
  s_tmp[tid] = routes;
  __syncthreads();
  for (int o = 1; o < 1024; o <<= 1) {
    const int add = tid >= o ? s_tmp[tid - o] : 0;
    __syncthreads();
    s_tmp[tid] += add;
    __syncthreads();
  }
  int qbase = s_tmp[tid] - routes;
  const int qtot = s_tmp[1023];
  for (int t = t0; t < t1; ++t) {
    const int c = tok_cnt[(size_t)t * world + d];
    row_idx[(size_t)t * world + d] = c > 0 ? rbase : -1;
    route_base[(size_t)t * world + d] = qbase;
    rbase += c > 0 ? 1 : 0;
    qbase += c;
  }
  if (tid == 0) {
    dest_rows[d] = rtot;
    dest_routes[d] = qtot;
  }
}

// One warp per token: copy the token row once per destination, write the
// route metadata (row in the destination chunk, expert, score bits) and the
// route's index in the send order.
__global__ void ep_pack_kernel(const uint16_t *__restrict__ x, const int32_t *__restrict__ inds,
                               const float *__restrict__ scores, const int32_t *__restrict__ owner,
                               int T, int k, int H, int world,
                               const int32_t *__restrict__ tok_cnt,
                               const int32_t *__restrict__ row_idx,
                               const int32_t *__restrict__ route_base,
                               const int32_t *__restrict__ dest_rows,
                               const int32_t *__restrict__ dest_routes,
                               uint16_t *__restrict__ send_x, int32_t *__restrict__ send_meta,
                               int32_t *__restrict__ route_send_idx) {
  // Per-destination chunk offsets in shared memory (indexed by a routed
  // expert's owner: a per-thread array would live in local memory).
  __shared__ int row_off[EP_MAX_WORLD], route_off[EP_MAX_WORLD];
  if (threadIdx.x == 0) {
    int ro = 0, qo = 0;
    for (int d = 0; d < world; ++d) {
      row_off[d] = ro;
      route_off[d] = qo;
      ro += dest_rows[d];
      qo += dest_routes[d];
    }
  }
  __syncthreads();
  const int lane = threadIdx.x & 31;
  const int t = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  if (t >= T) return;
  if (lane < k) {
    const int e = inds[t * k + lane];
    const int d = owner[e];
    int rank = 0;
    for (int j = 0; j < lane; ++j) rank += owner[inds[t * k + j]] == d ? 1 : 0;
    const int idx = route_off[d] + route_base[(size_t)t * world + d] + rank;
    send_meta[3 * (size_t)idx] = row_idx[(size_t)t * world + d];
    send_meta[3 * (size_t)idx + 1] = e;
    send_meta[3 * (size_t)idx + 2] = __float_as_int(scores[t * k + lane]);
    route_send_idx[t * k + lane] = idx;
  }
  const uint4 *src = reinterpret_cast<const uint4 *>(x + (size_t)t * H);
  for (int d = 0; d < world; ++d) {
    if (tok_cnt[(size_t)t * world + d] == 0) continue;
    uint4 *dst = reinterpret_cast<uint4 *>(send_x + (size_t)(row_off[d] + row_idx[(size_t)t * world + d]) * H);
    for (int c = lane; c < H / 8; c += 32) dst[c] = __ldg(src + c);
  }
}

// Received routes: source s's routes [route_off[s], route_off[s+1]) refer to
// rows relative to s's chunk, which starts at row_off[s].
__global__ void ep_unpack_kernel(const int32_t *__restrict__ meta, int n,
                                 const int32_t *__restrict__ route_off,
                                 const int32_t *__restrict__ row_off, int world,
                                 int32_t *__restrict__ r_row, int32_t *__restrict__ r_exp,
                                 float *__restrict__ r_score) {
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= n) return;
  int s = 0;
  while (s + 1 < world && i >= route_off[s + 1]) ++s;
  r_row[i] = row_off[s] + meta[3 * (size_t)i];
  r_exp[i] = meta[3 * (size_t)i + 1];
  r_score[i] = __int_as_float(meta[3 * (size_t)i + 2]);
}

// ----------------------------------------------------------------------------
// Host side
// ----------------------------------------------------------------------------
// Workspace of the route phase (router GEMM + top-k).
struct RouteLayout {
  size_t wr, logits, mtiles, n_mtiles, total;
  int NRP;
};
static RouteLayout route_layout(int T, int H, int E) {
  RouteLayout L;
  // Router rows (E experts + the shared gate): full PF_BN-row tiles, then a
  // tail tile of the remaining rows rounded up to 16 (the MMA's N step).
  L.NRP = (E + 1) / PF_BN * PF_BN + ((E + 1) % PF_BN + 15) / 16 * 16;
  size_t off = 0;
  auto take = [&](size_t bytes) {
    const size_t o = off;
    off = align_up(off + bytes, 1024);
    return o;
  };
  L.wr = take((size_t)L.NRP * H * 2);
  L.logits = take((size_t)T * L.NRP * 2);
  L.mtiles = take((size_t)((T + PF_BM - 1) / PF_BM) * 12);
  L.n_mtiles = take(4);
  L.total = off;
  return L;
}

// Workspace of the expert phase for n routes (experts 0..E, E = shared).
struct ExpertsLayout {
  size_t counts, offsets, slot_of, heavy_of, heavy_e, n_heavy, cursor, mtiles, n_mtiles, pos_of,
      row_score, tok_of, hs, ys, wgu, wd, total;
  int max_mtiles, rows_alloc;
};
static ExpertsLayout experts_layout(int n, int H, int I, int E) {
  ExpertsLayout L;
  L.max_mtiles = n / PF_BM + E + 2;
  L.rows_alloc = n + PF_BM;
  size_t off = 0;
  auto take = [&](size_t bytes) {
    const size_t o = off;
    off = align_up(off + bytes, 1024);
    return o;
  };
  L.counts = take((size_t)(E + 2) * 4);
  L.offsets = take((size_t)(E + 2) * 4);
  L.slot_of = take((size_t)(E + 1) * 4);
  L.heavy_of = take((size_t)(E + 1) * 4);
  L.heavy_e = take((size_t)PF_HEAVY_MAX * 4);
  L.n_heavy = take(4);
  L.cursor = take((size_t)(E + 1) * 4);
  L.mtiles = take((size_t)L.max_mtiles * 12);
  L.n_mtiles = take(4);
  L.pos_of = take((size_t)n * 4 + 4);
  L.row_score = take((size_t)n * 4 + 4);
  L.tok_of = take((size_t)L.rows_alloc * 4);
  L.hs = take((size_t)L.rows_alloc * I * 2);
  L.ys = take((size_t)L.rows_alloc * H * 2);
  L.wgu = take((size_t)PF_HEAVY_MAX * 2 * I * H * 2);
  L.wd = take((size_t)PF_HEAVY_MAX * H * I * 2);
  L.total = off;
  return L;
}

// Single-call prefill: route + route list + experts + combine.
struct PrefillLayout {
  RouteLayout R;
  ExpertsLayout X;
  size_t route, inds, scores, sgate, counts, r_row, r_exp, r_score, group_of, experts, total;
};
static PrefillLayout prefill_layout(int T, int H, int I, int E, int k) {
  PrefillLayout L;
  L.R = route_layout(T, H, E);
  const int n = T * k + T;
  L.X = experts_layout(n, H, I, E);
  size_t off = 0;
  auto take = [&](size_t bytes) {
    const size_t o = off;
    off = align_up(off + bytes, 1024);
    return o;
  };
  L.route = take(L.R.total);
  L.inds = take((size_t)T * k * 4);
  L.scores = take((size_t)T * k * 4);
  L.sgate = take((size_t)T * 4);
  L.counts = take((size_t)(E + 2) * 4);
  L.r_row = take((size_t)n * 4);
  L.r_exp = take((size_t)n * 4);
  L.r_score = take((size_t)n * 4);
  L.group_of = take((size_t)(E + 1) * 4);
  L.experts = take(L.X.total);
  L.total = off;
  return L;
}

typedef CUresult (*EncodeTiledFn)(CUtensorMap *, CUtensorMapDataType, cuuint32_t, void *,
                                  const cuuint64_t *, const cuuint64_t *, const cuuint32_t *,
                                  const cuuint32_t *, CUtensorMapInterleave, CUtensorMapSwizzle,
                                  CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

static EncodeTiledFn encode_fn() {
  static EncodeTiledFn fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void *ptr = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &ptr, cudaEnableDefault, &q) ==
            cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeTiledFn>(ptr);
  });
  return fn;
}

// bf16 [rows, cols] row-major, box {64 cols, box_rows}, 128-byte swizzle.
static int make_map_bf16(CUtensorMap *m, const void *base, uint64_t rows, uint64_t cols,
                         uint32_t box_rows) {
  EncodeTiledFn f = encode_fn();
  if (!f) return set_error(VB_ERR_CUDA, "cuTensorMapEncodeTiled unavailable");
  const cuuint64_t dims[2] = {cols, rows};
  const cuuint64_t strides[1] = {cols * 2};
  const cuuint32_t box[2] = {64, box_rows};
  const cuuint32_t estr[2] = {1, 1};
  CUresult r = f(m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void *>(base), dims, strides,
                 box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                 CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return set_error(VB_ERR_INVALID, "tensor map (bf16) failed: %d", (int)r);
  return VB_OK;
}

// Output rows of a GEMM: bf16 [rows, cols] row-major, box {32 cols, 32 rows},
// 64-byte swizzle (the epilogue's staging layout).
static int make_map_out(CUtensorMap *m, const void *base, uint64_t rows, uint64_t cols) {
  EncodeTiledFn f = encode_fn();
  if (!f) return set_error(VB_ERR_CUDA, "cuTensorMapEncodeTiled unavailable");
  const cuuint64_t dims[2] = {cols, rows};
  const cuuint64_t strides[1] = {cols * 2};
  const cuuint32_t box[2] = {32, 32};
  const cuuint32_t estr[2] = {1, 1};
  CUresult r = f(m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void *>(base), dims, strides,
                 box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_64B,
                 CU_TENSOR_MAP_L2_PROMOTION_NONE, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return set_error(VB_ERR_INVALID, "tensor map (out) failed: %d", (int)r);
  return VB_OK;
}

// bf16 [n][rows][cols] (row-major), box {64 cols, box_rows, 1}, 128-byte swizzle.
static int make_map_bf16_3d(CUtensorMap *m, const void *base, uint64_t n, uint64_t rows,
                            uint64_t cols, uint32_t box_rows) {
  EncodeTiledFn f = encode_fn();
  if (!f) return set_error(VB_ERR_CUDA, "cuTensorMapEncodeTiled unavailable");
  const cuuint64_t dims[3] = {cols, rows, n};
  const cuuint64_t strides[2] = {cols * 2, rows * cols * 2};
  const cuuint32_t box[3] = {64, box_rows, 1};
  const cuuint32_t estr[3] = {1, 1, 1};
  CUresult r = f(m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, const_cast<void *>(base), dims, strides,
                 box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                 CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return set_error(VB_ERR_INVALID, "tensor map (bf16 3d) failed: %d", (int)r);
  return VB_OK;
}

// Packed 4-bit codes of one pool tensor: bytes [slots][rows][cols/2], box
// {32 bytes, box_rows, 1}.
static int make_map_codes(CUtensorMap *m, const void *base, uint64_t slots, uint64_t slot_stride,
                          uint64_t rows, uint64_t cols, uint32_t box_rows) {
  EncodeTiledFn f = encode_fn();
  if (!f) return set_error(VB_ERR_CUDA, "cuTensorMapEncodeTiled unavailable");
  const cuuint64_t dims[3] = {cols / 2, rows, slots};
  const cuuint64_t strides[2] = {cols / 2, slot_stride};
  const cuuint32_t box[3] = {32, box_rows, 1};
  const cuuint32_t estr[3] = {1, 1, 1};
  CUresult r = f(m, CU_TENSOR_MAP_DATA_TYPE_UINT8, 3, const_cast<void *>(base), dims, strides,
                 box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE,
                 CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return set_error(VB_ERR_INVALID, "tensor map (codes) failed: %d", (int)r);
  return VB_OK;
}

static int pf_sm_count() {
  static int n = 0;
  if (!n) {
    int dev = 0;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
    if (n <= 0) n = 148;
  }
  return n;
}

template <int MODE>
static int launch_gemm(const CUtensorMap &a, const CUtensorMap &b0, const CUtensorMap &b1,
                       const CUtensorMap &s0, const CUtensorMap &s1, const CUtensorMap &hv,
                       const CUtensorMap &out, const PfGemmParams &p, int max_tiles,
                       cudaStream_t s) {
  static std::once_flag once;
  static cudaError_t attr_err = cudaSuccess;
  std::call_once(once, [] {
    attr_err = cudaFuncSetAttribute(pf_gemm_kernel<MODE>,
                                    cudaFuncAttributeMaxDynamicSharedMemorySize, pf_smem(MODE));
  });
  if (attr_err != cudaSuccess)
    return set_error(VB_ERR_CUDA, "pf_gemm_kernel attributes: %s", cudaGetErrorString(attr_err));
  const int grid = std::max(1, std::min(pf_sm_count(), max_tiles));
  pf_gemm_kernel<MODE><<<grid, PF_THREADS, pf_smem(MODE), s>>>(a, b0, b1, s0, s1, hv, out, p);
  return check_launch("pf_gemm_kernel");
}

// ---- phase implementations ----

static int run_route(const uint16_t *x, int T, int H, int E, int k, int norm_topk,
                     const uint16_t *router_w, const float *bias, const uint16_t *wsg,
                     const int32_t *table, int cap, int32_t *inds, float *scores, float *sgate,
                     int32_t *counts, int32_t *out_inds, uint16_t *out_scores,
                     uint16_t *out_logits, int32_t *status, uint8_t *ws, cudaStream_t s) {
  const RouteLayout L = route_layout(T, H, E);
  auto W = [&](size_t off) { return ws + off; };
  int rc;
  pf_router_rows_kernel<<<256, 256, 0, s>>>(router_w, wsg, E, H, L.NRP, (uint16_t *)W(L.wr));
  if ((rc = check_launch("pf_router_rows_kernel")) != VB_OK) return rc;
  if (cudaMemsetAsync(counts, 0, (size_t)(E + 1) * 4, s) != cudaSuccess)
    return set_error(VB_ERR_CUDA, "route: memset");
  const int nm = (T + PF_BM - 1) / PF_BM;
  pf_row_tiles_kernel<<<(nm + 255) / 256, 256, 0, s>>>(T, (int32_t *)W(L.mtiles),
                                                       (int32_t *)W(L.n_mtiles));
  if ((rc = check_launch("pf_row_tiles_kernel")) != VB_OK) return rc;
  CUtensorMap ta, tb, tbn;
  const int full = L.NRP / PF_BN, tail = L.NRP % PF_BN;
  if ((rc = make_map_bf16(&ta, x, T, H, PF_BM)) != VB_OK) return rc;
  if ((rc = make_map_bf16(&tb, W(L.wr), L.NRP, H, full > 0 ? PF_BN : tail)) != VB_OK) return rc;
  if ((rc = make_map_bf16(&tbn, W(L.wr), L.NRP, H, tail > 0 ? tail : PF_BN)) != VB_OK) return rc;
  PfGemmParams p{};
  p.mode = PF_ROUTER;
  p.K = H;
  p.nt = full + (tail > 0 ? 1 : 0);
  p.tail_n = tail;
  p.shared_e = -1;
  p.n_valid = E;
  p.mtiles = (const int32_t *)W(L.mtiles);
  p.n_mtiles = (const int32_t *)W(L.n_mtiles);
  p.out = (uint16_t *)W(L.logits);
  p.out_ld = L.NRP;
  p.bias = bias;
  p.status = status;
  if ((rc = launch_gemm<PF_ROUTER>(ta, tb, tbn, tb, tb, tb, tb, p, nm * p.nt, s)) != VB_OK) return rc;
  const int per = E <= 256 ? 8 : (E <= 512 ? 16 : 32);
  auto kfn = per == 8 ? pf_topk_kernel<8> : per == 16 ? pf_topk_kernel<16> : pf_topk_kernel<32>;
  const int tk_grid = std::max(1, std::min((T + 7) / 8, pf_sm_count() * 4));
  kfn<<<tk_grid, 256, (size_t)E * sizeof(int32_t), s>>>((const uint16_t *)W(L.logits), L.NRP, T, E, k, norm_topk,
                                  wsg ? 1 : 0, table, cap, inds, scores, counts, sgate, out_inds,
                                  out_scores, out_logits, status);
  return check_launch("pf_topk_kernel");
}

// Expert phase: rows x [R, H], n routes (row, expert 0..E with E = shared,
// score). Output: expert-sorted weighted rows in L.ys and pos_of (route ->
// row of L.ys, -1 = skipped).
static int run_experts(const uint16_t *x, int R, const int32_t *r_row, const int32_t *r_exp,
                       const float *r_score, int n, int H, int I, int E, int gshift,
                       const int32_t *table, const VbQuantPool &pool, const VbQuantPool &shared,
                       bool has_shared, int32_t *status, uint8_t *ws, const ExpertsLayout &L,
                       cudaStream_t s, bool counts_ready) {
  auto W = [&](size_t off) { return ws + off; };
  int rc;
  if (!counts_ready) {
    if (cudaMemsetAsync(W(L.counts), 0, (size_t)(E + 2) * 4, s) != cudaSuccess)
      return set_error(VB_ERR_CUDA, "experts: memset");
    pf_hist_kernel<<<std::max(1, std::min(pf_sm_count() * 2, (n + 255) / 256)), 256,
                     (size_t)(E + 1) * sizeof(int32_t), s>>>(
        r_exp, n, E, (int32_t *)W(L.counts));
    if ((rc = check_launch("pf_hist_kernel")) != VB_OK) return rc;
  }
  pf_plan_kernel<<<1, PF_PLAN_THREADS, 0, s>>>(
      (int32_t *)W(L.counts), table, E, pool.cap, has_shared ? 1 : 0, (int32_t *)W(L.offsets),
      (int32_t *)W(L.slot_of), (int32_t *)W(L.heavy_of), (int32_t *)W(L.heavy_e),
      (int32_t *)W(L.n_heavy), (int32_t *)W(L.cursor), (int32_t *)W(L.mtiles),
      (int32_t *)W(L.n_mtiles));
  if ((rc = check_launch("pf_plan_kernel")) != VB_OK) return rc;
  pf_predequant_kernel<<<dim3(128, PF_HEAVY_MAX), 256, 0, s>>>(
      pool, shared, has_shared ? E : -1, (const int32_t *)W(L.heavy_e),
      (const int32_t *)W(L.n_heavy), (const int32_t *)W(L.slot_of), H, I, gshift,
      (uint16_t *)W(L.wgu), (uint16_t *)W(L.wd));
  if ((rc = check_launch("pf_predequant_kernel")) != VB_OK) return rc;
  if (n > 0) {
    pf_sort_kernel<<<(n + PF_SORT_ROUTES - 1) / PF_SORT_ROUTES, 256,
                     (size_t)2 * (E + 1) * sizeof(int32_t), s>>>(
        n, E, r_row, r_exp, r_score, (const int32_t *)W(L.slot_of),
        (const int32_t *)W(L.offsets), (int32_t *)W(L.cursor), (int32_t *)W(L.tok_of),
        (float *)W(L.row_score), (int32_t *)W(L.pos_of));
    if ((rc = check_launch("pf_sort_kernel")) != VB_OK) return rc;
  }
  // gate/up
  {
    CUtensorMap ta, g, u, sg, su, hv, to;
    if ((rc = make_map_codes(&g, pool.ptr[0], pool.cap, pool.slot_stride[0], I, H, 128)) != VB_OK) return rc;
    if ((rc = make_map_codes(&u, pool.ptr[3], pool.cap, pool.slot_stride[3], I, H, 128)) != VB_OK) return rc;
    if (has_shared) {
      if ((rc = make_map_codes(&sg, shared.ptr[0], 1, (uint64_t)I * H / 2, I, H, 128)) != VB_OK) return rc;
      if ((rc = make_map_codes(&su, shared.ptr[3], 1, (uint64_t)I * H / 2, I, H, 128)) != VB_OK) return rc;
    } else {
      sg = g;
      su = u;
    }
    if ((rc = make_map_bf16_3d(&hv, W(L.wgu), PF_HEAVY_MAX, 2 * (uint64_t)I, H, PF_BN)) != VB_OK) return rc;
    ta = hv;  // the A rows are copied from x by the kernel's gather warps
    PfGemmParams p{};
    p.mode = PF_GATEUP;
    p.heavy_of = (const int32_t *)W(L.heavy_of);
    p.K = H;
    p.nt = I / 128;
    p.gshift = gshift;
    p.shared_e = has_shared ? E : -1;
    p.mtiles = (const int32_t *)W(L.mtiles);
    p.n_mtiles = (const int32_t *)W(L.n_mtiles);
    p.slot_of = (const int32_t *)W(L.slot_of);
    p.pool = pool;
    p.shared = shared;
    p.out = (uint16_t *)W(L.hs);
    p.out_ld = I;
    p.x = x;
    p.tok_of = (const int32_t *)W(L.tok_of);
    p.status = status;
    if ((rc = make_map_out(&to, W(L.hs), L.rows_alloc, I)) != VB_OK) return rc;
    if ((rc = launch_gemm<PF_GATEUP>(ta, g, u, sg, su, hv, to, p, L.max_mtiles * p.nt, s)) != VB_OK) return rc;
  }
  // down
  {
    CUtensorMap ta, d, sd, hv, to;
    if ((rc = make_map_bf16(&ta, W(L.hs), L.rows_alloc, I, PF_BM)) != VB_OK) return rc;
    if ((rc = make_map_codes(&d, pool.ptr[6], pool.cap, pool.slot_stride[6], H, I, PF_BN)) != VB_OK) return rc;
    if (has_shared) {
      if ((rc = make_map_codes(&sd, shared.ptr[6], 1, (uint64_t)H * I / 2, H, I, PF_BN)) != VB_OK) return rc;
    } else {
      sd = d;
    }
    if ((rc = make_map_bf16_3d(&hv, W(L.wd), PF_HEAVY_MAX, H, I, PF_BN)) != VB_OK) return rc;
    PfGemmParams p{};
    p.mode = PF_DOWN;
    p.heavy_of = (const int32_t *)W(L.heavy_of);
    p.K = I;
    p.nt = H / PF_BN;
    p.gshift = gshift;
    p.shared_e = has_shared ? E : -1;
    p.mtiles = (const int32_t *)W(L.mtiles);
    p.n_mtiles = (const int32_t *)W(L.n_mtiles);
    p.slot_of = (const int32_t *)W(L.slot_of);
    p.pool = pool;
    p.shared = shared;
    p.out = (uint16_t *)W(L.ys);
    p.out_ld = H;
    p.row_score = (const float *)W(L.row_score);
    p.status = status;
    if ((rc = make_map_out(&to, W(L.ys), L.rows_alloc, H)) != VB_OK) return rc;
    if ((rc = launch_gemm<PF_DOWN>(ta, d, d, sd, sd, hv, to, p, L.max_mtiles * p.nt, s)) != VB_OK) return rc;
  }
  return VB_OK;
}

static int check_pool(const VbQuantPool &pool, const VbQuantPool &shared, bool has_shared,
                      const char *what) {
  VB_REQUIRE(pool.ptr[0] && pool.cap > 0, "%s: empty pool", what);
  for (int i = 0; i < 9; ++i)
    VB_REQUIRE(((uintptr_t)pool.ptr[i] % 16) == 0 && (pool.slot_stride[i] % 16) == 0 &&
                   (!has_shared || ((uintptr_t)shared.ptr[i] % 16) == 0),
               "%s: pool tensors must be 16-byte aligned", what);
  return VB_OK;
}

}  // namespace vb

using namespace vb;

extern "C" {

size_t vb_moe_prefill_workspace_size(int32_t tokens, int32_t hidden, int32_t inter,
                                     int32_t num_experts, int32_t top_k) {
  if (tokens <= 0 || hidden <= 0 || inter <= 0 || num_experts <= 0 || top_k <= 0) return 0;
  return prefill_layout(tokens, hidden, inter, num_experts, top_k).total;
}

int vb_moe_prefill(const VbMoePrefillArgs *a, vb_stream_t stream) {
  VB_REQUIRE(a, "vb_moe_prefill: null args");
  const int T = a->tokens, H = a->hidden, I = a->inter, E = a->num_experts, k = a->top_k;
  VB_REQUIRE(T >= 1, "vb_moe_prefill: tokens=%d", T);
  VB_REQUIRE(a->bits == 4, "vb_moe_prefill: bits=%d (only 4-bit)", a->bits);
  VB_REQUIRE(a->group == 64 || a->group == 128, "vb_moe_prefill: group=%d", a->group);
  VB_REQUIRE(H % 256 == 0 && H >= 256 && H <= 8192, "vb_moe_prefill: hidden=%d", H);
  VB_REQUIRE(I % 128 == 0 && I >= 128 && I <= 4096, "vb_moe_prefill: inter=%d", I);
  VB_REQUIRE(E >= k && E < PF_PLAN_THREADS && k >= 1 && k <= 16, "vb_moe_prefill: experts/top_k");
  VB_REQUIRE(a->x && a->router_w && a->slot_table && a->out, "vb_moe_prefill: null tensor");
  const bool has_shared = a->shared.ptr[0] != nullptr;
  VB_REQUIRE(!has_shared || a->shared_gate_w, "vb_moe_prefill: shared expert without gate");
  int rc;
  if ((rc = check_pool(a->pool, a->shared, has_shared, "vb_moe_prefill")) != VB_OK) return rc;
  const PrefillLayout L = prefill_layout(T, H, I, E, k);
  VB_REQUIRE(a->workspace && a->workspace_bytes >= L.total, "vb_moe_prefill: workspace %zu < %zu",
             a->workspace_bytes, L.total);
  VB_REQUIRE(((uintptr_t)a->workspace % 1024) == 0, "vb_moe_prefill: workspace alignment");
  VB_REQUIRE(((uintptr_t)a->x % 16) == 0 && ((uintptr_t)a->out % 16) == 0,
             "vb_moe_prefill: x/out must be 16-byte aligned");
  uint8_t *ws = static_cast<uint8_t *>(a->workspace);
  auto W = [&](size_t off) { return ws + off; };
  cudaStream_t s = as_stream(stream);
  const int gshift = a->group == 128 ? 1 : 0;
  int32_t *inds = (int32_t *)W(L.inds), *counts = (int32_t *)W(L.counts);
  float *scores = (float *)W(L.scores), *sgate = (float *)W(L.sgate);
  if ((rc = run_route(a->x, T, H, E, k, a->norm_topk, a->router_w, a->router_bias,
                      has_shared ? a->shared_gate_w : nullptr, a->slot_table, a->pool.cap, inds,
                      scores, sgate, counts, a->out_inds, a->out_scores, a->out_logits, a->status,
                      W(L.route), s)) != VB_OK)
    return rc;
  // The reference's reduce groups from the routed counts (all experts).
  pf_groups_kernel<<<1, PF_PLAN_THREADS, 0, s>>>(
      counts, E, a->layer_cap > 0 ? a->layer_cap : E,
      a->max_assignments > 0 ? a->max_assignments : 32768, (int32_t *)W(L.group_of));
  if ((rc = check_launch("pf_groups_kernel")) != VB_OK) return rc;
  const int n = T * k + (has_shared ? T : 0);
  int32_t *r_row = (int32_t *)W(L.r_row), *r_exp = (int32_t *)W(L.r_exp);
  float *r_score = (float *)W(L.r_score);
  pf_routes_kernel<<<(n + 255) / 256, 256, 0, s>>>(T, k, E, has_shared ? 1 : 0, inds, scores, r_row,
                                                   r_exp, r_score);
  if ((rc = check_launch("pf_routes_kernel")) != VB_OK) return rc;
  const ExpertsLayout &X = L.X;
  uint8_t *xw = W(L.experts);
  // expert counts: routed from the top-k histogram, shared = T
  if (cudaMemcpyAsync(xw + X.counts, counts, (size_t)E * 4, cudaMemcpyDeviceToDevice, s) !=
      cudaSuccess)
    return set_error(VB_ERR_CUDA, "prefill: counts copy");
  pf_set_kernel<<<1, 1, 0, s>>>((int32_t *)(xw + X.counts) + E, has_shared ? T : 0);
  if ((rc = check_launch("pf_set_kernel")) != VB_OK) return rc;
  if ((rc = run_experts(a->x, T, r_row, r_exp, r_score, n, H, I, E, gshift, a->slot_table,
                        a->pool, a->shared, has_shared, a->status, xw, X, s, true)) != VB_OK)
    return rc;
  const int32_t *pos_of = (const int32_t *)(xw + X.pos_of);
  const uint16_t *ys = (const uint16_t *)(xw + X.ys);
  pf_combine_kernel<<<(T + 7) / 8, 256, 0, s>>>(ys, T, H, k, inds, (const int32_t *)W(L.group_of),
                                                pos_of, has_shared ? ys : nullptr,
                                                has_shared ? pos_of + (size_t)T * k : nullptr, sgate,
                                                a->out);
  return check_launch("pf_combine_kernel");
}

size_t vb_moe_route_workspace_size(int32_t tokens, int32_t hidden, int32_t num_experts) {
  if (tokens <= 0 || hidden <= 0 || num_experts <= 0) return 0;
  return route_layout(tokens, hidden, num_experts).total;
}

int vb_moe_route(const VbMoeRouteArgs *a, vb_stream_t stream) {
  VB_REQUIRE(a, "vb_moe_route: null args");
  const int T = a->tokens, H = a->hidden, E = a->num_experts, k = a->top_k;
  VB_REQUIRE(T >= 1 && H % 256 == 0 && H >= 256 && H <= 8192, "vb_moe_route: shape");
  VB_REQUIRE(E >= k && E < PF_PLAN_THREADS && k >= 1 && k <= 16, "vb_moe_route: experts/top_k");
  VB_REQUIRE(a->x && a->router_w && a->out_inds && a->out_scores && a->out_counts,
             "vb_moe_route: null tensor");
  VB_REQUIRE(!a->shared_gate_w || a->out_sgate, "vb_moe_route: shared gate without output");
  const size_t need = route_layout(T, H, E).total;
  VB_REQUIRE(a->workspace && a->workspace_bytes >= need && ((uintptr_t)a->workspace % 1024) == 0,
             "vb_moe_route: workspace %zu < %zu (1024-byte aligned)", a->workspace_bytes, need);
  return run_route(a->x, T, H, E, k, a->norm_topk, a->router_w, a->router_bias, a->shared_gate_w,
                   nullptr, 0, a->out_inds, a->out_scores, a->out_sgate, a->out_counts, nullptr,
                   nullptr, a->out_logits, a->status, static_cast<uint8_t *>(a->workspace),
                   as_stream(stream));
}

size_t vb_moe_experts_workspace_size(int32_t routes, int32_t hidden, int32_t inter,
                                     int32_t num_experts) {
  if (routes < 0 || hidden <= 0 || inter <= 0 || num_experts <= 0) return 0;
  return experts_layout(routes, hidden, inter, num_experts).total;
}

int vb_moe_experts(const VbMoeExpertsArgs *a, vb_stream_t stream) {
  VB_REQUIRE(a, "vb_moe_experts: null args");
  const int n = a->routes, H = a->hidden, I = a->inter, E = a->num_experts;
  VB_REQUIRE(n >= 0 && a->rows >= 0, "vb_moe_experts: sizes");
  VB_REQUIRE(a->bits == 4 && (a->group == 64 || a->group == 128), "vb_moe_experts: format");
  VB_REQUIRE(H % 256 == 0 && H >= 256 && H <= 8192 && I % 128 == 0 && I >= 128 && I <= 4096,
             "vb_moe_experts: hidden/inter");
  VB_REQUIRE(E >= 1 && E < PF_PLAN_THREADS, "vb_moe_experts: num_experts");
  VB_REQUIRE(n == 0 || (a->x && a->route_row && a->route_expert && a->route_score && a->out),
             "vb_moe_experts: null tensor");
  VB_REQUIRE(a->slot_table, "vb_moe_experts: null slot table");
  const bool has_shared = a->shared.ptr[0] != nullptr;
  int rc;
  if ((rc = check_pool(a->pool, a->shared, has_shared, "vb_moe_experts")) != VB_OK) return rc;
  const ExpertsLayout L = experts_layout(n, H, I, E);
  VB_REQUIRE(a->workspace && a->workspace_bytes >= L.total && ((uintptr_t)a->workspace % 1024) == 0,
             "vb_moe_experts: workspace %zu < %zu (1024-byte aligned)", a->workspace_bytes, L.total);
  if (n == 0) return VB_OK;
  cudaStream_t s = as_stream(stream);
  uint8_t *ws = static_cast<uint8_t *>(a->workspace);
  if ((rc = run_experts(a->x, a->rows, a->route_row, a->route_expert, a->route_score, n, H, I, E,
                        a->group == 128 ? 1 : 0, a->slot_table, a->pool, a->shared, has_shared,
                        a->status, ws, L, s, false)) != VB_OK)
    return rc;
  pf_unsort_kernel<<<(n + 7) / 8, 256, 0, s>>>((const uint16_t *)(ws + L.ys), H, n,
                                               (const int32_t *)(ws + L.pos_of), a->out);
  return check_launch("pf_unsort_kernel");
}

int vb_moe_combine(const VbMoeCombineArgs *a, vb_stream_t stream) {
  VB_REQUIRE(a, "vb_moe_combine: null args");
  const int T = a->tokens, H = a->hidden, E = a->num_experts, k = a->top_k;
  VB_REQUIRE(T >= 1 && H % 256 == 0 && E >= k && E < PF_PLAN_THREADS && k >= 1 && k <= 16,
             "vb_moe_combine: shape");
  VB_REQUIRE(a->inds && a->counts && a->y_routes && a->route_row && a->out && a->group_of_ws,
             "vb_moe_combine: null tensor");
  VB_REQUIRE(!a->y_shared || a->sgate, "vb_moe_combine: shared rows without gate");
  cudaStream_t s = as_stream(stream);
  pf_groups_kernel<<<1, PF_PLAN_THREADS, 0, s>>>(a->counts, E, a->layer_cap > 0 ? a->layer_cap : E,
                                                 a->max_assignments > 0 ? a->max_assignments : 32768,
                                                 a->group_of_ws);
  int rc;
  if ((rc = check_launch("pf_groups_kernel")) != VB_OK) return rc;
  pf_combine_kernel<<<(T + 7) / 8, 256, 0, s>>>(a->y_routes, T, H, k, a->inds, a->group_of_ws,
                                                a->route_row, a->y_shared, a->shared_row, a->sgate,
                                                a->out);
  return check_launch("pf_combine_kernel");
}

size_t vb_ep_pack_workspace_size(int32_t tokens, int32_t world) {
  if (tokens <= 0 || world <= 0) return 0;
  return align_up((size_t)tokens * world * 4, 256) * 3;
}

int vb_ep_pack(const VbEpPackArgs *a, vb_stream_t stream) {
  VB_REQUIRE(a, "vb_ep_pack: null args");
  const int T = a->tokens, k = a->top_k, H = a->hidden, N = a->world;
  VB_REQUIRE(T >= 1 && k >= 1 && k <= 32 && H % 8 == 0 && N >= 1 && N <= EP_MAX_WORLD,
             "vb_ep_pack: shape");
  VB_REQUIRE(a->x && a->inds && a->scores && a->owner && a->send_x && a->send_meta &&
                 a->route_send_idx && a->dest_rows && a->dest_routes,
             "vb_ep_pack: null tensor");
  const size_t seg = align_up((size_t)T * N * 4, 256);
  VB_REQUIRE(a->workspace && a->workspace_bytes >= 3 * seg, "vb_ep_pack: workspace");
  uint8_t *ws = static_cast<uint8_t *>(a->workspace);
  int32_t *tok_cnt = (int32_t *)ws, *row_idx = (int32_t *)(ws + seg),
          *route_base = (int32_t *)(ws + 2 * seg);
  cudaStream_t s = as_stream(stream);
  int rc;
  ep_count_kernel<<<(T + 255) / 256, 256, 0, s>>>(a->inds, a->owner, T, k, N, tok_cnt);
  if ((rc = check_launch("ep_count_kernel")) != VB_OK) return rc;
  ep_scan_kernel<<<N, 1024, 0, s>>>(tok_cnt, T, N, row_idx, route_base, a->dest_rows,
                                    a->dest_routes);
  if ((rc = check_launch("ep_scan_kernel")) != VB_OK) return rc;
  ep_pack_kernel<<<(T + 7) / 8, 256, 0, s>>>(a->x, a->inds, a->scores, a->owner, T, k, H, N,
                                             tok_cnt, row_idx, route_base, a->dest_rows,
                                             a->dest_routes, a->send_x, a->send_meta,
                                             a->route_send_idx);
  return check_launch("ep_pack_kernel");
}

int vb_ep_unpack(const int32_t *recv_meta, int32_t routes, const int32_t *src_route_off,
                 const int32_t *src_row_off, int32_t world, int32_t *route_row,
                 int32_t *route_expert, float *route_score, vb_stream_t stream) {
  VB_REQUIRE(routes >= 0 && world >= 1 && world <= EP_MAX_WORLD, "vb_ep_unpack: shape");
  if (routes == 0) return VB_OK;
  VB_REQUIRE(recv_meta && src_route_off && src_row_off && route_row && route_expert && route_score,
             "vb_ep_unpack: null tensor");
  ep_unpack_kernel<<<(routes + 255) / 256, 256, 0, as_stream(stream)>>>(
      recv_meta, routes, src_route_off, src_row_off, world, route_row, route_expert, route_score);
  return check_launch("ep_unpack_kernel");
}

}  // extern "C"
