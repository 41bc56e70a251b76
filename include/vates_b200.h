/*
 * vates_b200 — C ABI of the B200 (sm_100a) kernels for the AMOS144/Vates hot
 * path: fused quantized MoE, pool slot-table gather, IsoQuant K4/V3 KV cache.
 *
 * Conventions
 *  - Every pointer argument is a device pointer unless documented otherwise.
 *  - bf16 tensors are passed as uint16_t (raw bf16 bits), like the reference
 *    extension, which keeps scales/biases as uint16 holding bf16 bits
 *    (mlx_streaming/core/moe/native_moe.py:57-72).
 *  - `stream` is a cudaStream_t (CUstream) handle; NULL is the legacy stream.
 *  - Functions return VB_OK (0) or an error code; vb_last_error() gives the
 *    message of the calling thread's last failing call. No function throws,
 *    allocates device memory, or synchronises the stream unless stated.
 *  - Conditions only the device can see (a routed expert whose slot is -1,
 *    an out-of-range id) are OR-ed as VB_STATUS_* bits into the optional
 *    device int32 `status` word; the host reads it when it chooses.
 *  - Scratch memory is supplied by the caller (`workspace`), sized by the
 *    matching *_workspace_size() query.
 */
#ifndef VATES_B200_H
#define VATES_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

typedef void *vb_stream_t;

enum {
  VB_OK = 0,
  VB_ERR_INVALID = 1,   /* bad argument or unsupported shape */
  VB_ERR_CUDA = 2,      /* CUDA runtime error while launching */
  VB_ERR_WORKSPACE = 3, /* workspace too small */
  VB_ERR_CAPACITY = 4,  /* residency request does not fit the layer's slots */
};

/* Device status bits (OR-ed into *status by kernels). */
enum {
  VB_STATUS_MISS = 1,     /* routed expert not resident (slot -1) */
  VB_STATUS_BOUNDS = 2,   /* id or slot out of range; access skipped */
  VB_STATUS_TIMEOUT = 4,  /* a bounded inter-CTA wait gave up */
};

int vb_version(void);
const char *vb_last_error(void);

/* Nine-tensor quantized expert pool, MLX affine format (uint32-packed codes,
 * continuous LSB-first bitstream per row; bf16 scale and bias per group).
 * Order: gate_w, gate_s, gate_b, up_w, up_s, up_b, down_w, down_s, down_b.
 * ptr[i] + slot * slot_stride[i] is the start of that slot's tensor, so both
 * the reference's nine stacked arrays [cap, out, ...] (fused_moe.cpp:635-664)
 * and one packed blob row per expert (prep/blob_layout.py:14-32) are
 * described. gate/up are [inter, hidden*bits/32] words, down is
 * [hidden, inter*bits/32] words; scale/bias rows are [out, in/group]. */
typedef struct VbQuantPool {
  const void *ptr[9];
  int64_t slot_stride[9]; /* bytes */
  int32_t cap;            /* number of slots */
  int32_t reserved;
} VbQuantPool;

/* ---------------------------------------------------------------------------
 * Pool slot-table gather.
 * Replaces demand_gpu_remap_only (native/ext/pool/demand.cpp:1954-1970,
 * Metal kernel demand_gpu_remap 1201-1232) and the mx.take of
 * ResidentExpertPool.acquire_gpu (mlx_streaming/core/cache/resident_pool.py:
 * 560-569). local[i] = table[ids[i]] (-1 = not resident). Ids outside
 * [0, table_size) give -1 and VB_STATUS_BOUNDS. miss_count (nullable) is
 * incremented once per -1 produced. */
int vb_slot_remap(const uint32_t *ids, const int32_t *table, int32_t *local,
                  int64_t n, int32_t table_size, int32_t *miss_count,
                  int32_t *status, vb_stream_t stream);

/* ---------------------------------------------------------------------------
 * Fused MoE, float32 native-extension semantics.
 * vb_fused_moe_slots replaces fused_moe_slots (native/ext/compute/
 * fused_moe.cpp:635-664, bindings.cpp:300-320): x f32 [tokens, hidden],
 * local_slots u32 [tokens*k], scores f32 [tokens*k], out f32 [tokens, hidden];
 * pair p uses token p/k and pool slot local_slots[p]; out[t] =
 * sum_j y[t*k+j] * scores[t*k+j] (reduce_pairs, fused_moe.cpp:284-298).
 * local_slots == NULL selects the staged variant, pair p -> slot p
 * (fused_moe_staged, fused_moe.cpp:605-633, bindings.cpp:31-50).
 * bits in {2,3,4,5,6,8}; (hidden*bits)%32 == (inter*bits)%32 == 0;
 * hidden and inter multiples of group. */
size_t vb_fused_moe_workspace_size(int32_t pairs, int32_t inter);
int vb_fused_moe_slots(const float *x, const uint32_t *local_slots,
                       const float *scores, const VbQuantPool *pool,
                       int32_t tokens, int32_t k, int32_t hidden,
                       int32_t inter, int32_t group, int32_t bits, float *out,
                       int32_t *status, void *workspace, size_t workspace_bytes,
                       vb_stream_t stream);

/* Per-pair fused expert (no combine): replaces _custom_fused_moe_indexed
 * (mlx_streaming/core/moe/custom_kernel.py:226-383). x f32 [pairs, hidden]
 * (one row per pair), indices u32 [pairs], active_mask u8 [pairs] nullable
 * (0 -> zero row), y f32 [pairs, hidden]. */
int vb_fused_moe_pairs(const float *x, const uint32_t *indices,
                       const uint8_t *active_mask, const VbQuantPool *pool,
                       int32_t pairs, int32_t hidden, int32_t inter,
                       int32_t group, int32_t bits, float *y, int32_t *status,
                       void *workspace, size_t workspace_bytes,
                       vb_stream_t stream);

/* ---------------------------------------------------------------------------
 * Whole decode / MTP-verify MoE block, T <= 8 tokens, MLX bf16 dtype chain.
 * Replaces FileStreamingMoeBlock.__call__ for decode (mlx_streaming/core/moe/
 * block.py:245-1013): router GEMV (block.py:253) -> precise softmax -> top-k
 * -> renormalise (321-329) -> slot gather (resident_pool.py:560-569) ->
 * gate/up -> SwiGLU -> down (compute.py:145-199) -> weighted combine
 * (block.py:1008) -> + sigmoid(x.w_sg) * shared_expert(x) (1009-1012).
 * 4-bit weights, group 64 or 128, hidden in {512, 1024, 2048, 4096}, inter
 * in {128, 256, 512}. One persistent kernel with one CTA per SM; its CTAs
 * synchronise through the workspace with bounded waits (2 s, then
 * VB_STATUS_TIMEOUT), so it needs every SM's share of the GPU. */
typedef struct VbMoeDecodeArgs {
  int32_t tokens;       /* T, 1..8 */
  int32_t hidden;       /* H */
  int32_t inter;        /* I (routed and shared experts) */
  int32_t group;        /* 64 or 128 */
  int32_t bits;         /* 4 */
  int32_t num_experts;  /* E <= 1024 */
  int32_t top_k;        /* k <= 16 */
  int32_t norm_topk;    /* renormalise the top-k scores */
  float norm_eps;       /* > 0: the block input is rmsnorm(x) (unit weight,
                           float32 math, bf16 result); 0: x as given */
  int32_t flags;        /* VB_DECODE_* bits, 0 for the whole block */
  const uint16_t *x;            /* bf16 [T, H]; x, residual and out are
                                   16-byte aligned */
  const uint16_t *router_w;     /* bf16 [E, H] */
  const float *router_bias;     /* nullable f32 [E], added before rounding */
  const int32_t *slot_table;    /* [E], -1 = not resident */
  VbQuantPool pool;             /* routed experts */
  VbQuantPool shared;           /* shared expert in slot 0; ptr[0]==NULL: none */
  const uint16_t *shared_gate_w; /* bf16 [H] */
  const uint16_t *residual;     /* nullable bf16 [T, H]: out = residual + moe */
  uint16_t *out;                /* bf16 [T, H] */
  int32_t *out_inds;            /* nullable [T, k] expert ids */
  uint16_t *out_scores;         /* nullable bf16 [T, k] */
  int32_t *out_local;           /* nullable [T, k] pool slots */
  int32_t *status;              /* nullable device status word */
  void *workspace;
  size_t workspace_bytes;
  void *const *timing_events;   /* nullable: 2 cudaEvent_t recorded before
                                   and after the layer kernel; the launch
                                   then leaves the PDL chain (profiling only) */
  uint64_t *trace;              /* nullable device [16] %globaltimer (ns)
                                   markers of the layer kernel (profiling
                                   only): [0] min CTA start, [1] max CTA end,
                                   initialised by the caller to
                                   (UINT64_MAX, 0); latest CTA past the PDL
                                   wait [2], done with its router rows [3],
                                   past the grid barrier [4], done routing
                                   [5]; latest warp done with gate/up [6],
                                   with its down items [7], with its
                                   combines [8]; [2..15] initialised to 0 */
} VbMoeDecodeArgs;

/* flags: VB_DECODE_ROUTE_ONLY stops after routing: out_inds, out_scores,
 * out_local and the status bits (VB_STATUS_MISS for a routed expert without a
 * slot) are written; out is not. The same routing as the whole-block call, so
 * a demand on its ids followed by the whole-block call sees no miss. */
enum { VB_DECODE_ROUTE_ONLY = 1 };

/* The decode workspace must be zero-filled before its first use; every call
 * leaves it reusable by the next call on the same stream with the same
 * hidden size (any tokens, inter, experts, top_k within its size; after a
 * call that reported VB_STATUS_TIMEOUT it must be zero-filled again). Calls
 * sharing one workspace must not overlap on the GPU. */
size_t vb_moe_decode_workspace_size(int32_t tokens, int32_t hidden,
                                    int32_t inter, int32_t num_experts,
                                    int32_t top_k);
int vb_moe_decode(const VbMoeDecodeArgs *args, vb_stream_t stream);

/* Decode block without a caller workspace. No counterpart in the reference:
 * this is for callers that cannot allocate device memory for scratch, such
 * as a host framework that owns every device buffer through its own pool
 * and hands a plugin only the tensors of the op, or a latency-critical
 * decode loop that must not call cudaMalloc (which can synchronise the
 * device). The scratch is one fixed device array inside this library of
 * VB_MOE_DECODE_NOALLOC_SCRATCH_BYTES; shapes whose
 * vb_moe_decode_workspace_size exceeds it are rejected with
 * VB_ERR_WORKSPACE and a message naming both sizes.
 * args->workspace and args->workspace_bytes are ignored. Apart from that it
 * computes exactly what vb_moe_decode computes.
 * - The first call on a device (current device at the call) looks up the
 *   array's device address once; make that first call before any stream
 *   capture on that device. The address belongs to the device's primary
 *   context: do not call this entry point again after cudaDeviceReset.
 * - Every call clears the array's counters on `stream` before its kernels
 *   and allocates nothing (no cudaMalloc, cudaFree or allocating library).
 * - All calls on a device share the one array, which keeps the last call's
 *   contents: calls that can overlap on the GPU (other streams, other
 *   threads) race on it; serialise them on one stream. */
#define VB_MOE_DECODE_NOALLOC_SCRATCH_BYTES (2u << 20)
int vb_moe_decode_noalloc(const VbMoeDecodeArgs *args, vb_stream_t stream);

/* ---------------------------------------------------------------------------
 * Expert-major prefill of one sparse-MoE block (T tokens, any T >= 1).
 * Replaces the prefill branch of FileStreamingMoeBlock.__call__
 * (mlx_streaming/core/moe/block.py:318-347) and _expert_major_forward
 * (block.py:111-243): router -> precise softmax -> top-k -> renormalise ->
 * per-expert grouped gate/up -> SwiGLU -> down (gather_qmm matrix path,
 * compute.py:156-199; dequantized weights rounded once to bf16) -> y * score
 * -> reduce in the reference's order (expert group of block.py:154-172, then
 * route rank; bf16 rounding after every add, custom_kernel.py:63-77) ->
 * + bf16(sigmoid(x.w_sg) * shared_expert(x)) (block.py:345-346).
 * 4-bit weights, group 64 or 128; hidden % 256 == 0, inter % 128 == 0.
 * Routed experts whose slot is -1 are skipped (VB_STATUS_MISS). The
 * workspace (vb_moe_prefill_workspace_size) is 1024-byte aligned; its
 * contents need no initialisation. */
typedef struct VbMoePrefillArgs {
  int32_t tokens;
  int32_t hidden;
  int32_t inter;
  int32_t group;
  int32_t bits;
  int32_t num_experts;
  int32_t top_k;
  int32_t norm_topk;
  int32_t layer_cap;        /* experts per reduce group: min(layer_cap, 128);
                               <= 0: num_experts (block.py:154) */
  int32_t max_assignments;  /* routes per reduce group; <= 0: 32768 (155) */
  const uint16_t *x;            /* bf16 [T, H] */
  const uint16_t *router_w;     /* bf16 [E, H] */
  const float *router_bias;     /* nullable f32 [E], added before rounding */
  const int32_t *slot_table;    /* [E], -1 = not resident */
  VbQuantPool pool;
  VbQuantPool shared;           /* ptr[0] == NULL: no shared expert */
  const uint16_t *shared_gate_w; /* bf16 [H] */
  uint16_t *out;                /* bf16 [T, H] */
  int32_t *out_inds;            /* nullable [T, k] */
  uint16_t *out_scores;         /* nullable bf16 [T, k] */
  uint16_t *out_logits;         /* nullable bf16 [T, E] router logits */
  int32_t *status;              /* nullable device status word */
  void *workspace;
  size_t workspace_bytes;
} VbMoePrefillArgs;

size_t vb_moe_prefill_workspace_size(int32_t tokens, int32_t hidden,
                                     int32_t inter, int32_t num_experts,
                                     int32_t top_k);
int vb_moe_prefill(const VbMoePrefillArgs *args, vb_stream_t stream);

/* ---------------------------------------------------------------------------
 * Phases of the expert-major prefill, for callers that place experts
 * themselves (the expert-parallel prefill: every rank owns a subset of the
 * experts). vb_moe_prefill = route + experts + combine on one device.
 *
 * vb_moe_route: router GEMM, precise softmax, top-k, renormalisation for T
 * tokens (block.py:253, 321-329) and the route histogram (block.py:142-144;
 * out_counts[E] overwritten, [E] entries). out_scores are bf16 values stored
 * as f32; out_sgate (when shared_gate_w is given) = bf16(sigmoid(x.w_sg)). */
typedef struct VbMoeRouteArgs {
  int32_t tokens;
  int32_t hidden;
  int32_t num_experts;
  int32_t top_k;
  int32_t norm_topk;
  int32_t reserved0;
  const uint16_t *x;            /* bf16 [T, H] */
  const uint16_t *router_w;     /* bf16 [E, H] */
  const float *router_bias;     /* nullable f32 [E] */
  const uint16_t *shared_gate_w; /* nullable bf16 [H] */
  int32_t *out_inds;            /* [T, k] */
  float *out_scores;            /* [T, k] */
  float *out_sgate;             /* [T] when shared_gate_w */
  int32_t *out_counts;          /* [E + 1] (entry E left 0) */
  uint16_t *out_logits;         /* nullable bf16 [T, E] */
  int32_t *status;
  void *workspace;              /* vb_moe_route_workspace_size, 1024-aligned */
  size_t workspace_bytes;
} VbMoeRouteArgs;
size_t vb_moe_route_workspace_size(int32_t tokens, int32_t hidden,
                                   int32_t num_experts);
int vb_moe_route(const VbMoeRouteArgs *args, vb_stream_t stream);

/* vb_moe_experts: the per-group expert work of _expert_major_forward
 * (block.py:206-216: gather rows, gather_qmm gate/up -> SwiGLU -> down,
 * y * score) for an arbitrary route list. Route i reads row route_row[i] of
 * x, runs expert route_expert[i] (num_experts = the shared expert, < 0 =
 * skipped) and writes bf16(bf16(y) * route_score[i]) to row i of out (zeros
 * for skipped routes or experts without a slot). */
typedef struct VbMoeExpertsArgs {
  int32_t rows;                 /* rows of x */
  int32_t routes;
  int32_t hidden;
  int32_t inter;
  int32_t group;
  int32_t bits;                 /* 4 */
  int32_t num_experts;
  int32_t reserved0;
  const uint16_t *x;            /* bf16 [rows, H] */
  const int32_t *route_row;     /* [routes] */
  const int32_t *route_expert;  /* [routes] */
  const float *route_score;     /* [routes] */
  const int32_t *slot_table;    /* [E], -1 = not resident on this device */
  VbQuantPool pool;
  VbQuantPool shared;           /* ptr[0] == NULL: no shared expert */
  uint16_t *out;                /* bf16 [routes, H] */
  int32_t *status;
  void *workspace;              /* vb_moe_experts_workspace_size, 1024-aligned */
  size_t workspace_bytes;
} VbMoeExpertsArgs;
size_t vb_moe_experts_workspace_size(int32_t routes, int32_t hidden,
                                     int32_t inter, int32_t num_experts);
int vb_moe_experts(const VbMoeExpertsArgs *args, vb_stream_t stream);

/* vb_moe_combine: the reduce of _expert_major_forward (block.py:220 with
 * deterministic_route_reduce, custom_kernel.py:63-77) and the shared expert
 * add (block.py:345-346). Per token the k routed rows y_routes[route_row[t*k
 * + j]] (route_row -1 = skipped) are added from zero in the order (reference
 * group of the expert, route rank j), rounding to bf16 after every add; the
 * groups come from `counts`, the route histogram of the WHOLE prefill batch
 * (all ranks), with layer_cap / max_assignments as in VbMoePrefillArgs. Then
 * + bf16(sgate[t] * y_shared[shared_row ? shared_row[t] : t]). */
typedef struct VbMoeCombineArgs {
  int32_t tokens;
  int32_t hidden;
  int32_t num_experts;
  int32_t top_k;
  int32_t layer_cap;
  int32_t max_assignments;
  const int32_t *inds;          /* [T, k] */
  const int32_t *counts;        /* [E] */
  const uint16_t *y_routes;     /* bf16 rows */
  const int32_t *route_row;     /* [T, k] */
  const uint16_t *y_shared;     /* nullable bf16 rows */
  const int32_t *shared_row;    /* nullable [T] */
  const float *sgate;           /* [T] when y_shared */
  uint16_t *out;                /* bf16 [T, H] */
  int32_t *group_of_ws;         /* device scratch [E] */
} VbMoeCombineArgs;
int vb_moe_combine(const VbMoeCombineArgs *args, vb_stream_t stream);

/* Expert-parallel dispatch (no counterpart in the reference, which runs on
 * one device). vb_ep_pack: for T local tokens and owner[e] = rank holding
 * expert e, packs the rows to send (each token row once per destination
 * rank; destination-major, tokens ascending) and the route metadata
 * (row in the destination's chunk, expert, score bits; routes (t, j)
 * ascending), and returns per-destination row / route counts and, per local
 * route, its index in the send order. Buffers are sized for the worst case:
 * send_x [T * min(k, world), H], send_meta [T * k, 3]. */
typedef struct VbEpPackArgs {
  int32_t tokens;
  int32_t top_k;
  int32_t hidden;
  int32_t world;                /* <= 8 */
  const uint16_t *x;            /* bf16 [T, H] */
  const int32_t *inds;          /* [T, k] */
  const float *scores;          /* [T, k] */
  const int32_t *owner;         /* [E] */
  uint16_t *send_x;
  int32_t *send_meta;
  int32_t *route_send_idx;      /* [T, k] */
  int32_t *dest_rows;           /* [world] */
  int32_t *dest_routes;         /* [world] */
  void *workspace;              /* vb_ep_pack_workspace_size */
  size_t workspace_bytes;
} VbEpPackArgs;
size_t vb_ep_pack_workspace_size(int32_t tokens, int32_t world);
int vb_ep_pack(const VbEpPackArgs *args, vb_stream_t stream);
/* Received routes -> (row of the received rows, expert, score): source s
 * sent routes [src_route_off[s], src_route_off[s+1]) whose rows start at
 * src_row_off[s] in the received rows. */
int vb_ep_unpack(const int32_t *recv_meta, int32_t routes,
                 const int32_t *src_route_off, const int32_t *src_row_off,
                 int32_t world, int32_t *route_row, int32_t *route_expert,
                 float *route_score, vb_stream_t stream);

/* ---------------------------------------------------------------------------
 * Expert-parallel expert-major prefill over NCCL (one rank per GPU): the
 * prefill branch of FileStreamingMoeBlock.__call__ (mlx_streaming/core/moe/
 * block.py:330-347) and _expert_major_forward (block.py:111-243) with the
 * experts spread over the ranks. Every rank calls it with its own tokens
 * (base.tokens, base.x, base.out) and the experts it holds (base.pool and
 * base.slot_table, -1 for experts it does not hold); owner[e] is the rank
 * that computes expert e for this rank's routes (experts held by every rank
 * map to the caller's own rank). Schedule on `stream`: route, all-reduce of
 * the route histogram, pack, count exchange (read on the host: the call
 * synchronises the stream once), grouped ncclSend/ncclRecv of token rows and
 * route metadata, the rank's experts and the shared expert, the weighted
 * route rows back, the reference-order reduce. The output is bit-identical
 * to vb_moe_prefill on one device for any world size and placement.
 * nccl_comm is an ncclComm_t of `world` ranks (this process is `rank`); NCCL
 * is resolved at run time from the loaded libnccl.so.2. Every rank must make
 * the call with the same world, experts and top_k. The workspace
 * (vb_moe_prefill_ep_workspace_size, 1024-byte aligned) covers the worst
 * case, every route of every rank sent to this rank: max_tokens_per_rank is
 * the largest token count of any rank. */
typedef struct VbMoePrefillEpArgs {
  VbMoePrefillArgs base;
  const int32_t *owner;         /* device [E] */
  int32_t world;                /* <= 8 */
  int32_t rank;
  int32_t max_tokens_per_rank;
  int32_t reserved;
} VbMoePrefillEpArgs;
size_t vb_moe_prefill_ep_workspace_size(int32_t tokens, int32_t hidden,
                                        int32_t inter, int32_t num_experts,
                                        int32_t top_k, int32_t world,
                                        int32_t max_tokens_per_rank);
int vb_moe_prefill_ep(const VbMoePrefillEpArgs *args, void *nccl_comm,
                      vb_stream_t stream);

/* ---------------------------------------------------------------------------
 * Deterministic route reduce: replaces deterministic_route_reduce
 * (mlx_streaming/core/moe/custom_kernel.py:20-118). previous [tokens, H],
 * weighted [G, H], assignment_pos int32 [G] (unique flat route positions in
 * [0, tokens*k)); out [tokens, H] (may alias previous). For each token the
 * routes present are added in ascending route rank to previous[token], with
 * a rounding to the output dtype after each add. dtype: 0 = f32, 1 = bf16. */
size_t vb_route_reduce_workspace_size(int32_t tokens, int32_t k);
int vb_route_reduce(const void *previous, const void *weighted,
                    const int32_t *assignment_pos, int32_t groups,
                    int32_t tokens, int32_t hidden, int32_t k, int32_t dtype,
                    void *out, int32_t *status, void *workspace,
                    size_t workspace_bytes, vb_stream_t stream);

/* ---------------------------------------------------------------------------
 * IsoQuant KV append: rotate (optional) + quantize + pack rows into a cache.
 * Replaces rotate_last (mlx_streaming/core/cache/quant_kv.py:68-70) on k/v and
 * mx.quantize + slice-assign of AsymmetricQuantizedKVCache.update_and_fetch
 * (quant_kv.py:105-137). src bf16 [B, H, n, D] contiguous; so4_blocks f32
 * [D/4, 4, 4] (rounded to bf16 inside) or NULL for no rotation; codes u32
 * [B, H, cap, D*bits/32], scales/biases bf16 [B, H, cap, D/group]; rows are
 * written at sequence positions [offset, offset+n). D in {64,128,256},
 * group 64, bits in {2,3,4,5,6,8}. */
int vb_kv_quant_append(const uint16_t *src, const float *so4_blocks,
                       int32_t batch, int32_t heads, int32_t n, int32_t dim,
                       int32_t group, int32_t bits, int32_t offset,
                       int32_t cap, uint32_t *codes, uint16_t *scales,
                       uint16_t *biases, vb_stream_t stream);

/* The same with the row offset read on the device (*offset; rows past cap
 * are skipped and flag VB_STATUS_BOUNDS in the nullable status word). */
int vb_kv_quant_append_at(const uint16_t *src, const float *so4_blocks,
                          int32_t batch, int32_t heads, int32_t n, int32_t dim,
                          int32_t group, int32_t bits, const int32_t *offset,
                          int32_t cap, uint32_t *codes, uint16_t *scales,
                          uint16_t *biases, int32_t *status, vb_stream_t stream);

/* Rotation only: dst = src @ R (4x4 SO(4) blocks, R rounded to bf16),
 * bf16 [rows, D]; transpose != 0 applies R^T (quant_kv.py:68-70 with Rv.T,
 * kv_quant_patch.py:67-68). */
int vb_so4_rotate(const uint16_t *src, const float *so4_blocks, int64_t rows,
                  int32_t dim, int32_t transpose, uint16_t *dst,
                  vb_stream_t stream);

/* Quantized GQA attention over a packed cache: replaces asym_quantized_sdpa
 * (quant_kv.py:212-249) plus the inverse V rotation (kv_quant_patch.py:
 * 67-68) when rv_blocks != NULL. q bf16 [B, Hq, L, D] (already rotated);
 * K: codes [B, Hkv, cap, D*k_bits/32], scales/biases [B, Hkv, cap, D/group];
 * V likewise with v_bits. keys = valid sequence length; causal: query i of L
 * sees keys <= keys-L+i. out bf16 [B, Hq, L, D]. L <= 4, Hq/Hkv <= 8 and
 * (Hq/Hkv)*L <= 32; D = 256, group 64, k_bits 4, v_bits 3. */
size_t vb_kv_attn_workspace_size(int32_t batch, int32_t q_heads, int32_t L,
                                 int32_t dim, int32_t keys);
int vb_kv_decode_attn(const uint16_t *q, const uint32_t *k_codes,
                      const uint16_t *k_scales, const uint16_t *k_biases,
                      const uint32_t *v_codes, const uint16_t *v_scales,
                      const uint16_t *v_biases, const float *rv_blocks,
                      int32_t batch, int32_t q_heads, int32_t kv_heads,
                      int32_t L, int32_t dim, int32_t keys, int32_t cap,
                      int32_t group, int32_t k_bits, int32_t v_bits,
                      float scale, int32_t causal, uint16_t *out,
                      void *workspace, size_t workspace_bytes,
                      vb_stream_t stream);

/* The same with the key count read on the device: keys = *pos + L (pos =
 * cache length before this step's L rows); keys_max (<= cap) sizes the split
 * grid, so one launch (and one CUDA graph node) serves every step. Used by the
 * decode stack, whose cache offset lives in device memory. With gate_proj
 * (batch 1) the output gate of the attention layer is applied in the same
 * pass (kv_quant_patch.py:70-71, = vb_attn_gate): out bf16 [L, Hq * 256] =
 * bf16(o * bf16(sigmoid(g))), g = gate_proj[l * gate_stride + hq * 512 + 256
 * + d] (the gate half of each query head's projection); without it, out bf16
 * [B, Hq, L, 256] = o. */
int vb_kv_decode_attn_at(const uint16_t *q, const uint32_t *k_codes,
                         const uint16_t *k_scales, const uint16_t *k_biases,
                         const uint32_t *v_codes, const uint16_t *v_scales,
                         const uint16_t *v_biases, const float *rv_blocks,
                         int32_t batch, int32_t q_heads, int32_t kv_heads,
                         int32_t L, int32_t dim, const int32_t *pos, int32_t keys_max,
                         int32_t cap, int32_t group, int32_t k_bits, int32_t v_bits,
                         float scale, int32_t causal, const uint16_t *gate_proj,
                         int32_t gate_stride, uint16_t *out, void *workspace,
                         size_t workspace_bytes, vb_stream_t stream);

/* GQA decode attention over a plain bf16 cache [B, Hkv, cap, 256] (the MTP
 * layer's mlx-lm KVCache attended by mx.fast.scaled_dot_product_attention,
 * mtp/qwen3_next_mtp.py:40-56): float32 scores, softmax and P V, one bf16
 * rounding. keys = *pos + pos_add + L, read on the device; q bf16
 * [B, Hq, L, 256]; out bf16 [B, Hq, L, 256], or the gated [L, Hq * 256] rows
 * with gate_proj as in vb_kv_decode_attn_at; (Hq/Hkv) * L <= 32. Workspace as
 * vb_kv_attn_workspace_size(batch, q_heads, L, dim, keys_max) + 256. */
int vb_kv_bf16_attn_at(const uint16_t *q, const uint16_t *k_cache, const uint16_t *v_cache,
                       int32_t batch, int32_t q_heads, int32_t kv_heads, int32_t L,
                       int32_t dim, const int32_t *pos, int32_t pos_add, int32_t keys_max,
                       int32_t cap, float scale, int32_t causal, const uint16_t *gate_proj,
                       int32_t gate_stride, uint16_t *out, void *workspace,
                       size_t workspace_bytes, vb_stream_t stream);

/* ---------------------------------------------------------------------------
 * Expert residency: per-layer expert -> slot state of a pool of `cap` slots
 * (host state machine, one mutex per manager).
 * Replaces the native demand path behind ResidentExpertPool
 * (mlx_streaming/core/cache/resident_pool.py:54-580; native/ext/pool/
 * demand.cpp). A slot is taken from the front of the free rows, else from the
 * LFU victim: the resident expert with the smallest access count, ties to the
 * earliest inserted, never pinned and never one of the current request
 * (choose_victim_locked 514-529, alloc_slot_locked 542-564). Counts go up by
 * one per unique expert of each demand and, with decay_interval > 0, halve
 * every decay_interval accesses (note_access_locked 566-637). lfu = 0 keeps
 * every count at zero, so the victim is the earliest inserted (FIFO). */
typedef struct VbResidency VbResidency;
VbResidency *vb_res_create(int32_t layers, int32_t cap, int32_t num_experts,
                           int32_t lfu, int32_t decay_interval);
void vb_res_destroy(VbResidency *r);
/* demand_core_locked (demand.cpp:966-1027): local[i] = slot of ids[i] after
 * the call. Every unique miss gets a slot; the (expert, slot) pairs to load
 * go to place_expert / place_slot (nullable, room for n) in first-miss order,
 * their count to *n_place. stats (nullable) = {hits, misses, loads}. When the
 * unique experts of ids plus the pinned experts not in ids exceed cap,
 * nothing is placed, local is all 0 and the call returns VB_ERR_CAPACITY
 * (the reference's over_capacity). */
int vb_res_demand(VbResidency *r, int32_t layer, const int32_t *ids, int32_t n,
                  int32_t *local, int32_t *place_expert, int32_t *place_slot,
                  int32_t *n_place, int64_t *stats);
/* real_pin (demand.cpp:364-394): pins the unique experts of `experts`
 * (first-seen order, count in *n_unique) and gives each a slot; placed[u] = 1
 * where the expert was not resident and must be loaded. VB_ERR_CAPACITY when
 * the pinned set would exceed cap (nothing changes). */
int vb_res_pin(VbResidency *r, int32_t layer, const int32_t *experts, int32_t n,
               int32_t *slots, int32_t *placed, int32_t *n_unique);
/* The layer's expert -> slot table (num_experts entries, -1 = not resident),
 * the table the slot-table gather and the decode kernel read
 * (real_table_set_locked, demand.cpp:306-318). */
int vb_res_table(VbResidency *r, int32_t layer, int32_t *table);
/* LFU access counts per expert (num_experts entries; the reference's
 * RealLayer::freq, demand.cpp:22-37). */
int vb_res_counts(VbResidency *r, int32_t layer, uint32_t *counts);
/* Resident (expert, slot) pairs in insertion order (nullable outputs with room
 * for cap; count in *n). */
int vb_res_resident(VbResidency *r, int32_t layer, int32_t *experts,
                    int32_t *slots, int32_t *n);

/* One decode block over a resident pool with misses loaded on demand (the
 * per-layer demand_dual flow of demand.cpp:1081-1171 with the fused kernel):
 * route_first != 0: a VB_DECODE_ROUTE_ONLY launch, read back status and
 * routed ids (one stream synchronisation), vb_res_demand, vb_blob_gather of
 * the placed experts from blob_store (this layer's num_experts blob rows of
 * blob_stride bytes, device or mapped pinned host memory) into the pool,
 * the layer's table copied to args->slot_table, then the whole-block launch.
 * route_first == 0: the whole block first; only when it flagged
 * VB_STATUS_MISS are the experts loaded and the block run again. args:
 * flags 0, out_inds and status required, pool = one blob row per slot of the
 * manager's capacity. The last launch's status is left in *args->status
 * (not read). counts (nullable, int64[4]) accumulates unique routed experts
 * that hit, unique experts loaded, hit positions and kernel launches.
 * VB_ERR_CAPACITY when the routed experts plus the unused pins exceed the
 * slots (out not written). Calls on one manager must use one stream and not
 * overlap (the staging buffers are per layer and reused). */
int vb_moe_decode_resident(const VbMoeDecodeArgs *args, VbResidency *r,
                           int32_t layer, const void *blob_store,
                           int64_t blob_stride, int32_t route_first,
                           int64_t *counts, vb_stream_t stream);

/* Pool fill: copies n expert blobs (host or device memory, the expert_blob_v1
 * layout of prep/blob_layout.py:14-32: gate, up, down x {weight, scales,
 * biases}) into pool slots slots[i] on `stream` (stream-ordered; host blobs
 * should be pinned for asynchronous copies). A pool whose nine tensors are one
 * blob row per slot takes one copy per expert, otherwise nine. Replaces the
 * per-miss loads of ResidentExpertPool (resident_pool.py:414-470) and the
 * blob_loader path feeding them. */
int vb_pool_fill(const VbQuantPool *pool, int32_t hidden, int32_t inter,
                 int32_t group, int32_t bits, const int32_t *slots,
                 const void *const *blobs, int32_t n, vb_stream_t stream);
/* Device gather of whole expert blobs: row out_rows[r] (r when out_rows is
 * NULL) of out = row experts[r] of blob_store, rows of blob_stride bytes (a
 * multiple of 16; 16-byte aligned pointers). experts and out_rows are device
 * arrays; blob_store may be device memory or mapped pinned host memory. With
 * out = a blob pool and out_rows = its slots this fills the misses of one
 * demand in one launch. Ids and rows are not range-checked on the device: the
 * caller passes the placements of vb_res_demand. Replaces the
 * blob_mmap_gather_u4 kernel (native/ext/io/blob_load.cpp:185-196). */
int vb_blob_gather(const void *blob_store, int64_t blob_stride,
                   const int32_t *experts, const int32_t *out_rows, int32_t n,
                   void *out, vb_stream_t stream);

/* Prefill attention over a packed cache: replaces _tiled_asymmetric_attention
 * (mlx_streaming/core/attention/expert_major.py:32-95; the query tiling of
 * 107-182 is not needed) plus the inverse V rotation (kv_quant_patch.py:
 * 67-68) when rv_blocks != NULL. Arguments as vb_kv_decode_attn, any L <=
 * keys; q_heads / kv_heads must divide 128. One tcgen05 kernel (S = QK^T and
 * O += PV in TMEM, online softmax); status (nullable device word) receives
 * VB_STATUS_TIMEOUT if a bounded wait gave up. No workspace. */
int vb_kv_prefill_attn(const uint16_t *q, const uint32_t *k_codes,
                       const uint16_t *k_scales, const uint16_t *k_biases,
                       const uint32_t *v_codes, const uint16_t *v_scales,
                       const uint16_t *v_biases, const float *rv_blocks,
                       int32_t batch, int32_t q_heads, int32_t kv_heads,
                       int32_t L, int32_t dim, int32_t keys, int32_t cap,
                       int32_t group, int32_t k_bits, int32_t v_bits,
                       float scale, int32_t causal, uint16_t *out,
                       int32_t *status, vb_stream_t stream);

/* ---------------------------------------------------------------------------
 * Gated-DeltaNet recurrent steps (the linear-attention state update of the
 * Qwen3-Next GDN layers at decode / MTP verify). Replaces the gated-delta
 * kernel of mlx_streaming/core/linear_attn/gated_delta_multistate.py:28-198
 * (vendored from mlx-lm; y, final state and the state after every step) and
 * the blocked scan of mlx_streaming/core/attention/gdn_fused.py:13-126.
 * Per value head hv (key head hv / (v_heads / k_heads)) and step t, in
 * float32: S *= g; kv = S k; delta = (v - kv) * beta; S += delta k^T;
 * y = bf16(S q). A step with mask[b, t] == 0 leaves S unchanged and gives
 * y = 0. q, k bf16 [B, T, k_heads, 128]; v bf16 [B, T, v_heads, v_dim];
 * g f32 [B, T, v_heads] (g_per_key = 0) or [B, T, v_heads, 128]; beta f32
 * [B, T, v_heads]; state_in/state_out f32 [B, v_heads, v_dim, 128] (may
 * alias); states_out nullable f32 [B, T, v_heads, v_dim, 128]; mask nullable
 * u8 [B, T]; y bf16 [B, T, v_heads, v_dim]. tokens <= 16, v_dim % 16 == 0. */
int vb_gated_delta_step(const uint16_t *q, const uint16_t *k,
                        const uint16_t *v, const float *g, int32_t g_per_key,
                        const float *beta, const float *state_in,
                        float *state_out, float *states_out,
                        const uint8_t *mask, uint16_t *y, int32_t batch,
                        int32_t tokens, int32_t k_heads, int32_t v_heads,
                        int32_t k_dim, int32_t v_dim, vb_stream_t stream);

/* Speculative-verify form (batch 1): states f32 [slots, v_heads, v_dim, 128];
 * the step starts from states[*in_slot] (slot index read on the device: the
 * accepted count - 1 of the previous verify) and writes the state after
 * token t to states[t], t < tokens <= slots (mtp/kv_cache.py:80-100 keeps
 * these per-token checkpoints for the commit). */
int vb_gated_delta_step_at(const uint16_t *q, const uint16_t *k, const uint16_t *v,
                           const float *g, int32_t g_per_key, const float *beta,
                           float *states, int32_t slots, const int32_t *in_slot,
                           const uint8_t *mask, uint16_t *y, int32_t batch,
                           int32_t tokens, int32_t k_heads, int32_t v_heads,
                           int32_t k_dim, int32_t v_dim, vb_stream_t stream);

/* ---------------------------------------------------------------------------
 * Affine dequantization (MLX mx.dequantize; the reference's per-element
 * `qvalue`, native/ext/compute/fused_moe.cpp:131-145, and its inline form in
 * mlx_streaming/core/moe/custom_kernel.py:268-285):
 * out[r, c] = q * scale[r, c/group] + bias[r, c/group], q the c-th
 * `bits`-wide field of row r's LSB-first uint32 bitstream (straddling fields
 * continue in the next word). words [rows, cols*bits/32], scales/biases bf16
 * [rows, cols/group]; out_bf16 != 0: bf16 [rows, cols] (the value rounded
 * once, as fed to the tensor cores; 4-bit rows use the same device routine as
 * the prefill GEMMs), 0: f32 [rows, cols]. bits 2..8. */
int vb_dequantize(const uint32_t *words, const uint16_t *scales,
                  const uint16_t *biases, int64_t rows, int32_t cols,
                  int32_t group, int32_t bits, int32_t out_bf16, void *out,
                  vb_stream_t stream);

/* ---------------------------------------------------------------------------
 * Dense decoder layers of the Qwen3-Next stack around the MoE block (mlx-lm
 * 0.31.3 models/qwen3_next.py as patched by the reference; 4-bit group-64
 * quantized linears as in mtp/qwen3_next_mtp.py:170-181).
 *
 * vb_qlinear: y[T, N] = x' @ dequant(W)^T (+ residual), MLX quantized_matmul
 * (per group s * sum(x q) + b * sum(x), float32, one bf16 rounding; the
 * residual add is a second bf16 rounding, h = x + r of the decoder layer).
 * x' = x, or rms_norm(x) * norm_w (bf16 at each op) when norm_w != NULL.
 * T <= 8, in_features a multiple of 256 (of 512 above 2048, at most 4096),
 * bits 4, group 64; x, scales, biases and norm_w 16-byte aligned, codes 8. No
 * workspace is needed (vb_qlinear_workspace_size returns 0; the K reduction
 * stays inside a CTA). */
size_t vb_qlinear_workspace_size(int32_t tokens, int32_t in_features, int32_t out_features);
int vb_qlinear(const uint16_t *x, int32_t tokens, int32_t in_features,
               const uint32_t *codes, const uint16_t *scales, const uint16_t *biases,
               int32_t out_features, int32_t group, int32_t bits, const uint16_t *norm_w,
               float norm_eps, const uint16_t *residual, uint16_t *y, void *workspace,
               size_t workspace_bytes, vb_stream_t stream);

/* mx.fast.rms_norm with an optional residual add before it: h = bf16(x + r)
 * (written to h_out when given), y = bf16(bf16(h * rsqrt(mean(h^2) + eps)) * w)
 * (w NULL: unit weight). x, residual, h_out [rows, dim]; y rows y_stride
 * elements apart (0: dim), so two norms can fill the halves of one
 * concatenated row (the MTP head's fc input). */
int vb_rms_norm(const uint16_t *x, const uint16_t *residual, const uint16_t *weight,
                int32_t rows, int32_t dim, float eps, uint16_t *h_out, uint16_t *y,
                int32_t y_stride, vb_stream_t stream);

/* mx.argmax over each row of bf16 values (ties to the smallest index). The
 * workspace (vb_argmax_workspace_size, zero-filled once) holds tickets. */
size_t vb_argmax_workspace_size(int32_t rows);
int vb_argmax(const uint16_t *values, int32_t rows, int32_t n, int32_t *out, void *workspace,
              size_t workspace_bytes, vb_stream_t stream);

/* The MTP head's fc input (qwen3_next_mtp.py:40-46) in one launch: row t of
 * out bf16 [T, 2 * hidden] = [rms_norm(embed(ids[t])) * emb_norm_w |
 * rms_norm(prev_hidden[t]) * hid_norm_w], bit for bit vb_embed_rows followed
 * by two vb_rms_norm into the halves (weights NULL: unit). hidden <= 8192.
 * Ids out of range give a zero embedding half and VB_STATUS_BOUNDS. */
int vb_mtp_fc_input(const int32_t *ids, int32_t tokens, const uint32_t *codes,
                    const uint16_t *scales, const uint16_t *biases, int32_t vocab,
                    int32_t hidden, const uint16_t *emb_norm_w, const uint16_t *prev_hidden,
                    const uint16_t *hid_norm_w, float eps, uint16_t *out, int32_t *status,
                    vb_stream_t stream);

/* nn.QuantizedEmbedding: out[t] = dequant(table row ids[t]) (bf16, 4-bit
 * group 64). Ids out of range give zero rows and VB_STATUS_BOUNDS. */
int vb_embed_rows(const int32_t *ids, int32_t tokens, const uint32_t *codes,
                  const uint16_t *scales, const uint16_t *biases, int32_t vocab,
                  int32_t hidden, int32_t group, int32_t bits, uint16_t *out, int32_t *status,
                  vb_stream_t stream);

/* Gated-DeltaNet input side (mtp/kv_cache.py:34-91; gated_delta_multistate.py:
 * 201-226): proj bf16 [T, proj_stride] = in_proj_qkvz | in_proj_ba outputs
 * (per key head [q Dk, k Dk, v r*Dv, z r*Dv], then per key head [b r, a r]).
 * conv_buf bf16 [3 + max_tokens, C], C = 2 Hk Dk + Hv Dv: rows [*conv_off,
 * *conv_off + 3) hold the conv state (conv_off NULL: 0); the call leaves the
 * state in rows 0..2 and the T new rows in 3..3+T-1, so the state after
 * accepting a rows is rows [a, a+3). conv_w bf16 [C, 4]. Outputs q, k bf16
 * [T, Hk, Dk] (rms-normalised and scaled by Dk^-1 / Dk^-0.5), v bf16
 * [T, Hv, Dv], g and beta f32 [T, Hv]. T <= max_tokens <= 8. */
int vb_gdn_prepare(const uint16_t *proj, int32_t proj_stride, int32_t tokens, int32_t k_heads,
                   int32_t v_heads, int32_t head_k, int32_t head_v, uint16_t *conv_buf,
                   int32_t max_tokens, const int32_t *conv_off, const uint16_t *conv_w,
                   const float *a_log, const uint16_t *dt_bias, uint16_t *q, uint16_t *k,
                   uint16_t *v, float *g, float *beta, int32_t *status, vb_stream_t stream);

/* Gated RMSNorm of the recurrence output (kv_cache.py:102, mlx-lm
 * Qwen3NextRMSNormGated): out = silu(z) * (w * rms_norm(y)), z read from the
 * projection rows. y, out bf16 [T, Hv, Dv]; weight bf16 [Dv]. */
int vb_gdn_gated_norm(const uint16_t *y, const uint16_t *proj, int32_t proj_stride,
                      int32_t tokens, int32_t k_heads, int32_t v_heads, int32_t head_k,
                      int32_t head_v, const uint16_t *weight, float eps, uint16_t *out,
                      vb_stream_t stream);

/* The three calls above (vb_gdn_prepare -> vb_gated_delta_step_at ->
 * vb_gdn_gated_norm, batch 1) in one launch, bit-identical to them: one
 * thread-block cluster of (v_heads / k_heads) x (head_v / 32) <= 8 CTAs per
 * key head; the conv window is moved after a cluster barrier and the gated
 * norm's row sums cross the cluster through distributed shared memory.
 * states f32 [slots, v_heads, head_v, 128] as vb_gated_delta_step_at (start
 * state in slot *in_slot, the state after row t in slot t); out bf16
 * [T, v_heads * head_v]. head_k = 128, T <= max_tokens <= 8. */
int vb_gdn_fused(const uint16_t *proj, int32_t proj_stride, int32_t tokens, int32_t k_heads,
                 int32_t v_heads, int32_t head_k, int32_t head_v, uint16_t *conv_buf,
                 int32_t max_tokens, const int32_t *conv_off, const uint16_t *conv_w,
                 const float *a_log, const uint16_t *dt_bias, float *states, int32_t slots,
                 const int32_t *in_slot, const uint16_t *norm_w, float eps, uint16_t *out,
                 int32_t *status, vb_stream_t stream);

/* Attention input side (kv_quant_patch.py:29-56): proj bf16 [T, proj_stride]
 * = q_proj (per head [query 256, gate 256]) | k_proj | v_proj. Queries and
 * keys get their RMSNorm (weights [256]) and RoPE over the first rope_dims
 * dims at position *pos + pos_add + t (non-traditional pairs (i, i + dims/2),
 * theta = pos * base^(-2i/dims)); queries are then rotated by the SO(4)
 * blocks rk_blocks (NULL: none). q_out bf16 [Hq, T, 256]; keys and values go
 * to k_out/v_out [Hkv, T, 256] (kv_cap 0) or into bf16 caches
 * [Hkv, kv_cap, 256] at their positions. */
int vb_attn_prepare(const uint16_t *proj, int32_t proj_stride, int32_t tokens, int32_t q_heads,
                    int32_t kv_heads, int32_t head_dim, const uint16_t *q_norm_w,
                    const uint16_t *k_norm_w, float eps, int32_t rope_dims, float rope_base,
                    const int32_t *pos, int32_t pos_add, const float *rk_blocks,
                    uint16_t *q_out, uint16_t *k_out, uint16_t *v_out, int32_t kv_cap,
                    int32_t *status, vb_stream_t stream);

/* vb_attn_prepare with the IsoQuant cache append fused in (kv_quant_patch.py
 * :29-56 and AsymmetricQuantizedKVCache.update_and_fetch, quant_kv.py:
 * 105-137): queries as in vb_attn_prepare (RoPE at *pos + t, rotated by
 * rk_blocks) into q_out [Hq, T, 256]; keys (after their norm and RoPE) rotated
 * by rk_blocks and values by rv_blocks, quantized (group 64, k_bits / v_bits)
 * and packed into the caches [Hkv, cap, ...] at position *pos + t: the same
 * bits as vb_attn_prepare to bf16 rows followed by vb_kv_quant_append_at of
 * each, in one launch. A position outside [0, cap) sets VB_STATUS_BOUNDS and
 * stores nothing for that row. */
int vb_attn_prepare_quant(const uint16_t *proj, int32_t proj_stride, int32_t tokens,
                          int32_t q_heads, int32_t kv_heads, int32_t head_dim,
                          const uint16_t *q_norm_w, const uint16_t *k_norm_w, float eps,
                          int32_t rope_dims, float rope_base, const int32_t *pos,
                          const float *rk_blocks, const float *rv_blocks, uint16_t *q_out,
                          int32_t cap, int32_t k_bits, uint32_t *k_codes, uint16_t *k_scales,
                          uint16_t *k_biases, int32_t v_bits, uint32_t *v_codes,
                          uint16_t *v_scales, uint16_t *v_biases, int32_t *status,
                          vb_stream_t stream);

/* output * sigmoid(gate) (kv_quant_patch.py:70-71): attn_out bf16 [Hq, T, 256]
 * -> out bf16 [T, Hq * 256], gate read from the projection rows. */
int vb_attn_gate(const uint16_t *attn_out, const uint16_t *proj, int32_t proj_stride,
                 int32_t tokens, int32_t q_heads, uint16_t *out, vb_stream_t stream);

/* Speculative (MTP) loop, device side. state int32 [16]: [0] main cache
 * length, [1] MTP cache length, [2] accepted rows of the last verify or
 * prefill chunk, [3] that minus one (recurrent state slot), [4] pending
 * token, [5] emitted tokens, [6] verify steps, [7..14] histogram of matched
 * drafts. ids int32 [1 + drafts]: ids[0] pending token, ids[1..] drafts; the
 * verify step feeds ids[0..verify_len).
 * vb_spec_accept (generate.py:338-352, 818-853): mode 0 compares the verify
 * argmaxes preds[verify_len] with the drafts, commits a = min(matched + 1,
 * verify_len) rows, appends the emitted tokens (drafts[:matched] and the
 * model's token at the first mismatch) to out_tokens, sets the pending token;
 * mode 1 (prefill chunk) commits all rows and also writes the pending token
 * to ids[0]. Both copy h_last to prev_h and the last committed row of
 * verify_hidden [verify_len, hidden] to h_last. */
int vb_spec_accept(int32_t *state, int32_t *ids, const int32_t *preds, int32_t verify_len,
                   int32_t drafts, int32_t mode, const uint16_t *verify_hidden,
                   uint16_t *h_last, uint16_t *prev_h, int32_t hidden, int32_t *out_tokens,
                   int32_t out_cap, vb_stream_t stream);
/* MTP cache sync inputs (drafter.py:178-186): slot i < a gets ids[i] and
 * hidden (i == 0 ? prev_h : verify_hidden[i - 1]); later slots repeat slot
 * a - 1. sync_ids [verify_len], sync_hidden [verify_len, hidden]. Then
 * ids[0] = the pending token, for the next drafts. */
int vb_spec_sync_inputs(const int32_t *state, int32_t *ids, const uint16_t *verify_hidden,
                        const uint16_t *prev_h, int32_t verify_len, int32_t hidden,
                        int32_t *sync_ids, uint16_t *sync_hidden, vb_stream_t stream);
/* MTP cache length += accepted rows. */
int vb_spec_advance_mtp(int32_t *state, vb_stream_t stream);
/* Prompt chunk: ids[i] = prompt[state[0] + i], i < tokens. */
int vb_spec_prompt_ids(const int32_t *state, const int32_t *prompt, int32_t prompt_len,
                       int32_t tokens, int32_t *ids, vb_stream_t stream);

/* ---------------------------------------------------------------------------
 * Seeded synthetic data (bench and tests): fills `words` uint32 with a
 * counter hash of (seed, index) and bf16 scales uniform in [lo, hi) with
 * biases = -8*scale (MLX 4-bit affine weights as in the benchmark configs).
 * Not part of the reference interface. */
int vb_synth_fill_u32(uint32_t *words, int64_t n, uint64_t seed,
                      vb_stream_t stream);
int vb_synth_fill_scales(uint16_t *scales, uint16_t *biases, int64_t n,
                         uint64_t seed, float lo, float hi, float bias_mul,
                         vb_stream_t stream);
/* The nine tensors of n experts in one launch: slot slots[i] (host array)
 * gets expert seed seeds[i] (host array); every tensor holds the values that
 * vb_synth_fill_u32 / vb_synth_fill_scales give it with the per-tensor seed
 * mix(seed, 3*proj) for codes and mix(seed, 3*proj + 1) for scales, where
 * mix(s, t) = z ^ (z >> 31), z = s*0x9E3779B97F4A7C15 + t*0xBF58476D1CE4E5B9
 * + 0x94D049BB133111EB (mod 2^64). */
int vb_synth_fill_pool(const VbQuantPool *pool, const int32_t *slots,
                       const uint64_t *seeds, int32_t n, int32_t hidden,
                       int32_t inter, int32_t bits, int32_t group, float lo,
                       float hi, float bias_mul, vb_stream_t stream);

#ifdef __cplusplus
}
#endif
#endif /* VATES_B200_H */
