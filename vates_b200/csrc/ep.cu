// Expert-parallel expert-major prefill: one rank per GPU, NCCL between them.
//
// The reference runs the expert-major prefill on one device
// (FileStreamingMoeBlock._expert_major_forward, mlx_streaming/core/moe/
// block.py:111-243, entered from block.py:330-347). Here every rank holds a
// subset of the experts (owner[e] == rank; experts replicated on every rank
// map to the rank itself) and starts with its own slice of the tokens. One
// call runs, on the caller's stream:
//   1. route the local tokens (router GEMM, softmax, top-k)      vb_moe_route
//   2. all-reduce of the route histogram: the reference's reduce groups are
//      a property of the whole batch, so every rank adds its routes in the
//      same order and the result does not depend on the number of ranks
//   3. pack each token row once per destination rank, plus the route
//      metadata (row, expert, score)                             vb_ep_pack
//   4. exchange the per-destination counts; the host reads them (NCCL's
//      point-to-point sizes live on the host)
//   5. grouped ncclSend/ncclRecv of the rows and metadata; the chunk a rank
//      keeps for itself is a device copy, not a collective
//   6. the rank's experts on the received routes, the shared expert on the
//      local tokens                                              vb_moe_experts
//   7. grouped ncclSend/ncclRecv of the weighted route rows back to their
//      token's rank (own rows again by device copy)
//   8. reduce every token's k route rows in the reference's order, then the
//      gated shared expert                                       vb_moe_combine
// Every route row is computed exactly as on one device and the reduce order
// is the reference's, so the output is bit-identical for any number of
// ranks and any placement.
//
// NCCL is not linked: its entry points are looked up at the first call in
// the libnccl.so.2 the process already loaded (the one that created the
// communicator), else loaded by name.
#include <dlfcn.h>
#include <nccl.h>

#include <algorithm>
#include <mutex>

#include "common.cuh"

namespace vb {

constexpr int EPX_MAX_WORLD = 8;

struct NcclApi {
  ncclResult_t (*group_start)();
  ncclResult_t (*group_end)();
  ncclResult_t (*send)(const void *, size_t, ncclDataType_t, int, ncclComm_t, cudaStream_t);
  ncclResult_t (*recv)(void *, size_t, ncclDataType_t, int, ncclComm_t, cudaStream_t);
  ncclResult_t (*all_reduce)(const void *, void *, size_t, ncclDataType_t, ncclRedOp_t,
                             ncclComm_t, cudaStream_t);
  const char *(*error_string)(ncclResult_t);
  bool ok;
};

static const NcclApi &nccl_api() {
  static NcclApi api{};
  static std::once_flag once;
  std::call_once(once, [] {
    void *h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_NOLOAD);
    if (!h) h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_GLOBAL);
    if (!h) return;
    api.group_start = (decltype(api.group_start))dlsym(h, "ncclGroupStart");
    api.group_end = (decltype(api.group_end))dlsym(h, "ncclGroupEnd");
    api.send = (decltype(api.send))dlsym(h, "ncclSend");
    api.recv = (decltype(api.recv))dlsym(h, "ncclRecv");
    api.all_reduce = (decltype(api.all_reduce))dlsym(h, "ncclAllReduce");
    api.error_string = (decltype(api.error_string))dlsym(h, "ncclGetErrorString");
    api.ok = api.group_start && api.group_end && api.send && api.recv && api.all_reduce &&
             api.error_string;
  });
  return api;
}

// Workspace carve-up (every piece 1024-byte aligned). Receive buffers hold
// the worst case: every route of every rank sent to this rank.
struct EpLayout {
  size_t route_ws, inds, scores, sgate, counts, gcounts, send_x, send_meta, rsi, cnt, pack_ws,
      recv_x, recv_meta, offs, r_row, r_exp, r_score, y_recv, experts_ws, s_row, s_exp,
      s_score, y_shared, shared_ws, y_back, combine_ws, total;
};

static EpLayout ep_layout(int T, int H, int I, int E, int k, int world, int max_t) {
  EpLayout L;
  size_t off = 0;
  auto take = [&](size_t bytes) {
    const size_t at = off;
    off = align_up(off + std::max<size_t>(bytes, 1), 1024);
    return at;
  };
  const size_t rows_in = (size_t)world * max_t;      // token rows received, worst case
  const size_t routes_in = (size_t)world * max_t * k;  // routes received, worst case
  L.route_ws = take(vb_moe_route_workspace_size(T, H, E));
  L.inds = take((size_t)T * k * 4);
  L.scores = take((size_t)T * k * 4);
  L.sgate = take((size_t)T * 4);
  L.counts = take((size_t)(E + 1) * 4);
  L.gcounts = take((size_t)(E + 1) * 4);
  L.send_x = take((size_t)T * std::min(k, world) * H * 2);
  L.send_meta = take((size_t)T * k * 12);
  L.rsi = take((size_t)T * k * 4);
  L.cnt = take((size_t)4 * world * 4);  // [2][world] sent counts, [world][2] received
  L.pack_ws = take(vb_ep_pack_workspace_size(T, world));
  L.recv_x = take(rows_in * H * 2);
  L.recv_meta = take(routes_in * 12);
  L.offs = take((size_t)(4 * world + 2) * 4);  // received pairs [W][2], offsets [2W + 2]
  L.r_row = take(routes_in * 4);
  L.r_exp = take(routes_in * 4);
  L.r_score = take(routes_in * 4);
  L.y_recv = take(routes_in * H * 2);
  L.experts_ws = take(vb_moe_experts_workspace_size((int32_t)routes_in, H, I, E));
  L.s_row = take((size_t)T * 4);
  L.s_exp = take((size_t)T * 4);
  L.s_score = take((size_t)T * 4);
  L.y_shared = take((size_t)T * H * 2);
  L.shared_ws = take(vb_moe_experts_workspace_size(T, H, I, E));
  L.y_back = take((size_t)T * k * H * 2);
  L.combine_ws = take((size_t)E * 4);
  L.total = off;
  return L;
}

__global__ void ep_shared_routes_kernel(int T, int E, int32_t *row, int32_t *ex, float *score) {
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i < T) {
    row[i] = i;
    ex[i] = E;
    score[i] = 1.f;
  }
}

// [2][world] sent counts (rows, routes per destination) -> [world][2] pairs.
__global__ void ep_pair_counts_kernel(const int32_t *cnt, int world, int32_t *pairs) {
  const int d = threadIdx.x;
  if (d < world) {
    pairs[2 * d] = cnt[d];
    pairs[2 * d + 1] = cnt[world + d];
  }
}

#define VB_NCCL(call)                                                                    \
  do {                                                                                   \
    const ncclResult_t r_ = (call);                                                      \
    if (r_ != ncclSuccess)                                                               \
      return set_error(VB_ERR_CUDA, "vb_moe_prefill_ep: %s: %s", #call, api.error_string(r_)); \
  } while (0)

#define VB_CALL(call)                 \
  do {                                \
    const int rc_ = (call);           \
    if (rc_ != VB_OK) return rc_;     \
  } while (0)

#define VB_CUDA(call)                                                                     \
  do {                                                                                    \
    const cudaError_t e_ = (call);                                                        \
    if (e_ != cudaSuccess)                                                                \
      return set_error(VB_ERR_CUDA, "vb_moe_prefill_ep: %s: %s", #call, cudaGetErrorString(e_)); \
  } while (0)

}  // namespace vb

using namespace vb;

extern "C" {

size_t vb_moe_prefill_ep_workspace_size(int32_t tokens, int32_t hidden, int32_t inter,
                                        int32_t num_experts, int32_t top_k, int32_t world,
                                        int32_t max_tokens_per_rank) {
  if (tokens <= 0 || hidden <= 0 || inter <= 0 || num_experts <= 0 || top_k <= 0 ||
      world <= 0 || max_tokens_per_rank < tokens)
    return 0;
  return ep_layout(tokens, hidden, inter, num_experts, top_k, world, max_tokens_per_rank).total;
}

int vb_moe_prefill_ep(const VbMoePrefillEpArgs *a, void *nccl_comm, vb_stream_t stream) {
  VB_REQUIRE(a && nccl_comm, "vb_moe_prefill_ep: null args or communicator");
  const VbMoePrefillArgs &b = a->base;
  const int T = b.tokens, H = b.hidden, I = b.inter, E = b.num_experts, k = b.top_k;
  const int W = a->world, R = a->rank;
  VB_REQUIRE(W >= 1 && W <= EPX_MAX_WORLD && R >= 0 && R < W,
             "vb_moe_prefill_ep: world=%d rank=%d", W, R);
  VB_REQUIRE(T >= 1 && a->max_tokens_per_rank >= T, "vb_moe_prefill_ep: tokens=%d max=%d", T,
             a->max_tokens_per_rank);
  VB_REQUIRE(b.bits == 4 && (b.group == 64 || b.group == 128),
             "vb_moe_prefill_ep: bits=%d group=%d", b.bits, b.group);
  VB_REQUIRE(b.x && b.router_w && b.slot_table && b.out && a->owner,
             "vb_moe_prefill_ep: null tensor");
  const EpLayout L = ep_layout(T, H, I, E, k, W, a->max_tokens_per_rank);
  VB_REQUIRE(b.workspace && b.workspace_bytes >= L.total && ((uintptr_t)b.workspace % 1024) == 0,
             "vb_moe_prefill_ep: workspace %zu < %zu or not 1024-byte aligned",
             b.workspace_bytes, L.total);
  const NcclApi &api = nccl_api();
  VB_REQUIRE(api.ok, "vb_moe_prefill_ep: libnccl.so.2 not found");
  ncclComm_t comm = reinterpret_cast<ncclComm_t>(nccl_comm);
  cudaStream_t s = as_stream(stream);
  uint8_t *ws = static_cast<uint8_t *>(b.workspace);
  auto at = [&](size_t off) { return (void *)(ws + off); };
  const bool has_shared = b.shared.ptr[0] != nullptr;

  // 1. route
  VbMoeRouteArgs ra = {};
  ra.tokens = T; ra.hidden = H; ra.num_experts = E; ra.top_k = k; ra.norm_topk = b.norm_topk;
  ra.x = b.x; ra.router_w = b.router_w; ra.router_bias = b.router_bias;
  ra.shared_gate_w = has_shared ? b.shared_gate_w : nullptr;
  ra.out_inds = (int32_t *)at(L.inds); ra.out_scores = (float *)at(L.scores);
  ra.out_sgate = (float *)at(L.sgate); ra.out_counts = (int32_t *)at(L.counts);
  ra.out_logits = b.out_logits; ra.status = b.status;
  ra.workspace = at(L.route_ws); ra.workspace_bytes = vb_moe_route_workspace_size(T, H, E);
  VB_CALL(vb_moe_route(&ra, stream));
  if (b.out_inds)
    VB_CUDA(cudaMemcpyAsync(b.out_inds, at(L.inds), (size_t)T * k * 4, cudaMemcpyDeviceToDevice, s));

  // 2. route histogram of the whole batch
  VB_NCCL(api.all_reduce(at(L.counts), at(L.gcounts), (size_t)E, ncclInt32, ncclSum, comm, s));

  // 3. pack
  int32_t *cnt = (int32_t *)at(L.cnt);  // [2][W] sent, then [W][2] pairs, then [W][2] received
  VbEpPackArgs pa = {};
  pa.tokens = T; pa.top_k = k; pa.hidden = H; pa.world = W;
  pa.x = b.x; pa.inds = (const int32_t *)at(L.inds); pa.scores = (const float *)at(L.scores);
  pa.owner = a->owner;
  pa.send_x = (uint16_t *)at(L.send_x); pa.send_meta = (int32_t *)at(L.send_meta);
  pa.route_send_idx = (int32_t *)at(L.rsi);
  pa.dest_rows = cnt; pa.dest_routes = cnt + W;
  pa.workspace = at(L.pack_ws); pa.workspace_bytes = vb_ep_pack_workspace_size(T, W);
  VB_CALL(vb_ep_pack(&pa, stream));

  // 4. counts: (rows, routes) per destination -> per source; host read
  int32_t *pairs = cnt + 2 * W;  // [W][2]
  ep_pair_counts_kernel<<<1, 32, 0, s>>>(cnt, W, pairs);
  VB_CALL(check_launch("ep_pair_counts_kernel"));
  int32_t *recv_pairs = (int32_t *)at(L.offs);  // [W][2]; offsets follow after the read
  VB_NCCL(api.group_start());
  for (int d = 0; d < W; ++d) {
    if (d == R) continue;
    VB_NCCL(api.send(pairs + 2 * d, 2, ncclInt32, d, comm, s));
    VB_NCCL(api.recv(recv_pairs + 2 * d, 2, ncclInt32, d, comm, s));
  }
  VB_NCCL(api.group_end());
  VB_CUDA(cudaMemcpyAsync(recv_pairs + 2 * R, pairs + 2 * R, 8, cudaMemcpyDeviceToDevice, s));
  int32_t h_send[2 * EPX_MAX_WORLD], h_recv[2 * EPX_MAX_WORLD];
  VB_CUDA(cudaMemcpyAsync(h_send, pairs, 8 * W, cudaMemcpyDeviceToHost, s));
  VB_CUDA(cudaMemcpyAsync(h_recv, recv_pairs, 8 * W, cudaMemcpyDeviceToHost, s));
  VB_CUDA(cudaStreamSynchronize(s));
  // per-source offsets of the received routes and rows (host) -> device
  int32_t h_offs[2 * (EPX_MAX_WORLD + 1)];
  int64_t n_routes = 0, n_rows = 0;
  size_t row_at[EPX_MAX_WORLD], route_at[EPX_MAX_WORLD], back_at[EPX_MAX_WORLD],
      send_row_at[EPX_MAX_WORLD], send_route_at[EPX_MAX_WORLD];
  for (int q = 0; q < W; ++q) {
    h_offs[q] = (int32_t)n_routes;                  // src_route_off[q]
    h_offs[W + 1 + q] = (int32_t)n_rows;            // src_row_off[q]
    route_at[q] = (size_t)n_routes;
    row_at[q] = (size_t)n_rows;
    n_routes += h_recv[2 * q + 1];
    n_rows += h_recv[2 * q];
  }
  h_offs[W] = (int32_t)n_routes;
  h_offs[2 * W + 1] = (int32_t)n_rows;
  {
    size_t rr = 0, rt = 0;
    for (int d = 0; d < W; ++d) {
      send_row_at[d] = rr;
      send_route_at[d] = rt;
      back_at[d] = rt;  // route rows come back in the order they were sent
      rr += h_send[2 * d];
      rt += h_send[2 * d + 1];
    }
  }
  int32_t *d_offs = recv_pairs + 2 * W;
  VB_CUDA(cudaMemcpyAsync(d_offs, h_offs, 4 * (2 * W + 2), cudaMemcpyHostToDevice, s));

  // 5. rows and metadata to their expert's rank
  uint16_t *send_x = (uint16_t *)at(L.send_x), *recv_x = (uint16_t *)at(L.recv_x);
  int32_t *send_meta = (int32_t *)at(L.send_meta), *recv_meta = (int32_t *)at(L.recv_meta);
  VB_NCCL(api.group_start());
  for (int q = 0; q < W; ++q) {
    if (q == R) continue;
    if (h_send[2 * q])
      VB_NCCL(api.send(send_x + send_row_at[q] * H, (size_t)h_send[2 * q] * H, ncclBfloat16, q,
                       comm, s));
    if (h_send[2 * q + 1])
      VB_NCCL(api.send(send_meta + send_route_at[q] * 3, (size_t)h_send[2 * q + 1] * 3, ncclInt32,
                       q, comm, s));
    if (h_recv[2 * q])
      VB_NCCL(api.recv(recv_x + row_at[q] * H, (size_t)h_recv[2 * q] * H, ncclBfloat16, q, comm,
                       s));
    if (h_recv[2 * q + 1])
      VB_NCCL(api.recv(recv_meta + route_at[q] * 3, (size_t)h_recv[2 * q + 1] * 3, ncclInt32, q,
                       comm, s));
  }
  VB_NCCL(api.group_end());
  if (h_send[2 * R])
    VB_CUDA(cudaMemcpyAsync(recv_x + row_at[R] * H, send_x + send_row_at[R] * H,
                            (size_t)h_send[2 * R] * H * 2, cudaMemcpyDeviceToDevice, s));
  if (h_send[2 * R + 1])
    VB_CUDA(cudaMemcpyAsync(recv_meta + route_at[R] * 3, send_meta + send_route_at[R] * 3,
                            (size_t)h_send[2 * R + 1] * 12, cudaMemcpyDeviceToDevice, s));

  // 6. experts on the received routes; the shared expert on the local tokens
  int32_t *r_row = (int32_t *)at(L.r_row), *r_exp = (int32_t *)at(L.r_exp);
  float *r_score = (float *)at(L.r_score);
  uint16_t *y_recv = (uint16_t *)at(L.y_recv);
  if (n_routes > 0) {
    VB_CALL(vb_ep_unpack(recv_meta, (int32_t)n_routes, d_offs, d_offs + W + 1, W, r_row, r_exp,
                         r_score, stream));
    VbMoeExpertsArgs xa = {};
    xa.rows = (int32_t)std::max<int64_t>(n_rows, 1); xa.routes = (int32_t)n_routes;
    xa.hidden = H; xa.inter = I; xa.group = b.group; xa.bits = b.bits; xa.num_experts = E;
    xa.x = recv_x; xa.route_row = r_row; xa.route_expert = r_exp; xa.route_score = r_score;
    xa.slot_table = b.slot_table; xa.pool = b.pool; xa.out = y_recv; xa.status = b.status;
    xa.workspace = at(L.experts_ws);
    xa.workspace_bytes = vb_moe_experts_workspace_size((int32_t)n_routes, H, I, E);
    VB_CALL(vb_moe_experts(&xa, stream));
  }
  uint16_t *y_shared = nullptr;
  if (has_shared) {
    int32_t *s_row = (int32_t *)at(L.s_row), *s_exp = (int32_t *)at(L.s_exp);
    float *s_score = (float *)at(L.s_score);
    ep_shared_routes_kernel<<<(T + 255) / 256, 256, 0, s>>>(T, E, s_row, s_exp, s_score);
    VB_CALL(check_launch("ep_shared_routes_kernel"));
    y_shared = (uint16_t *)at(L.y_shared);
    VbMoeExpertsArgs sa = {};
    sa.rows = T; sa.routes = T; sa.hidden = H; sa.inter = I; sa.group = b.group;
    sa.bits = b.bits; sa.num_experts = E;
    sa.x = b.x; sa.route_row = s_row; sa.route_expert = s_exp; sa.route_score = s_score;
    sa.slot_table = b.slot_table; sa.pool = b.pool; sa.shared = b.shared; sa.out = y_shared;
    sa.status = b.status;
    sa.workspace = at(L.shared_ws); sa.workspace_bytes = vb_moe_experts_workspace_size(T, H, I, E);
    VB_CALL(vb_moe_experts(&sa, stream));
  }

  // 7. weighted route rows back to their token's rank
  uint16_t *y_back = (uint16_t *)at(L.y_back);
  VB_NCCL(api.group_start());
  for (int q = 0; q < W; ++q) {
    if (q == R) continue;
    if (h_recv[2 * q + 1])
      VB_NCCL(api.send(y_recv + route_at[q] * H, (size_t)h_recv[2 * q + 1] * H, ncclBfloat16, q,
                       comm, s));
    if (h_send[2 * q + 1])
      VB_NCCL(api.recv(y_back + back_at[q] * H, (size_t)h_send[2 * q + 1] * H, ncclBfloat16, q,
                       comm, s));
  }
  VB_NCCL(api.group_end());
  if (h_send[2 * R + 1])
    VB_CUDA(cudaMemcpyAsync(y_back + back_at[R] * H, y_recv + route_at[R] * H,
                            (size_t)h_send[2 * R + 1] * H * 2, cudaMemcpyDeviceToDevice, s));

  // 8. reduce in the reference's order, then the gated shared expert
  VbMoeCombineArgs ca = {};
  ca.tokens = T; ca.hidden = H; ca.num_experts = E; ca.top_k = k;
  ca.layer_cap = b.layer_cap; ca.max_assignments = b.max_assignments;
  ca.inds = (const int32_t *)at(L.inds); ca.counts = (const int32_t *)at(L.gcounts);
  ca.y_routes = y_back; ca.route_row = (const int32_t *)at(L.rsi);
  ca.y_shared = y_shared; ca.shared_row = nullptr; ca.sgate = (const float *)at(L.sgate);
  ca.out = b.out; ca.group_of_ws = (int32_t *)at(L.combine_ws);
  VB_CALL(vb_moe_combine(&ca, stream));
  return VB_OK;
}

}  // extern "C"
