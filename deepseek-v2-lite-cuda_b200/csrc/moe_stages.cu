// Composable stages of the MoE layer, exported so that a caller can put a collective between
// them (expert parallelism: dispatch -> all-to-all -> expert MLP -> all-to-all -> combine).
// Each stage is one or more launches on the caller's stream, with no host synchronisation.
#include "kernels.cuh"

namespace ds {
namespace {

// Receive-side plan for expert parallelism.  counts[s * El + e] = rows that source rank s
// sends for local expert e; received rows arrive source-major (all of source 0's rows,
// expert-major inside, then source 1's, ...).  Produces expert-major offsets [El+1] and, for
// every expert-major row i, the source-major row it comes from (row_map[i]).
__global__ void __launch_bounds__(1024)
    ep_offsets_kernel(const int32_t* __restrict__ counts, int N, int El,
                      int32_t* __restrict__ exp_offsets, int32_t* __restrict__ seg_src,
                      int32_t* __restrict__ seg_exp) {
  // seg_src[s*El+e]: source-major start of segment (s, e); seg_exp[s*El+e]: expert-major start
  if (threadIdx.x == 0) {
    int run = 0;
    for (int s = 0; s < N; ++s)
      for (int e = 0; e < El; ++e) {
        seg_src[s * El + e] = run;
        run += counts[s * El + e];
      }
    run = 0;
    for (int e = 0; e < El; ++e) {
      exp_offsets[e] = run;
      for (int s = 0; s < N; ++s) {
        seg_exp[s * El + e] = run;
        run += counts[s * El + e];
      }
    }
    exp_offsets[El] = run;
  }
}

__global__ void __launch_bounds__(256)
    ep_rowmap_kernel(const int32_t* __restrict__ counts, const int32_t* __restrict__ seg_src,
                     const int32_t* __restrict__ seg_exp, int segs, int R,
                     int32_t* __restrict__ row_map) {
  extern __shared__ int32_t sm[];
  int32_t* ssrc = sm;
  int32_t* sexp = sm + segs + 1;
  for (int i = threadIdx.x; i < segs; i += blockDim.x) {
    ssrc[i] = seg_src[i];
    sexp[i] = seg_exp[i];
  }
  if (threadIdx.x == 0) ssrc[segs] = R;
  __syncthreads();
  for (int r = blockIdx.x * blockDim.x + threadIdx.x; r < R; r += gridDim.x * blockDim.x) {
    // segment containing source-major row r: last seg with ssrc[seg] <= r and nonempty
    int lo = 0, hi = segs;
    while (hi - lo > 1) {
      const int mid = (lo + hi) >> 1;
      if (ssrc[mid] <= r) lo = mid;
      else hi = mid;
    }
    row_map[sexp[lo] + (r - ssrc[lo])] = r;
  }
}

__global__ void __launch_bounds__(256)
    gather_rows_kernel(const uint4* __restrict__ src, const int32_t* __restrict__ map, int R,
                       int H8, uint4* __restrict__ dst) {
  const int lane = threadIdx.x & 31;
  const int warps = gridDim.x * (blockDim.x >> 5);
  for (int r = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5); r < R; r += warps) {
    const uint4* s = src + static_cast<int64_t>(__ldg(map + r)) * H8;
    uint4* d = dst + static_cast<int64_t>(r) * H8;
    for (int c = lane; c < H8; c += 32) d[c] = __ldg(s + c);
  }
}

// gate f32 [E, H] -> split [256, H] bf16: rows e, 64+e, 128+e = hi, mid, lo with
// gate = hi + mid + lo (each residual is exact in f32); all other rows zero.
__global__ void router_split_kernel(const float* __restrict__ gate, int E, int H,
                                    __nv_bfloat16* __restrict__ out) {
  const int64_t total = 256LL * H;
  for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < total;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int r = static_cast<int>(i / H);
    const int c = static_cast<int>(i - static_cast<int64_t>(r) * H);
    const int part = r >> 6, e = r & 63;
    float v = 0.f;
    if (part < 3 && e < E) {
      const float g = gate[static_cast<int64_t>(e) * H + c];
      const float hi = __bfloat162float(__float2bfloat16_rn(g));
      const float r1 = g - hi;
      const float mid = __bfloat162float(__float2bfloat16_rn(r1));
      const float r2 = r1 - mid;
      v = part == 0 ? hi : (part == 1 ? mid : r2);
    }
    out[i] = __float2bfloat16_rn(v);
  }
}

int grid_cap(int64_t items, int per_block, int num_sms) {
  const int64_t need = (items + per_block - 1) / per_block;
  const int64_t cap = static_cast<int64_t>(num_sms) * 8;
  return static_cast<int>(need < cap ? (need > 0 ? need : 1) : cap);
}

gemm::Problem mlp_gemm1(const void* A, int64_t rows, int H, const void* w1, int64_t w1_rows,
                        const int32_t* offsets, int groups, int I, void* h) {
  gemm::Problem p{};
  p.A = A;
  p.a_rows = rows;
  p.K = H;
  p.B = w1;
  p.b_rows = w1_rows;
  p.offsets = offsets;
  p.groups = groups;
  p.n_tiles = (I + 127) / 128;
  p.seg_cols = I;
  p.b_rows_per_group = 2 * I;
  p.b_tile_stride = 128;
  p.b_half1_off = I;
  p.weight_group_mod = groups;
  p.out = h;
  p.ldo = I;
  p.epilogue = gemm::kSwiGLU;
  p.out_row_map = nullptr;
  return p;
}

gemm::Problem mlp_gemm2(const void* h, int64_t rows, int I, const void* w2, int64_t w2_rows,
                        const int32_t* offsets, int groups, int H, void* out,
                        const int32_t* row_map) {
  gemm::Problem p{};
  p.A = h;
  p.a_rows = rows;
  p.K = I;
  p.B = w2;
  p.b_rows = w2_rows;
  p.offsets = offsets;
  p.groups = groups;
  p.n_tiles = (H + 255) / 256;
  p.seg_cols = H;
  p.b_rows_per_group = H;
  p.b_tile_stride = 256;
  p.b_half1_off = 128;
  p.weight_group_mod = groups;
  p.out = out;
  p.ldo = H;
  p.epilogue = gemm::kPlain;
  p.out_row_map = row_map;
  return p;
}

}  // namespace
}  // namespace ds

using ds::fail;

extern "C" {

size_t ds_moe_route_dispatch_workspace_size(int num_tokens, int num_experts, int top_k) {
  ds::Carve c(nullptr, 0);
  const size_t nblk = static_cast<size_t>(ds::route_blocks(num_tokens));
  c.take<int32_t>(nblk * num_experts);                       // hist
  c.take<int32_t>(nblk * num_experts);                       // base
  c.take<int32_t>(static_cast<size_t>(num_tokens) * top_k);  // rank
  return ds::align_up(c.used, 256);
}

int ds_moe_route_dispatch(const float* router_logits, const void* x_bf16, int num_tokens,
                          int hidden_size, int num_experts, int top_k, int32_t* topk_indices,
                          float* topk_weights, int32_t* expert_offsets, int32_t* slot_of,
                          int32_t* token_map, void* dispatched_bf16, void* workspace,
                          size_t workspace_bytes, void* stream) {
  const int T = num_tokens, H = hidden_size, E = num_experts, K = top_k;
  DS_REQUIRE(T >= 0 && H > 0 && H % 8 == 0, "route_dispatch: bad shape");
  DS_REQUIRE(E >= 1 && E <= ds::kMaxExperts, "route_dispatch: num_experts must be in [1, 64]");
  DS_REQUIRE(K >= 1 && K <= ds::kMaxTopK && K <= E, "route_dispatch: bad top_k");
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (T == 0) {
    if (expert_offsets) DS_CUDA(cudaMemsetAsync(expert_offsets, 0, sizeof(int32_t) * (E + 1), s));
    return DS_OK;
  }
  DS_REQUIRE(router_logits && x_bf16 && topk_indices && topk_weights && expert_offsets && slot_of &&
                 token_map && dispatched_bf16,
             "route_dispatch: null pointer");
  DS_REQUIRE(ds::aligned16(x_bf16) && ds::aligned16(dispatched_bf16),
             "route_dispatch: x/dispatched must be 16-byte aligned");
  const int nblk = ds::route_blocks(T);
  ds::Carve c(workspace, workspace_bytes);
  int32_t* hist = c.take<int32_t>(static_cast<size_t>(nblk) * E);
  int32_t* base = c.take<int32_t>(static_cast<size_t>(nblk) * E);
  int32_t* rank = c.take<int32_t>(static_cast<size_t>(T) * K);
  if (!c.ok()) return fail(DS_ERR_WORKSPACE, "route_dispatch: workspace needs %zu bytes", c.used);
  DS_TRY(ds::launch_route(router_logits, T, E, K, topk_indices, topk_weights, nullptr, hist, rank, s));
  DS_TRY(ds::launch_plan(hist, nblk, E, nullptr, nullptr, expert_offsets, base, s));
  return ds::launch_scatter(x_bf16, T, H, E, K, topk_indices, topk_weights, base, rank,
                            dispatched_bf16, token_map, nullptr, slot_of, T * K, s);
}

int ds_moe_expert_mlp(const void* rows_bf16, int num_rows, const int32_t* group_offsets,
                      int num_groups, const void* packed_w1_bf16, const void* w2_bf16,
                      int hidden_size, int intermediate_size, void* h_bf16, void* out_bf16,
                      const int32_t* out_row_map, int max_ctas, void* stream) {
  const int H = hidden_size, I = intermediate_size;
  DS_REQUIRE(num_rows >= 0 && num_groups >= 1, "expert_mlp: bad shape");
  DS_REQUIRE(H > 0 && I > 0 && H % 8 == 0 && I % 8 == 0,
             "expert_mlp: hidden_size and intermediate_size must be positive multiples of 8");
  if (num_rows == 0) return DS_OK;
  DS_REQUIRE(rows_bf16 && group_offsets && packed_w1_bf16 && w2_bf16 && h_bf16 && out_bf16,
             "expert_mlp: null pointer");
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  ds::gemm::Problem g1 = ds::mlp_gemm1(rows_bf16, num_rows, H, packed_w1_bf16,
                                       static_cast<int64_t>(num_groups) * 2 * I, group_offsets,
                                       num_groups, I, h_bf16);
  ds::gemm::Problem g2 = ds::mlp_gemm2(h_bf16, num_rows, I, w2_bf16,
                                       static_cast<int64_t>(num_groups) * H, group_offsets,
                                       num_groups, H, out_bf16, out_row_map);
  g1.max_ctas = g2.max_ctas = max_ctas;
  DS_TRY(ds::gemm::launch(g1, s));
  return ds::gemm::launch(g2, s);
}

int ds_dense_mlp(const void* x_bf16, int num_rows, const void* w1_bf16, const void* w2_bf16,
                 int hidden_size, int intermediate_size, void* h_bf16, void* out_bf16,
                 int max_ctas, void* stream) {
  const int H = hidden_size, I = intermediate_size;
  DS_REQUIRE(num_rows >= 0, "dense_mlp: bad shape");
  DS_REQUIRE(H > 0 && I > 0 && H % 8 == 0 && I % 8 == 0,
             "dense_mlp: hidden_size and intermediate_size must be positive multiples of 8");
  if (num_rows == 0) return DS_OK;
  DS_REQUIRE(x_bf16 && w1_bf16 && w2_bf16 && h_bf16 && out_bf16, "dense_mlp: null pointer");
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  ds::gemm::Problem g1 = ds::mlp_gemm1(x_bf16, num_rows, H, w1_bf16, 2 * static_cast<int64_t>(I),
                                       nullptr, 1, I, h_bf16);
  ds::gemm::Problem g2 = ds::mlp_gemm2(h_bf16, num_rows, I, w2_bf16, H, nullptr, 1, H, out_bf16,
                                       nullptr);
  g1.max_ctas = g2.max_ctas = max_ctas;
  DS_TRY(ds::gemm::launch(g1, s));
  return ds::gemm::launch(g2, s);
}

size_t ds_dense_mlp_workspace_size(int num_rows, int hidden_size, int intermediate_size) {
  ds::DeviceInfo di;
  if (ds::device_info(&di) != DS_OK || num_rows <= 0) return 0;
  const int H = hidden_size, I = intermediate_size;
  ds::gemm::Problem g1 = ds::mlp_gemm1(nullptr, num_rows, H, nullptr, 2 * static_cast<int64_t>(I),
                                       nullptr, 1, I, nullptr);
  ds::gemm::Problem g2 = ds::mlp_gemm2(nullptr, num_rows, I, nullptr, H, nullptr, 1, H, nullptr,
                                       nullptr);
  const size_t p1 = ds::gemm::partial_bytes(g1, ds::gemm::choose_k_splits(g1, di.num_sms));
  const size_t p2 = ds::gemm::partial_bytes(g2, ds::gemm::choose_k_splits(g2, di.num_sms));
  return ds::align_up(p1 > p2 ? p1 : p2, 256);
}

int ds_dense_mlp_ws(const void* x_bf16, int num_rows, const void* w1_bf16, const void* w2_bf16,
                    int hidden_size, int intermediate_size, void* h_bf16, void* out_bf16,
                    void* workspace, size_t workspace_bytes, void* stream) {
  const int H = hidden_size, I = intermediate_size;
  DS_REQUIRE(num_rows >= 0, "dense_mlp: bad shape");
  DS_REQUIRE(H > 0 && I > 0 && H % 8 == 0 && I % 8 == 0,
             "dense_mlp: hidden_size and intermediate_size must be positive multiples of 8");
  if (num_rows == 0) return DS_OK;
  DS_REQUIRE(x_bf16 && w1_bf16 && w2_bf16 && h_bf16 && out_bf16, "dense_mlp: null pointer");
  DS_REQUIRE(workspace_bytes >= ds_dense_mlp_workspace_size(num_rows, H, I),
             "dense_mlp: workspace needs %zu bytes", ds_dense_mlp_workspace_size(num_rows, H, I));
  ds::DeviceInfo di;
  DS_TRY(ds::device_info(&di));
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  ds::gemm::Problem g1 = ds::mlp_gemm1(x_bf16, num_rows, H, w1_bf16, 2 * static_cast<int64_t>(I),
                                       nullptr, 1, I, h_bf16);
  ds::gemm::Problem g2 = ds::mlp_gemm2(h_bf16, num_rows, I, w2_bf16, H, nullptr, 1, H, out_bf16,
                                       nullptr);
  g1.k_splits = ds::gemm::choose_k_splits(g1, di.num_sms);
  g2.k_splits = ds::gemm::choose_k_splits(g2, di.num_sms);
  g1.partial = g2.partial = static_cast<float*>(workspace);
  DS_TRY(ds::gemm::launch(g1, s));
  return ds::gemm::launch(g2, s);
}

int ds_dense_gemm1_swiglu(const void* x_bf16, int num_rows, const void* w1_bf16,
                          int hidden_size, int intermediate_size, void* h_bf16, int max_ctas,
                          void* stream) {
  DS_REQUIRE(num_rows >= 0 && hidden_size > 0 && hidden_size % 8 == 0 &&
                 intermediate_size % 8 == 0 && intermediate_size > 0,
             "dense_gemm1_swiglu: bad shape");
  if (num_rows == 0) return DS_OK;
  DS_REQUIRE(x_bf16 && w1_bf16 && h_bf16, "dense_gemm1_swiglu: null pointer");
  ds::gemm::Problem g = ds::mlp_gemm1(x_bf16, num_rows, hidden_size, w1_bf16,
                                      2 * static_cast<int64_t>(intermediate_size), nullptr, 1,
                                      intermediate_size, h_bf16);
  g.max_ctas = max_ctas;
  return ds::gemm::launch(g, static_cast<cudaStream_t>(stream));
}

int ds_dense_gemm2(const void* h_bf16, int num_rows, const void* w2_bf16, int intermediate_size,
                   int hidden_size, void* out_bf16, int max_ctas, void* stream) {
  DS_REQUIRE(num_rows >= 0 && intermediate_size > 0 && intermediate_size % 8 == 0 &&
                 hidden_size % 8 == 0 && hidden_size > 0,
             "dense_gemm2: bad shape");
  if (num_rows == 0) return DS_OK;
  DS_REQUIRE(h_bf16 && w2_bf16 && out_bf16, "dense_gemm2: null pointer");
  ds::gemm::Problem g = ds::mlp_gemm2(h_bf16, num_rows, intermediate_size, w2_bf16, hidden_size,
                                      nullptr, 1, hidden_size, out_bf16, nullptr);
  g.max_ctas = max_ctas;
  return ds::gemm::launch(g, static_cast<cudaStream_t>(stream));
}

int ds_moe_combine_slots(const void* expert_out_bf16, const int32_t* slot_of,
                         const float* topk_weights, int top_k, const void* shared_out_bf16,
                         void* out_bf16, int num_tokens, int hidden_size, void* stream) {
  DS_REQUIRE(num_tokens >= 0 && hidden_size > 0 && hidden_size % 8 == 0,
             "combine_slots: bad shape");
  DS_REQUIRE(top_k >= 1 && top_k <= ds::kMaxTopK, "combine_slots: bad top_k");
  if (num_tokens == 0) return DS_OK;
  DS_REQUIRE(expert_out_bf16 && slot_of && topk_weights && out_bf16, "combine_slots: null pointer");
  return ds::launch_combine_gather(expert_out_bf16, slot_of, topk_weights, top_k, shared_out_bf16,
                                   out_bf16, num_tokens, hidden_size,
                                   static_cast<cudaStream_t>(stream));
}

int ds_router_weight_split(const float* gate_weight, int num_experts, int hidden_size,
                           void* w_split_bf16, void* stream) {
  DS_REQUIRE(num_experts >= 1 && num_experts <= 64 && hidden_size > 0 && hidden_size % 8 == 0,
             "router_weight_split: num_experts in [1, 64], hidden_size %% 8 == 0");
  DS_REQUIRE(gate_weight && w_split_bf16, "router_weight_split: null pointer");
  ds::DeviceInfo di;
  DS_TRY(ds::device_info(&di));
  ds::router_split_kernel<<<ds::grid_cap(256LL * hidden_size, 256, di.num_sms), 256, 0,
                            static_cast<cudaStream_t>(stream)>>>(
      gate_weight, num_experts, hidden_size, static_cast<__nv_bfloat16*>(w_split_bf16));
  DS_LAUNCH_CHECK("router_split_kernel");
  return DS_OK;
}

size_t ds_moe_router_workspace_size(int num_tokens) {
  return ds::align_up(sizeof(float) * ds::kRouterSplits * static_cast<size_t>(num_tokens) *
                          ds::kRouterPartCols,
                      256);
}

int ds_moe_router(const void* x_bf16, const void* w_split_bf16, int num_tokens, int hidden_size,
                  int num_experts, int top_k, int32_t* topk_indices, float* topk_weights,
                  float* logits_out, void* workspace, size_t workspace_bytes, void* stream) {
  DS_REQUIRE(num_tokens >= 0 && hidden_size > 0 && hidden_size % 8 == 0, "moe_router: bad shape");
  DS_REQUIRE(num_experts >= 1 && num_experts <= 64, "moe_router: num_experts must be in [1, 64]");
  DS_REQUIRE(top_k >= 1 && top_k <= 8 && top_k <= num_experts, "moe_router: bad top_k");
  if (num_tokens == 0) return DS_OK;
  DS_REQUIRE(x_bf16 && w_split_bf16 && topk_indices && topk_weights, "moe_router: null pointer");
  if (workspace == nullptr || workspace_bytes < ds_moe_router_workspace_size(num_tokens))
    return fail(DS_ERR_WORKSPACE, "moe_router: workspace needs %zu bytes",
                ds_moe_router_workspace_size(num_tokens));
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  float* part = static_cast<float*>(workspace);
  ds::gemm::Problem p{};
  p.A = x_bf16;
  p.a_rows = num_tokens;
  p.K = hidden_size;
  p.B = w_split_bf16;
  p.b_rows = 256;
  p.offsets = nullptr;
  p.groups = 1;
  p.n_tiles = ds::router_splits(hidden_size);
  p.b_rows_per_group = 256;
  p.b_tile_stride = 0;
  p.b_half1_off = 128;
  p.weight_group_mod = 1;
  p.out = nullptr;
  p.ldo = 8;
  p.epilogue = ds::gemm::kRouter;
  p.logits_out = part;
  DS_TRY(ds::gemm::launch(p, s));
  return ds::launch_route_partials(part, p.n_tiles, num_tokens, num_experts, top_k,
                                   logits_out, topk_indices, topk_weights, nullptr, nullptr,
                                   nullptr, s);
}

int ds_moe_dispatch_routed(const int32_t* topk_indices, const float* topk_weights,
                           const void* x_bf16, int num_tokens, int hidden_size, int num_experts,
                           int top_k, int32_t* expert_offsets, int32_t* slot_of,
                           int32_t* token_map, void* dispatched_bf16, void* workspace,
                           size_t workspace_bytes, void* stream) {
  const int T = num_tokens, H = hidden_size, E = num_experts, K = top_k;
  DS_REQUIRE(T >= 0 && H > 0 && H % 8 == 0, "dispatch_routed: bad shape");
  DS_REQUIRE(E >= 1 && E <= ds::kMaxExperts, "dispatch_routed: num_experts must be in [1, 64]");
  DS_REQUIRE(K >= 1 && K <= ds::kMaxTopK && K <= E, "dispatch_routed: bad top_k");
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (T == 0) {
    if (expert_offsets) DS_CUDA(cudaMemsetAsync(expert_offsets, 0, sizeof(int32_t) * (E + 1), s));
    return DS_OK;
  }
  DS_REQUIRE(topk_indices && topk_weights && x_bf16 && expert_offsets && slot_of && token_map &&
                 dispatched_bf16,
             "dispatch_routed: null pointer");
  DS_REQUIRE(ds::aligned16(x_bf16) && ds::aligned16(dispatched_bf16),
             "dispatch_routed: x/dispatched must be 16-byte aligned");
  const int nblk = ds::route_blocks(T);
  ds::Carve c(workspace, workspace_bytes);
  int32_t* hist = c.take<int32_t>(static_cast<size_t>(nblk) * E);
  int32_t* base = c.take<int32_t>(static_cast<size_t>(nblk) * E);
  int32_t* rank = c.take<int32_t>(static_cast<size_t>(T) * K);
  if (!c.ok()) return fail(DS_ERR_WORKSPACE, "dispatch_routed: workspace needs %zu bytes", c.used);
  DS_TRY(ds::launch_rank(topk_indices, T, E, K, hist, rank, s));
  DS_TRY(ds::launch_plan(hist, nblk, E, nullptr, nullptr, expert_offsets, base, s));
  return ds::launch_scatter(x_bf16, T, H, E, K, topk_indices, topk_weights, base, rank,
                            dispatched_bf16, token_map, nullptr, slot_of, T * K, s);
}

size_t ds_ep_plan_workspace_size(int num_ranks, int local_experts) {
  return ds::align_up(2 * sizeof(int32_t) * static_cast<size_t>(num_ranks) * local_experts, 256);
}

int ds_ep_plan(const int32_t* recv_counts, int num_ranks, int local_experts, int recv_rows,
               int32_t* expert_offsets, int32_t* row_map, void* workspace,
               size_t workspace_bytes, void* stream) {
  const int N = num_ranks, El = local_experts;
  DS_REQUIRE(N >= 1 && El >= 1 && N * El <= 4096 && recv_rows >= 0, "ep_plan: bad shape");
  DS_REQUIRE(recv_counts && expert_offsets, "ep_plan: null pointer");
  ds::Carve c(workspace, workspace_bytes);
  int32_t* seg_src = c.take<int32_t>(static_cast<size_t>(N) * El);
  int32_t* seg_exp = c.take<int32_t>(static_cast<size_t>(N) * El);
  if (!c.ok()) return fail(DS_ERR_WORKSPACE, "ep_plan: workspace needs %zu bytes", c.used);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  ds::ep_offsets_kernel<<<1, 32, 0, s>>>(recv_counts, N, El, expert_offsets, seg_src, seg_exp);
  DS_LAUNCH_CHECK("ep_offsets_kernel");
  if (recv_rows == 0) return DS_OK;
  DS_REQUIRE(row_map != nullptr, "ep_plan: null row_map");
  ds::DeviceInfo di;
  DS_TRY(ds::device_info(&di));
  const int segs = N * El;
  ds::ep_rowmap_kernel<<<ds::grid_cap(recv_rows, 256, di.num_sms), 256,
                         2 * (segs + 1) * sizeof(int32_t), s>>>(recv_counts, seg_src, seg_exp, segs,
                                                                recv_rows, row_map);
  DS_LAUNCH_CHECK("ep_rowmap_kernel");
  return DS_OK;
}

int ds_gather_rows(const void* src_bf16, const int32_t* row_map, int num_rows, int hidden_size,
                   void* dst_bf16, void* stream) {
  DS_REQUIRE(num_rows >= 0 && hidden_size > 0 && hidden_size % 8 == 0, "gather_rows: bad shape");
  if (num_rows == 0) return DS_OK;
  DS_REQUIRE(src_bf16 && row_map && dst_bf16, "gather_rows: null pointer");
  DS_REQUIRE(ds::aligned16(src_bf16) && ds::aligned16(dst_bf16), "gather_rows: misaligned");
  ds::DeviceInfo di;
  DS_TRY(ds::device_info(&di));
  ds::gather_rows_kernel<<<ds::grid_cap(num_rows, 8, di.num_sms), 256, 0,
                           static_cast<cudaStream_t>(stream)>>>(
      static_cast<const uint4*>(src_bf16), row_map, num_rows, hidden_size / 8,
      static_cast<uint4*>(dst_bf16));
  DS_LAUNCH_CHECK("gather_rows_kernel");
  return DS_OK;
}

}  // extern "C"
