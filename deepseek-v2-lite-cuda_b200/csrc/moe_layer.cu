// Fused DeepSeek-V2-Lite MoE layer: routing -> plan -> dispatch -> grouped GEMM1+SwiGLU ->
// grouped GEMM2 -> (shared expert GEMMs) -> combine, all on one stream with no host
// synchronisation.  Mirrors the pipeline of src/kernels/moe_fused.py:118-154 and adds the
// shared expert of src/reference/moe.py:72-74,106-107.
#include "kernels.cuh"

namespace ds {
namespace {

struct LayerBuffers {
  int32_t* idx;
  float* w;
  int32_t* blk_hist;
  int32_t* local_rank;
  int32_t* offsets;
  int32_t* blk_base;
  int32_t* token_map;
  int32_t* slot_of;
  void* dispatched;  // bf16 [S, H]
  void* h;           // bf16 [S, I]
  void* eo;          // bf16 [S, H]
  void* sh;          // bf16 [T, Is]
  void* so;          // bf16 [T, H]
  float* router_part;  // f32 [kRouterSplits, T, 192] router GEMM partials (layer from x)
};

size_t carve_layer(Carve& c, LayerBuffers* b, int T, int H, int E, int K, int I, int Is) {
  const size_t S = static_cast<size_t>(T) * K;
  const size_t nblk = static_cast<size_t>(route_blocks(T));
  LayerBuffers x{};
  x.idx = c.take<int32_t>(S);
  x.w = c.take<float>(S);
  x.blk_hist = c.take<int32_t>(nblk * E);
  x.local_rank = c.take<int32_t>(S);
  x.offsets = c.take<int32_t>(E + 1);
  x.blk_base = c.take<int32_t>(nblk * E);
  x.token_map = c.take<int32_t>(S);
  x.slot_of = c.take<int32_t>(S);
  x.dispatched = c.take<__nv_bfloat16>(S * H);
  x.h = c.take<__nv_bfloat16>(S * I);
  x.eo = c.take<__nv_bfloat16>(S * H);
  x.sh = c.take<__nv_bfloat16>(Is > 0 ? static_cast<size_t>(T) * Is : 0);
  x.so = c.take<__nv_bfloat16>(Is > 0 ? static_cast<size_t>(T) * H : 0);
  x.router_part = c.take<float>(static_cast<size_t>(kRouterSplits) * T * kRouterPartCols);
  if (b) *b = x;
  return align_up(c.used, 256);
}

}  // namespace
}  // namespace ds

using ds::fail;

extern "C" size_t ds_moe_layer_workspace_size(int num_tokens, int hidden_size, int num_experts,
                                              int top_k, int intermediate_size,
                                              int shared_intermediate_size) {
  ds::Carve c(nullptr, 0);
  return ds::carve_layer(c, nullptr, num_tokens, hidden_size, num_experts, top_k,
                         intermediate_size, shared_intermediate_size);
}

extern "C" int ds_moe_layer_workspace_routing(int num_tokens, int hidden_size, int num_experts,
                                              int top_k, int intermediate_size,
                                              int shared_intermediate_size, size_t* idx_offset,
                                              size_t* weights_offset, size_t* slot_of_offset) {
  DS_REQUIRE(num_tokens >= 0 && top_k >= 1, "moe_layer_workspace_routing: bad shape");
  DS_REQUIRE(idx_offset && weights_offset && slot_of_offset,
             "moe_layer_workspace_routing: null pointer");
  ds::Carve c(reinterpret_cast<void*>(uintptr_t{256}), ~size_t{0} >> 1);
  ds::LayerBuffers b;
  ds::carve_layer(c, &b, num_tokens, hidden_size, num_experts, top_k, intermediate_size,
                  shared_intermediate_size);
  const uintptr_t base = 256;
  *idx_offset = reinterpret_cast<uintptr_t>(b.idx) - base;
  *weights_offset = reinterpret_cast<uintptr_t>(b.w) - base;
  *slot_of_offset = reinterpret_cast<uintptr_t>(b.slot_of) - base;
  return DS_OK;
}

namespace {

// One implementation for both entry points: routing from given f32 logits, or from x via the
// router GEMM (tcgen05, split f32 gate) whose epilogue does the top-k.
int layer_impl(const float* router_logits, const void* router_w_split, float* logits_out,
               const void* x_bf16, const void* packed_w1_bf16, const void* w2_bf16,
               const void* shared_w1_bf16, const void* shared_w2_bf16, void* out_bf16,
               int num_tokens, int hidden_size, int num_experts, int top_k,
               int intermediate_size, int shared_intermediate_size, void* workspace,
               size_t workspace_bytes, void** events, void* stream) {
  const int T = num_tokens, H = hidden_size, E = num_experts, K = top_k;
  const int I = intermediate_size;
  const bool has_shared = shared_w1_bf16 != nullptr && shared_w2_bf16 != nullptr;
  const int Is = has_shared ? shared_intermediate_size : 0;
  DS_REQUIRE(T >= 0, "moe_layer: num_tokens must be >= 0");
  DS_REQUIRE(E >= 1 && E <= ds::kMaxExperts, "moe_layer: num_experts must be in [1, 64]");
  DS_REQUIRE(K >= 1 && K <= ds::kMaxTopK && K <= E, "moe_layer: bad top_k");
  DS_REQUIRE(H > 0 && H % 8 == 0, "moe_layer: hidden_size must be a positive multiple of 8");
  DS_REQUIRE(I > 0 && I % 8 == 0, "moe_layer: intermediate_size must be a positive multiple of 8");
  DS_REQUIRE(!has_shared || (Is % 8 == 0 && Is > 0),
             "moe_layer: shared intermediate size must be a positive multiple of 8");
  DS_REQUIRE((shared_w1_bf16 == nullptr) == (shared_w2_bf16 == nullptr),
             "moe_layer: give both shared expert weights or neither");
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  auto mark = [&](int i) -> int {
    if (events != nullptr && events[i] != nullptr)
      DS_CUDA(cudaEventRecord(static_cast<cudaEvent_t>(events[i]), s));
    return DS_OK;
  };
  if (T == 0) return DS_OK;
  DS_REQUIRE((router_logits || router_w_split) && x_bf16 && packed_w1_bf16 && w2_bf16 && out_bf16,
             "moe_layer: null pointer");
  ds::Carve c(workspace, workspace_bytes);
  ds::LayerBuffers b;
  ds::carve_layer(c, &b, T, H, E, K, I, Is);
  if (!c.ok()) return fail(DS_ERR_WORKSPACE, "moe_layer: workspace needs %zu bytes", c.used);
  const int S = T * K;
  const int nblk = ds::route_blocks(T);

  DS_TRY(mark(0));
  if (router_w_split != nullptr) {
    ds::gemm::Problem r{};
    r.A = x_bf16;
    r.a_rows = T;
    r.K = H;
    r.B = router_w_split;
    r.b_rows = 256;
    r.offsets = nullptr;
    r.groups = 1;
    r.n_tiles = ds::router_splits(H);
    r.b_rows_per_group = 256;
    r.b_tile_stride = 0;
    r.b_half1_off = 128;
    r.weight_group_mod = 1;
    r.out = nullptr;
    r.ldo = 8;
    r.epilogue = ds::gemm::kRouter;
    r.logits_out = b.router_part;
    DS_TRY(ds::gemm::launch(r, s));
    DS_TRY(ds::launch_route_partials(b.router_part, r.n_tiles, T, E, K, logits_out, b.idx,
                                     b.w, nullptr, b.blk_hist, b.local_rank, s));
  } else {
    DS_TRY(ds::launch_route(router_logits, T, E, K, b.idx, b.w, nullptr, b.blk_hist, b.local_rank, s));
  }
  DS_TRY(mark(1));
  DS_TRY(ds::launch_plan(b.blk_hist, nblk, E, nullptr, nullptr, b.offsets, b.blk_base, s));
  DS_TRY(mark(2));
  DS_TRY(ds::launch_scatter(x_bf16, T, H, E, K, b.idx, b.w, b.blk_base, b.local_rank,
                            b.dispatched, b.token_map, nullptr, b.slot_of, S, s));
  DS_TRY(mark(3));

  // GEMM1 (+ SwiGLU) of the routed experts and of the shared expert in one persistent launch,
  // then GEMM2 of both (the shared expert's long-K tiles first, so the short routed tiles
  // fill the end of the launch).
  ds::gemm::Problem g1{};
  g1.A = b.dispatched;
  g1.a_rows = S;
  g1.K = H;
  g1.B = packed_w1_bf16;
  g1.b_rows = static_cast<int64_t>(E) * 2 * I;
  g1.offsets = b.offsets;
  g1.groups = E;
  g1.n_tiles = (I + 127) / 128;
  g1.seg_cols = I;
  g1.b_rows_per_group = 2 * I;
  g1.b_tile_stride = 128;
  g1.b_half1_off = I;
  g1.weight_group_mod = E;
  g1.out = b.h;
  g1.ldo = I;
  g1.epilogue = ds::gemm::kSwiGLU;

  ds::gemm::Problem s1{};
  if (has_shared) {
    s1.A = x_bf16;
    s1.a_rows = T;
    s1.K = H;
    s1.B = shared_w1_bf16;
    s1.b_rows = 2 * static_cast<int64_t>(Is);
    s1.offsets = nullptr;
    s1.groups = 1;
    s1.n_tiles = (Is + 127) / 128;
    s1.seg_cols = Is;
    s1.b_rows_per_group = 2 * Is;
    s1.b_tile_stride = 128;
    s1.b_half1_off = Is;
    s1.weight_group_mod = 1;
    s1.out = b.sh;
    s1.ldo = Is;
    s1.epilogue = ds::gemm::kSwiGLU;
  }
  {
    const ds::gemm::Problem* probs[2] = {&g1, has_shared ? &s1 : nullptr};
    DS_TRY(ds::gemm::launch_multi(probs, 2, s));
  }
  DS_TRY(mark(4));

  ds::gemm::Problem g2{};
  g2.A = b.h;
  g2.a_rows = S;
  g2.K = I;
  g2.B = w2_bf16;
  g2.b_rows = static_cast<int64_t>(E) * H;
  g2.offsets = b.offsets;
  g2.groups = E;
  g2.n_tiles = (H + 255) / 256;
  g2.seg_cols = H;
  g2.b_rows_per_group = H;
  g2.b_tile_stride = 256;
  g2.b_half1_off = 128;
  g2.weight_group_mod = E;
  g2.out = b.eo;
  g2.ldo = H;
  g2.epilogue = ds::gemm::kPlain;

  ds::gemm::Problem s2{};
  if (has_shared) {
    s2.A = b.sh;
    s2.a_rows = T;
    s2.K = Is;
    s2.B = shared_w2_bf16;
    s2.b_rows = H;
    s2.offsets = nullptr;
    s2.groups = 1;
    s2.n_tiles = (H + 255) / 256;
    s2.seg_cols = H;
    s2.b_rows_per_group = H;
    s2.b_tile_stride = 256;
    s2.b_half1_off = 128;
    s2.weight_group_mod = 1;
    s2.out = b.so;
    s2.ldo = H;
    s2.epilogue = ds::gemm::kPlain;
  }
  {
    const ds::gemm::Problem* probs[2] = {has_shared ? &s2 : &g2, has_shared ? &g2 : nullptr};
    DS_TRY(ds::gemm::launch_multi(probs, 2, s));
  }
  DS_TRY(mark(5));
  DS_TRY(mark(6));  // the shared expert now runs inside the two launches above
  DS_TRY(mark(7));
  DS_TRY(ds::launch_combine_gather(b.eo, b.slot_of, b.w, K, has_shared ? b.so : nullptr, out_bf16,
                                   T, H, s));
  DS_TRY(mark(8));
  return DS_OK;
}

}  // namespace

extern "C" {

int ds_moe_layer_forward(const float* router_logits, const void* x_bf16,
                         const void* packed_w1_bf16, const void* w2_bf16,
                         const void* shared_w1_bf16, const void* shared_w2_bf16,
                         void* out_bf16, int num_tokens, int hidden_size, int num_experts,
                         int top_k, int intermediate_size, int shared_intermediate_size,
                         void* workspace, size_t workspace_bytes, void** events,
                         void* stream) {
  return layer_impl(router_logits, nullptr, nullptr, x_bf16, packed_w1_bf16, w2_bf16,
                    shared_w1_bf16, shared_w2_bf16, out_bf16, num_tokens, hidden_size,
                    num_experts, top_k, intermediate_size, shared_intermediate_size, workspace,
                    workspace_bytes, events, stream);
}

int ds_moe_layer_forward_from_x(const void* x_bf16, const void* router_w_split_bf16,
                                float* logits_out, const void* packed_w1_bf16,
                                const void* w2_bf16, const void* shared_w1_bf16,
                                const void* shared_w2_bf16, void* out_bf16, int num_tokens,
                                int hidden_size, int num_experts, int top_k,
                                int intermediate_size, int shared_intermediate_size,
                                void* workspace, size_t workspace_bytes, void** events,
                                void* stream) {
  if (router_w_split_bf16 == nullptr)
    return fail(DS_ERR_INVALID_ARG, "moe_layer_from_x: router_w_split is null");
  return layer_impl(nullptr, router_w_split_bf16, logits_out, x_bf16, packed_w1_bf16, w2_bf16,
                    shared_w1_bf16, shared_w2_bf16, out_bf16, num_tokens, hidden_size,
                    num_experts, top_k, intermediate_size, shared_intermediate_size, workspace,
                    workspace_bytes, events, stream);
}

}  // extern "C"
