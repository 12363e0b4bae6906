// Expert parallelism over NVLink peer memory: the MoE layer's token all-to-all fused into the
// kernels that produce and consume the rows.  One process per GPU; each rank allocates one
// symmetric segment (the same layout on every rank) and maps every other rank's segment
// through CUDA IPC.  Experts are partitioned contiguously: expert e lives on rank e / El with
// El = E / world.
//
//   plan    : this rank's per-expert counts go into row `rank` of every rank's count matrix;
//             a bounded wait until all rows of this forward are in (this also separates
//             consecutive forwards: no rank passes it before every rank finished the previous
//             one); then the bases this rank sends to and its own receive offsets.
//   scatter : each token row is read once and written, per selected expert, straight into the
//             owner's receive buffer (expert-major, source rank minor, ascending token within)
//             together with its return address (source rank, slot); the launch's last CTA
//             raises every rank's arrival flag.
//   GEMM1   : the shared expert's GEMM1 runs on a side stream from the start of the forward,
//             beside the routing, plan and scatter; the routed GEMM1's producer waits for
//             the arrival flag (every rank's rows are in) before its first load.
//   GEMM2   : routed tiles store each output row straight into the source rank's return
//             buffer at its slot; the launch's last CTA raises every rank's return flag.
//   combine : waits for the return flag, then gathers in ascending slot order as on one GPU.
//
// The reference is single-GPU; this is the additive expert-parallel variant of its fused
// pipeline (src/kernels/moe_fused.py:118-154), with the same per-token semantics: each
// routed expert output is the same bf16 row a single GPU computes, and the combine sums the
// K rows of a token in the same (ascending global slot) order.
#include <climits>
#include <cstring>

#include "kernels.cuh"
#include "ptx.cuh"

namespace ds {
namespace ep {

constexpr int kMaxRanks = 8;
// int offsets inside the flag block (128 B apart); the counters are this rank's own
constexpr int kFlagMeta = 0, kFlagArrive = 32, kFlagReturn = 64;
constexpr int kCounterScatter = 96, kCounterGemm2 = 112;
constexpr int kFlagInts = 128;

struct SymLayout {
  size_t flags, counts, recv_meta, recv_rows, ret_rows, total;
  int64_t cap;  // receive capacity in rows
};

SymLayout sym_layout(int max_tokens, int H, int E, int K, int world) {
  SymLayout L{};
  const int El = E / world;
  L.cap = static_cast<int64_t>(world) * max_tokens * (K < El ? K : El);
  size_t off = 0;
  auto take = [&](size_t bytes) {
    const size_t o = off;
    off = align_up(off + bytes, 256);
    return o;
  };
  L.flags = take(kFlagInts * sizeof(int));
  L.counts = take(static_cast<size_t>(world) * E * sizeof(int));
  L.recv_meta = take(static_cast<size_t>(L.cap) * sizeof(int));
  L.recv_rows = take(static_cast<size_t>(L.cap) * H * 2);
  L.ret_rows = take(static_cast<size_t>(max_tokens) * K * H * 2);
  L.total = off;
  return L;
}

// SMs the shared-expert GEMM1 leaves to the dispatch kernel it overlaps
constexpr int kDispatchSMs = 32;

struct PeerTable {
  char* base[kMaxRanks];
};

__device__ __forceinline__ int* flag_at(char* const base, size_t flags_off, int which) {
  return reinterpret_cast<int*>(base + flags_off) + which;
}

// Plan + count exchange.  One CTA of 1024 threads = 16 partitions of the routing blocks x 64
// experts (the local part is the single-GPU plan).
__global__ void __launch_bounds__(1024, 1)
    ep_plan_kernel(const int32_t* __restrict__ hist, int nblk, int E, int El, int rank,
                   int world, const __grid_constant__ PeerTable peers, size_t flags_off,
                   size_t counts_off, int target,
                   int32_t* __restrict__ offsets, int32_t* __restrict__ blk_base,
                   int32_t* __restrict__ dest_base, int32_t* __restrict__ recv_off, int64_t cap,
                   int* status, long long timeout_cycles) {
  ptx::pdl_launch_dependents();
  ptx::pdl_wait();
  constexpr int P = 1024 / kMaxExperts;
  __shared__ int part[P][kMaxExperts];
  __shared__ int pbase[P][kMaxExperts];
  __shared__ int off[kMaxExperts + 1];
  __shared__ int cnt[kMaxRanks][kMaxExperts];
  __shared__ int ok;
  const int e = threadIdx.x % kMaxExperts;
  const int p = threadIdx.x / kMaxExperts;
  const int chunk = (nblk + P - 1) / P;
  const int b0 = min(nblk, p * chunk), b1 = min(nblk, b0 + chunk);
  // up to kPlanRegs histogram entries per thread stay in registers, loads issued together
  constexpr int kPlanRegs = 16;
  const bool in_regs = chunk <= kPlanRegs;
  int hv[kPlanRegs];
  int s = 0;
  if (e < E) {
    if (in_regs) {
#pragma unroll
      for (int j = 0; j < kPlanRegs; ++j)
        hv[j] = b0 + j < b1 ? __ldg(hist + static_cast<int64_t>(b0 + j) * E + e) : 0;
#pragma unroll
      for (int j = 0; j < kPlanRegs; ++j) s += hv[j];
    } else {
      for (int b = b0; b < b1; ++b) s += __ldg(hist + static_cast<int64_t>(b) * E + e);
    }
  }
  part[p][e] = s;
  __syncthreads();
  if (threadIdx.x < E) {
    int run = 0;
    for (int q = 0; q < P; ++q) {
      pbase[q][threadIdx.x] = run;
      run += part[q][threadIdx.x];
    }
    part[0][threadIdx.x] = run;  // this rank's tokens per expert
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    int run = 0;
    for (int i = 0; i < E; ++i) {
      off[i] = run;
      run += part[0][i];
    }
    off[E] = run;
  }
  __syncthreads();
  if (threadIdx.x <= E) offsets[threadIdx.x] = off[threadIdx.x];
  if (e < E) {
    int run = off[e] + pbase[p][e];
    if (in_regs) {
#pragma unroll
      for (int j = 0; j < kPlanRegs; ++j) {
        if (b0 + j < b1) blk_base[static_cast<int64_t>(b0 + j) * E + e] = run;
        run += hv[j];
      }
    } else {
      for (int b = b0; b < b1; ++b) {
        blk_base[static_cast<int64_t>(b) * E + e] = run;
        run += __ldg(hist + static_cast<int64_t>(b) * E + e);
      }
    }
  }
  // ---- count exchange: row `rank` of every rank's matrix, then one release per rank
  if (threadIdx.x < E) {
    for (int d = 0; d < world; ++d) {
      volatile int* c = reinterpret_cast<volatile int*>(peers.base[d] + counts_off);
      c[rank * E + threadIdx.x] = part[0][threadIdx.x];
    }
  }
  __threadfence_system();
  __syncthreads();
  if (threadIdx.x == 0) {
    for (int d = 0; d < world; ++d) ptx::red_release_sys_add(flag_at(peers.base[d], flags_off, kFlagMeta), 1);
    ok = ptx::wait_flag_ge(flag_at(peers.base[rank], flags_off, kFlagMeta), target, nullptr,
                           status, timeout_cycles, DS_ERR_TIMEOUT);
  }
  __syncthreads();
  if (!ok) {  // no routed work this forward: nothing to receive, nothing is sent
    if (threadIdx.x <= El) recv_off[threadIdx.x] = 0;
    if (threadIdx.x < E) dest_base[threadIdx.x] = -1;
    return;
  }
  {
    const volatile int* mine = reinterpret_cast<const volatile int*>(peers.base[rank] + counts_off);
    for (int i = threadIdx.x; i < world * E; i += blockDim.x) cnt[i / E][i % E] = mine[i];
  }
  __syncthreads();
  if (threadIdx.x < E) {
    int col = 0, pre = 0;
    for (int r = 0; r < world; ++r) {
      if (r == rank) pre = col;
      col += cnt[r][threadIdx.x];
    }
    part[1][threadIdx.x] = col;  // rows of expert e over all ranks
    part[2][threadIdx.x] = pre;  // rows of expert e from the ranks below this one
  }
  __syncthreads();
  if (threadIdx.x < world) {  // one thread per destination rank: its expert-major layout
    const int d = threadIdx.x;
    int run = 0;
    for (int j = 0; j < El; ++j) {
      const int g = d * El + j;
      dest_base[g] = run + part[2][g];
      if (d == rank) recv_off[j] = run;
      run += part[1][g];
    }
    if (d == rank) {
      recv_off[El] = run;
      if (run > cap) {  // cannot happen while every rank keeps T <= max_tokens
        atomicOr(status, DS_ERR_WORKSPACE);
        for (int j = 0; j <= El; ++j) recv_off[j] = 0;
      }
    }
  }
}

// Fused dispatch + send: one warp per token; lanes j < K resolve the K destinations (owner
// rank, row there) and write the return metadata; the warp reads the row once and stores it
// to each destination (local or a peer's memory over NVLink).
template <int K>
__global__ void __launch_bounds__(256)
    ep_scatter_kernel(const uint4* __restrict__ x, int T, int H8, int E, int El, int rank,
                      int world, const int32_t* __restrict__ idx,
                      const int32_t* __restrict__ blk_base, const int32_t* __restrict__ local_rank,
                      const int32_t* __restrict__ offsets, const int32_t* __restrict__ dest_base,
                      int32_t* __restrict__ slot_of, const __grid_constant__ PeerTable peers,
                      size_t flags_off,
                      size_t meta_off, size_t rows_off, int64_t cap, int* status) {
  ptx::pdl_launch_dependents();
  ptx::pdl_wait();
  __shared__ uint4* rows_of[kMaxRanks];
  __shared__ int* meta_of[kMaxRanks];
  __shared__ int bail;
  if (threadIdx.x < kMaxRanks) {
    char* b = threadIdx.x < world ? peers.base[threadIdx.x] : nullptr;
    rows_of[threadIdx.x] = b ? reinterpret_cast<uint4*>(b + rows_off) : nullptr;
    meta_of[threadIdx.x] = b ? reinterpret_cast<int*>(b + meta_off) : nullptr;
  }
  if (threadIdx.x == 0) bail = *reinterpret_cast<volatile int*>(status) != 0;
  __syncthreads();
  if (bail) return;  // an exchange already failed: send nothing, signal nothing
  const int lane = threadIdx.x & 31;
  const int warps = gridDim.x * (blockDim.x >> 5);
  for (int t = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5); t < T; t += warps) {
    int my_d = -1, my_row = -1;
    if (lane < K) {
      const int64_t tk = static_cast<int64_t>(t) * K + lane;
      const int e = __ldg(idx + tk);
      int pos = -1;
      if (e >= 0 && e < E) {
        pos = __ldg(blk_base + static_cast<int64_t>(t / kRouteTokens) * E + e) +
              __ldg(local_rank + tk);
        const int d = e / El;
        const int64_t row = static_cast<int64_t>(__ldg(dest_base + e)) + (pos - __ldg(offsets + e));
        if (d < world && __ldg(dest_base + e) >= 0 && row >= 0 && row < cap) {
          my_d = d;
          my_row = static_cast<int>(row);
          meta_of[d][row] = (rank << 24) | pos;
        }
      }
      slot_of[tk] = pos;
    }
    int dd[K], rr[K];
#pragma unroll
    for (int j = 0; j < K; ++j) {
      dd[j] = __shfl_sync(0xffffffffu, my_d, j);
      rr[j] = __shfl_sync(0xffffffffu, my_row, j);
    }
    const uint4* src = x + static_cast<int64_t>(t) * H8;
    for (int c0 = 0; c0 < H8; c0 += 32 * 8) {
      uint4 v[8];
#pragma unroll
      for (int u = 0; u < 8; ++u) {
        const int c = c0 + u * 32 + lane;
        if (c < H8) v[u] = __ldg(src + c);
      }
#pragma unroll
      for (int j = 0; j < K; ++j) {
        if (dd[j] < 0) continue;
        uint4* dst = rows_of[dd[j]] + static_cast<int64_t>(rr[j]) * H8;
#pragma unroll
        for (int u = 0; u < 8; ++u) {
          const int c = c0 + u * 32 + lane;
          if (c < H8) dst[c] = v[u];
        }
      }
    }
  }
  // completion: the last CTA raises every rank's arrival flag once all rows are visible
  __threadfence_system();
  __syncthreads();
  if (threadIdx.x == 0) {
    int* counter = flag_at(peers.base[rank], flags_off, kCounterScatter);
    const int prev = atomicAdd(counter, 1);
    if (prev == static_cast<int>(gridDim.x) - 1) {
      __threadfence_system();
      if (*reinterpret_cast<volatile int*>(status) == 0)
        for (int d = 0; d < world; ++d)
          ptx::red_release_sys_add(flag_at(peers.base[d], flags_off, kFlagArrive), 1);
      atomicExch(counter, 0);
    }
  }
}

struct EPBuffers {
  int32_t* idx;
  float* w;
  int32_t* blk_hist;
  int32_t* local_rank;
  int32_t* offsets;
  int32_t* blk_base;
  int32_t* slot_of;
  int32_t* dest_base;
  int32_t* recv_off;
  float* router_part;
  void* h;   // bf16 [cap, I]
  void* sh;  // bf16 [max_tokens, Is]
  void* so;  // bf16 [max_tokens, H]
};

size_t carve_ep(Carve& c, EPBuffers* b, int Tm, int H, int E, int K, int I, int Is, int world) {
  const size_t S = static_cast<size_t>(Tm) * K;
  const size_t nblk = static_cast<size_t>(route_blocks(Tm));
  const SymLayout L = sym_layout(Tm, H, E, K, world);
  EPBuffers x{};
  x.idx = c.take<int32_t>(S);
  x.w = c.take<float>(S);
  x.blk_hist = c.take<int32_t>(nblk * E);
  x.local_rank = c.take<int32_t>(S);
  x.offsets = c.take<int32_t>(E + 1);
  x.blk_base = c.take<int32_t>(nblk * E);
  x.slot_of = c.take<int32_t>(S);
  x.dest_base = c.take<int32_t>(E);
  x.recv_off = c.take<int32_t>(E / world + 1);
  x.router_part = c.take<float>(static_cast<size_t>(kRouterSplits) * Tm * kRouterPartCols);
  x.h = c.take<__nv_bfloat16>(static_cast<size_t>(L.cap) * I);
  x.sh = c.take<__nv_bfloat16>(Is > 0 ? static_cast<size_t>(Tm) * Is : 0);
  x.so = c.take<__nv_bfloat16>(Is > 0 ? static_cast<size_t>(Tm) * H : 0);
  if (b) *b = x;
  return align_up(c.used, 256);
}

int check_shape(int Tm, int H, int E, int K, int I, int world) {
  DS_REQUIRE(world >= 1 && world <= kMaxRanks, "ep: world size must be in [1, 8]");
  DS_REQUIRE(E >= 1 && E <= kMaxExperts && E % world == 0,
             "ep: num_experts must be in [1, 64] and divisible by the world size");
  DS_REQUIRE(K >= 1 && K <= kMaxTopK && K <= E, "ep: bad top_k");
  DS_REQUIRE(Tm >= 1 && static_cast<int64_t>(Tm) * K < (1 << 24),
             "ep: max_tokens * top_k must be below 2^24");
  DS_REQUIRE(H % 256 == 0, "ep: hidden_size must be a multiple of 256");
  DS_REQUIRE(I % 128 == 0, "ep: intermediate_size must be a multiple of 128");
  return DS_OK;
}

}  // namespace ep
}  // namespace ds

using ds::fail;
namespace ep = ds::ep;

extern "C" {

int ds_ep_symmetric_size(int max_tokens, int hidden_size, int num_experts, int top_k, int world,
                         size_t* bytes) {
  DS_REQUIRE(bytes != nullptr, "ep: bytes is null");
  DS_TRY(ep::check_shape(max_tokens, hidden_size, num_experts, top_k, 128, world));
  *bytes = ep::sym_layout(max_tokens, hidden_size, num_experts, top_k, world).total;
  return DS_OK;
}

int ds_ep_alloc(size_t bytes, void** ptr) {
  DS_REQUIRE(ptr != nullptr && bytes > 0, "ep_alloc: bad arguments");
  *ptr = nullptr;
  void* p = nullptr;
  DS_CUDA(cudaMalloc(&p, bytes));
  cudaError_t e = cudaMemset(p, 0, bytes);
  if (e == cudaSuccess) e = cudaDeviceSynchronize();
  if (e != cudaSuccess) {
    cudaFree(p);
    return ds::cuda_fail(e, "ep_alloc: zero fill");
  }
  *ptr = p;
  return DS_OK;
}

int ds_ep_free(void* ptr) {
  if (ptr != nullptr) DS_CUDA(cudaFree(ptr));
  return DS_OK;
}

int ds_ep_ipc_handle(void* ptr, void* handle_out) {
  static_assert(sizeof(cudaIpcMemHandle_t) == DS_EP_IPC_HANDLE_BYTES, "IPC handle size");
  DS_REQUIRE(ptr != nullptr && handle_out != nullptr, "ep_ipc_handle: null pointer");
  cudaIpcMemHandle_t h;
  DS_CUDA(cudaIpcGetMemHandle(&h, ptr));
  memcpy(handle_out, &h, sizeof(h));
  return DS_OK;
}

int ds_ep_ipc_open(const void* handle, void** ptr) {
  DS_REQUIRE(handle != nullptr && ptr != nullptr, "ep_ipc_open: null pointer");
  *ptr = nullptr;
  cudaIpcMemHandle_t h;
  memcpy(&h, handle, sizeof(h));
  DS_CUDA(cudaIpcOpenMemHandle(ptr, h, cudaIpcMemLazyEnablePeerAccess));
  return DS_OK;
}

int ds_ep_ipc_close(void* ptr) {
  if (ptr != nullptr) DS_CUDA(cudaIpcCloseMemHandle(ptr));
  return DS_OK;
}

size_t ds_ep_layer_workspace_size(int max_tokens, int hidden_size, int num_experts, int top_k,
                                  int intermediate_size, int shared_intermediate_size,
                                  int world) {
  if (world < 1 || world > ep::kMaxRanks || num_experts % world != 0 || max_tokens < 1) return 0;
  ds::Carve c(nullptr, 0);
  return ep::carve_ep(c, nullptr, max_tokens, hidden_size, num_experts, top_k,
                      intermediate_size, shared_intermediate_size, world);
}

int ds_ep_layer_forward(const void* x_bf16, int num_tokens, const void* router_w_split_bf16,
                        float* logits_out, const void* w1_local_bf16, const void* w2_local_bf16,
                        const void* shared_w1_bf16, const void* shared_w2_bf16, void* out_bf16,
                        int hidden_size, int num_experts, int top_k, int intermediate_size,
                        int shared_intermediate_size, int rank, int world, int max_tokens,
                        void* const* sym_bases, int epoch, int timeout_ms, void* workspace,
                        size_t workspace_bytes, void** events, void* stream) {
  const int T = num_tokens, H = hidden_size, E = num_experts, K = top_k;
  const int I = intermediate_size;
  const bool has_shared = shared_w1_bf16 != nullptr && shared_w2_bf16 != nullptr;
  const int Is = has_shared ? shared_intermediate_size : 0;
  DS_TRY(ep::check_shape(max_tokens, H, E, K, I, world));
  DS_REQUIRE(rank >= 0 && rank < world, "ep: rank %d outside [0, %d)", rank, world);
  DS_REQUIRE(T >= 0 && T <= max_tokens, "ep: num_tokens=%d outside [0, max_tokens=%d]", T,
             max_tokens);
  DS_REQUIRE(epoch >= 1 && static_cast<int64_t>(epoch) * world < INT_MAX, "ep: bad epoch");
  DS_REQUIRE(timeout_ms >= 1, "ep: timeout_ms must be positive");
  DS_REQUIRE(!has_shared || (Is % 128 == 0 && Is > 0),
             "ep: shared intermediate size must be a positive multiple of 128");
  DS_REQUIRE((shared_w1_bf16 == nullptr) == (shared_w2_bf16 == nullptr),
             "ep: give both shared expert weights or neither");
  DS_REQUIRE(router_w_split_bf16 && w1_local_bf16 && w2_local_bf16 && sym_bases,
             "ep: null pointer");
  DS_REQUIRE(T == 0 || (x_bf16 && out_bf16), "ep: null token pointer");
  ep::PeerTable peers{};
  for (int r = 0; r < world; ++r) {
    DS_REQUIRE(sym_bases[r] != nullptr && (reinterpret_cast<uintptr_t>(sym_bases[r]) & 255u) == 0,
               "ep: symmetric base of rank %d is null or not 256-byte aligned", r);
    peers.base[r] = static_cast<char*>(sym_bases[r]);
  }
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  auto mark = [&](int i) -> int {
    if (events != nullptr && events[i] != nullptr)
      DS_CUDA(cudaEventRecord(static_cast<cudaEvent_t>(events[i]), s));
    return DS_OK;
  };
  ds::Carve c(workspace, workspace_bytes);
  ep::EPBuffers b;
  ep::carve_ep(c, &b, max_tokens, H, E, K, I, Is, world);
  if (!c.ok()) return fail(DS_ERR_WORKSPACE, "ep_layer: workspace needs %zu bytes", c.used);
  ds::DeviceInfo di;
  DS_TRY(ds::device_info(&di));
  int* status = ds::device_status_ptr();
  if (status == nullptr) return fail(DS_ERR_CUDA, "device status word unavailable");
  const long long timeout_cycles = static_cast<long long>(timeout_ms) * di.clock_khz;
  const ep::SymLayout L = ep::sym_layout(max_tokens, H, E, K, world);
  const int El = E / world;
  const int nblk = ds::route_blocks(T);
  const int target = epoch * world;
  char* mine = peers.base[rank];
  int* my_flags = reinterpret_cast<int*>(mine + L.flags);

  DS_TRY(mark(0));
  // the shared expert's GEMM1 (SwiGLU) needs only this rank's tokens: it runs on a side
  // stream, capped below the SM count, while the router GEMM and routing (a few CTAs at few
  // tokens per rank), the plan and the dispatch kernel (bound by NVLink, not by SMs) run on
  // the SMs it leaves; joined back before GEMM2
  const bool side = has_shared && T > 0;
  if (side) {
    ds::SideStream ss;
    DS_TRY(ds::side_stream(di.device, &ss));
    ds::gemm::Problem s1{};
    s1.A = x_bf16;
    s1.a_rows = T;
    s1.K = H;
    s1.B = shared_w1_bf16;
    s1.b_rows = 2 * static_cast<int64_t>(Is);
    s1.groups = 1;
    s1.n_tiles = Is / 128;
    s1.b_rows_per_group = 2 * Is;
    s1.b_tile_stride = 128;
    s1.b_half1_off = Is;
    s1.weight_group_mod = 1;
    s1.out = b.sh;
    s1.ldo = Is;
    s1.epilogue = ds::gemm::kSwiGLU;
    s1.max_ctas = di.num_sms > 2 * ep::kDispatchSMs ? di.num_sms - ep::kDispatchSMs : di.num_sms;
    DS_CUDA(cudaEventRecord(ss.fork, s));
    DS_CUDA(cudaStreamWaitEvent(ss.stream, ss.fork, 0));
    DS_TRY(ds::gemm::launch(s1, ss.stream));
    DS_CUDA(cudaEventRecord(ss.join, ss.stream));
  }
  if (T > 0) {
    ds::gemm::Problem r{};
    r.A = x_bf16;
    r.a_rows = T;
    r.K = H;
    r.B = router_w_split_bf16;
    r.b_rows = 256;
    r.groups = 1;
    r.n_tiles = ds::router_splits(H);
    r.b_rows_per_group = 256;
    r.b_tile_stride = 0;
    r.b_half1_off = 128;
    r.weight_group_mod = 1;
    r.ldo = 8;
    r.epilogue = ds::gemm::kRouter;
    r.logits_out = b.router_part;
    DS_TRY(ds::gemm::launch(r, s));
    DS_TRY(ds::launch_route_partials(b.router_part, r.n_tiles, T, E, K, logits_out, b.idx,
                                     b.w, nullptr, b.blk_hist, b.local_rank, s));
  }
  DS_TRY(mark(1));
  DS_CUDA(ds::launch_pdl(ep::ep_plan_kernel, dim3(1), dim3(1024), 0, s, b.blk_hist, nblk, E, El,
                         rank, world, peers, L.flags, L.counts, target, b.offsets, b.blk_base,
                         b.dest_base, b.recv_off, L.cap, status, timeout_cycles));
  DS_TRY(mark(2));
  {
    const int grid = T > 0 ? (T + 7) / 8 < 4 * di.num_sms ? (T + 7) / 8 : 4 * di.num_sms : 1;
#define DS_EP_SCATTER(KK)                                                                     \
  DS_CUDA(ds::launch_pdl(ep::ep_scatter_kernel<KK>, dim3(grid), dim3(256), 0, s,               \
                         static_cast<const uint4*>(x_bf16), T, H / 8, E, El, rank, world,     \
                         b.idx, b.blk_base, b.local_rank, b.offsets, b.dest_base, b.slot_of,  \
                         peers, L.flags, L.recv_meta, L.recv_rows, L.cap, status))
    switch (K) {
      case 1: DS_EP_SCATTER(1); break;
      case 2: DS_EP_SCATTER(2); break;
      case 3: DS_EP_SCATTER(3); break;
      case 4: DS_EP_SCATTER(4); break;
      case 5: DS_EP_SCATTER(5); break;
      case 6: DS_EP_SCATTER(6); break;
      case 7: DS_EP_SCATTER(7); break;
      default: DS_EP_SCATTER(8); break;
    }
#undef DS_EP_SCATTER
    DS_LAUNCH_CHECK("ep_scatter_kernel");
  }
  DS_TRY(mark(3));

  // GEMM1 (+ SwiGLU) of the routed rows of this rank's experts as they arrive from every rank
  ds::gemm::Problem g1{};
  g1.A = mine + L.recv_rows;
  g1.a_rows = L.cap;
  g1.K = H;
  g1.B = w1_local_bf16;
  g1.b_rows = static_cast<int64_t>(El) * 2 * I;
  g1.offsets = b.recv_off;
  g1.groups = El;
  g1.n_tiles = I / 128;
  g1.b_rows_per_group = 2 * I;
  g1.b_tile_stride = 128;
  g1.b_half1_off = I;
  g1.weight_group_mod = El;
  g1.out = b.h;
  g1.ldo = I;
  g1.epilogue = ds::gemm::kSwiGLU;
  g1.wait_flag = my_flags + ep::kFlagArrive;
  g1.wait_target = target;
  g1.wait_timeout_cycles = timeout_cycles;
  DS_TRY(ds::gemm::launch(g1, s));
  DS_TRY(mark(4));
  if (side) {
    ds::SideStream ss;
    DS_TRY(ds::side_stream(di.device, &ss));
    DS_CUDA(cudaStreamWaitEvent(s, ss.join, 0));  // the shared expert's h for GEMM2
  }

  // GEMM2: routed rows first (their outputs cross NVLink while the shared tiles run), each
  // row stored at its source rank's return slot; then the shared expert.  The launch's last
  // CTA raises every rank's return flag.
  ds::gemm::Problem g2{};
  g2.A = b.h;
  g2.a_rows = L.cap;
  g2.K = I;
  g2.B = w2_local_bf16;
  g2.b_rows = static_cast<int64_t>(El) * H;
  g2.offsets = b.recv_off;
  g2.groups = El;
  g2.n_tiles = H / 256;
  g2.b_rows_per_group = H;
  g2.b_tile_stride = 256;
  g2.b_half1_off = 128;
  g2.weight_group_mod = El;
  g2.out = mine + L.ret_rows;
  g2.ldo = H;
  g2.epilogue = ds::gemm::kPlain;
  g2.out_meta = reinterpret_cast<const int32_t*>(mine + L.recv_meta);
  for (int r = 0; r < world; ++r) g2.out_peers[r] = peers.base[r] + L.ret_rows;
  ds::gemm::Problem s2{};
  if (has_shared && T > 0) {
    s2.A = b.sh;
    s2.a_rows = T;
    s2.K = Is;
    s2.B = shared_w2_bf16;
    s2.b_rows = H;
    s2.groups = 1;
    s2.n_tiles = H / 256;
    s2.b_rows_per_group = H;
    s2.b_tile_stride = 256;
    s2.b_half1_off = 128;
    s2.weight_group_mod = 1;
    s2.out = b.so;
    s2.ldo = H;
    s2.epilogue = ds::gemm::kPlain;
  }
  {
    ds::gemm::Signal sig{};
    sig.done_counter = my_flags + ep::kCounterGemm2;
    sig.nsignal = world;
    for (int r = 0; r < world; ++r)
      sig.flags[r] = reinterpret_cast<int*>(peers.base[r] + L.flags) + ep::kFlagReturn;
    const ds::gemm::Problem* probs[2] = {&g2, (has_shared && T > 0) ? &s2 : nullptr};
    DS_TRY(ds::gemm::launch_multi(probs, 2, s, &sig));
  }
  DS_TRY(mark(5));
  DS_TRY(ds::launch_combine_gather(mine + L.ret_rows, b.slot_of, b.w, K,
                                   has_shared ? b.so : nullptr, out_bf16, T, H, s,
                                   my_flags + ep::kFlagReturn, target, timeout_cycles));
  DS_TRY(mark(6));
  return DS_OK;
}

}  // extern "C"
